"""Shared expert + gate fused with the routed combine, against the oracle.

``SharedExpertB200`` replaces ``BackboneDecodeGraph._shared_impl`` and
``_post_impl`` (src/drama_low_vram/backbone_graph.py:327-337).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_parity, np_f32
from oracle import restate as R

pytestmark = pytest.mark.gpu


def _weights(hidden, inter, seed, device):
    g = torch.Generator(device="cpu").manual_seed(seed)
    def w(*shape, std):
        return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16).to(device)
    return (w(inter, hidden, std=0.03), w(inter, hidden, std=0.03), w(hidden, inter, std=0.03),
            w(1, hidden, std=0.05))


@pytest.mark.parametrize("tokens,hidden,inter", [(1, 2048, 768), (3, 2048, 512), (16, 2048, 768), (5, 256, 128)])
def test_shared_and_fused_post_match_oracle(cuda_device, tokens, hidden, inter):
    from drama_b200 import synthetic
    from drama_b200.shared import SharedExpertB200

    gp, up, dp, gw = _weights(hidden, inter, tokens + hidden, cuda_device)
    mod = SharedExpertB200(gp, up, dp, gw)
    x = synthetic.hidden_states(tokens, hidden, 11, device=cuda_device)
    routed = synthetic.hidden_states(tokens, hidden, 12, device=cuda_device) * 0.1
    # residual below 4 in magnitude: one bf16 ulp there (2^-6) stays under the 2e-2 bar, so a one-ulp
    # difference in `shared` (fp32 summation order) cannot fail the final rounding by itself
    after = synthetic.hidden_states(tokens, hidden, 13, device=cuda_device) * 0.5
    shared = mod.shared(x)
    fused = mod.post(after, routed, x)
    torch.cuda.synchronize()
    ref_shared = R.shared_expert(np_f32(x), np_f32(gp), np_f32(up), np_f32(dp), np_f32(gw))
    assert_parity(np_f32(shared), ref_shared, label=f"shared T={tokens}")
    ref_post = R.post_moe(np_f32(after), np_f32(routed), ref_shared)
    assert_parity(np_f32(fused), ref_post, label=f"post T={tokens}")
    # the fused pass equals the unfused composition of its own parts, bit for bit
    assert np.array_equal(np_f32(fused), R.post_moe(np_f32(after), np_f32(routed), np_f32(shared)))


def test_in_place_and_graph_replay(cuda_device):
    from drama_b200 import synthetic
    from drama_b200.shared import SharedExpertB200

    gp, up, dp, gw = _weights(2048, 768, 5, cuda_device)
    mod = SharedExpertB200(gp, up, dp, gw)
    x = synthetic.hidden_states(1, 2048, 21, device=cuda_device)
    routed = synthetic.hidden_states(1, 2048, 22, device=cuda_device) * 0.1
    after = synthetic.hidden_states(1, 2048, 23, device=cuda_device)
    want = mod.post(after, routed, x).clone()
    inplace = after.clone()
    mod.post(inplace, routed, x, out=inplace)
    torch.cuda.synchronize()
    assert torch.equal(inplace, want)
    stream = torch.cuda.Stream(cuda_device)
    stream.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(stream):
        mod.post(after, routed, x)
    torch.cuda.current_stream(cuda_device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        static = mod.post(after, routed, x)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(static, want)


def test_layer_chain_matches_oracle_and_replays(cuda_device):
    """Six distinct shared experts chained through the residual, as the
    decode stack calls them: one row at the reference's shape runs one
    launch per layer whose weight loads start before the previous layer has
    finished. Each layer matches the oracle applied to the previous layer's
    output, and a CUDA graph of the chain replays bit for bit."""
    from drama_b200 import synthetic
    from drama_b200.shared import SharedExpertB200

    mods, ws = [], []
    for layer in range(6):
        w = _weights(2048, 768, 100 + layer, cuda_device)
        ws.append(w)
        mods.append(SharedExpertB200(*w))
    x = synthetic.hidden_states(1, 2048, 31, device=cuda_device)
    routed = synthetic.hidden_states(1, 2048, 32, device=cuda_device) * 0.1
    h0 = synthetic.hidden_states(1, 2048, 33, device=cuda_device) * 0.5
    outs, h = [], h0
    for m in mods:
        h = m.post(h, routed, x)
        outs.append(h)
    torch.cuda.synchronize()
    prev = h0
    for layer, (gp, up, dp, gw) in enumerate(ws):
        ref = R.post_moe(np_f32(prev), np_f32(routed),
                         R.shared_expert(np_f32(x), np_f32(gp), np_f32(up), np_f32(dp), np_f32(gw)))
        assert_parity(np_f32(outs[layer]), ref, label=f"layer {layer}")
        prev = outs[layer]
    stream = torch.cuda.Stream(cuda_device)
    stream.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(stream):  # the workspace is per stream: one eager pass before capture
        g = h0
        for m in mods:
            g = m.post(g, routed, x)
    torch.cuda.current_stream(cuda_device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        g = h0
        for m in mods:
            g = m.post(g, routed, x)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(g, outs[-1])


def test_one_row_after_larger_batches(cuda_device):
    """The one-launch layer's arrival tickets share the workspace with the
    two-launch schedule of larger batches: one row after 16 and 3 rows (and
    again) still matches the oracle."""
    from drama_b200 import synthetic
    from drama_b200.shared import SharedExpertB200

    gp, up, dp, gw = _weights(2048, 768, 41, cuda_device)
    mod = SharedExpertB200(gp, up, dp, gw)
    for step, tokens in enumerate((16, 1, 3, 1, 1)):
        x = synthetic.hidden_states(tokens, 2048, 42 + step, device=cuda_device)
        out = mod.shared(x)
        torch.cuda.synchronize()
        ref = R.shared_expert(np_f32(x), np_f32(gp), np_f32(up), np_f32(dp), np_f32(gw))
        assert_parity(np_f32(out), ref, label=f"step {step} T={tokens}")
