"""W8A8 modes 1-3 (INT8-ConvRot, W6A8, W4A8 codebook) on a B200 against the oracle.

``QuantizedB200Backend(mode)`` replaces ``QuantizedExpertBackend(mode)``
(src/drama_low_vram/quantized_kernels.py:217-248). The integer sums are exact
and the rotation is rounded once from float64 on both sides, so most outputs
match the oracle bit for bit; the bar is the north-star 2e-2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_parity, np_f32
from oracle import restate as R

pytestmark = pytest.mark.gpu


def _device_bank(bank, device):
    from types import SimpleNamespace

    return SimpleNamespace(**{k: v.to(device) for k, v in bank.items()})


def _np(bank):
    return {k: v.numpy() for k, v in bank.items()}


@pytest.mark.parametrize("mode", [1, 2, 3])
def test_golden_case_matches_reference_and_oracle(cuda_device, mode):
    from drama_b200.backend import QuantizedB200Backend
    from golden.make_convrot_golden import inputs

    golden = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "convrot_w8a8.npz")
    bank, x, ids, w = inputs(mode)
    out = QuantizedB200Backend(mode).forward(x.to(cuda_device), ids.to(cuda_device), w.to(cuda_device),
                                             _device_bank(bank, cuda_device))
    torch.cuda.synchronize()
    ref = R.convrot_forward(np_f32(x), ids.numpy(), np_f32(w), _np(bank), mode)
    assert_parity(np_f32(out), ref, label=f"mode {mode} vs oracle")
    assert_parity(np_f32(out), golden[f"forward{mode}"], label=f"mode {mode} vs reference")
    assert (np_f32(out) == ref).mean() >= 0.95


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("tokens,top_k,experts", [(1, 8, 16), (4, 8, 16), (16, 8, 32)])
def test_drama_shape_matches_oracle(cuda_device, mode, tokens, top_k, experts):
    from drama_b200 import synthetic
    from drama_b200.backend import QuantizedB200Backend

    bank = synthetic.w8a8_bank(mode, experts, 2048, 768, seed=600 + mode)
    x = synthetic.hidden_states(tokens, 2048, 601, device=cuda_device)
    ids, w = synthetic.uniform_routes(tokens, top_k, experts, 602, device=cuda_device)
    w = w.to(torch.bfloat16)
    backend = QuantizedB200Backend(mode)
    staged = _device_bank(bank, cuda_device)
    out = backend.forward(x, ids, w, staged)
    pairs = backend.forward_pairs(x[:1].repeat(top_k, 1), ids[:1].reshape(-1, 1), w[:1].reshape(-1, 1), staged)
    torch.cuda.synchronize()
    ref = R.convrot_forward(np_f32(x), ids.cpu().numpy(), np_f32(w), _np(bank), mode)
    assert_parity(np_f32(out), ref, label=f"mode {mode} T={tokens}")
    ref_pairs = R.convrot_pairs(np.repeat(np_f32(x[:1]), top_k, 0), ids[:1].cpu().numpy().reshape(-1),
                                np_f32(w[:1]).reshape(-1), _np(bank), mode)
    assert_parity(np_f32(pairs), ref_pairs, label=f"mode {mode} pairs")


def test_out_of_range_ids_contribute_zero_and_graph_replays_bitwise(cuda_device):
    from drama_b200 import synthetic
    from drama_b200.backend import QuantizedB200Backend

    mode, experts = 2, 8
    bank = synthetic.w8a8_bank(mode, experts, 512, 256, seed=70)
    staged = _device_bank(bank, cuda_device)
    x = synthetic.hidden_states(3, 512, 71, device=cuda_device)
    ids, w = synthetic.uniform_routes(3, 4, experts, 72, device=cuda_device)
    w = w.to(torch.bfloat16)
    backend = QuantizedB200Backend(mode, validate_ids=False)
    bad = ids.clone()
    bad[1, 2] = experts + 3
    out = backend.forward(x, bad, w, staged)
    keep = bad.cpu().numpy() < experts
    ref = R.convrot_forward(np_f32(x), np.where(keep, bad.cpu().numpy(), 0), np_f32(w) * keep, _np(bank), mode)
    torch.cuda.synchronize()
    assert_parity(np_f32(out), ref, label="dropped slot")
    stream = torch.cuda.Stream(cuda_device)
    stream.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(stream):
        eager = backend.forward(x, ids, w, staged)
    torch.cuda.current_stream(cuda_device).wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        static = backend.forward(x, ids, w, staged)
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(static.view(torch.int16), eager.view(torch.int16))


@pytest.mark.parametrize("mode", [2, 3])
def test_every_relative_scale_byte(cuda_device, mode):
    """Every non-NaN FP8 E4M3 relative-scale byte (zero, subnormals, negatives, and values whose grid saturates at
    +-127) through the W6A8 f16x2 dequantisation and the W4A8 grid table (one table row per byte). The channel
    scales are powers of two that keep the projections O(1); the integer sums are exact, so a wrong grid value
    shows up as a changed output, not only as a larger error."""
    from drama_b200 import synthetic
    from drama_b200.backend import QuantizedB200Backend

    hidden, inter, experts, tokens, top_k = 512, 256, 4, 3, 2
    bank = synthetic.w8a8_bank(mode, experts, hidden, inter, seed=80 + mode)
    usable = np.array([b for b in range(256) if b & 0x7F != 0x7F], dtype=np.uint8)  # 0x7F / 0xFF are NaN
    for name, k, channel in (("w13", hidden, 2.0 ** -11), ("w2", inter, 2.0 ** -11)):
        aux = bank[f"{name}_scale_inv"].numpy()  # shares memory with the tensor
        e, n = aux.shape[:2]
        cells = np.arange(e * n * (k // 16)).reshape(e, n, k // 16)
        aux[..., :k // 16] = usable[(cells * 37 + cells // usable.size) % usable.size]
        aux[..., k // 16:k // 16 + 4] = np.frombuffer(np.float32(channel).tobytes(), dtype=np.uint8)
    assert all(np.isin(usable, bank[f"{name}_scale_inv"].numpy()[..., :k // 16]).all()
               for name, k in (("w13", hidden), ("w2", inter)))
    x = synthetic.hidden_states(tokens, hidden, 81, device=cuda_device)
    ids, w = synthetic.uniform_routes(tokens, top_k, experts, 82, device=cuda_device)
    w = w.to(torch.bfloat16)
    out = QuantizedB200Backend(mode).forward(x, ids, w, _device_bank(bank, cuda_device))
    torch.cuda.synchronize()
    ref = R.convrot_forward(np_f32(x), ids.cpu().numpy(), np_f32(w), _np(bank), mode)
    assert np.isfinite(ref).all() and 0.05 < np.abs(ref).max() < 64
    assert_parity(np_f32(out), ref, label=f"mode {mode} every relative-scale byte")
    assert (np_f32(out) == ref).mean() >= 0.9
