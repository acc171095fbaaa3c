"""The fused decode layer's routing against the reference's own router arithmetic.

The reference routes a decode row in ``BackboneDecodeGraph._route_impl``
(``src/drama_low_vram/backbone_graph.py:316-323``): the upstream RMSNorm in
fp32 (eps 1e-6) cast to bf16, ``moe.gate`` as a bf16 ``F.linear`` (cuBLAS),
``softmax(logits.float())``, ``topk``, renormalisation, cast to bf16. This
test runs exactly those torch ops on the B200, one row at a time as the decode
graph does, on config-1 inputs (hidden 2048, 128 experts, top-8) for 1,024
seeded tokens through 8 layers of the synthetic stack, teacher-forced: every
layer's torch router sees the same input row as the layer kernel did.

It reports how many normalised rows and route-index lists differ, and splits
the index differences into those caused by the RMSNorm rounding and those
caused by the router GEMV's summation order.
"""

from __future__ import annotations

import json
import os

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

TOKENS, LAYERS, HIDDEN, INTER, EXPERTS, TOP_K, EPS = 1024, 8, 2048, 768, 128, 8, 1e-6


def torch_router(normed: torch.Tensor, gate: torch.Tensor):
    """``_route_impl`` lines 319-323 on one bf16 row: (ids, bf16 weights)."""
    probabilities = torch.softmax(F.linear(normed, gate).float(), dim=-1)
    weights, ids = probabilities.topk(TOP_K, dim=-1)
    weights = weights / weights.sum(dim=-1, keepdim=True)
    return ids, weights.to(normed.dtype)


def torch_rms_norm(hidden: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """The RMSNorm the decode graph applies before routing, in torch ops (fp32 math, bf16 out)."""
    x = hidden.float()
    return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + EPS) * gamma).to(torch.bfloat16)


def run_stack(device, *, exact: bool):
    from drama_b200 import stack, synthetic
    from drama_b200.stack import LayerTrace

    layers = stack.synthetic_stack(LAYERS, experts=EXPERTS, hidden=HIDDEN, intermediate=INTER, seed=7,
                                   device=device)
    ws = stack.moe_layer_workspace(1, TOP_K, HIDDEN, INTER, EXPERTS, device)
    hs = torch.empty(LAYERS + 1, TOKENS, 1, HIDDEN, dtype=torch.bfloat16, device=device)
    hs[0] = synthetic.hidden_states(TOKENS, HIDDEN, 31, device=device).view(TOKENS, 1, HIDDEN)
    ids = torch.empty(LAYERS, TOKENS, 1, TOP_K, dtype=torch.int64, device=device)
    wts = torch.empty(LAYERS, TOKENS, 1, TOP_K, dtype=torch.bfloat16, device=device)
    normed = torch.empty(LAYERS, TOKENS, 1, HIDDEN, dtype=torch.bfloat16, device=device)
    for s in range(TOKENS):
        for i, layer in enumerate(layers):
            tr = LayerTrace(ids[i, s], wts[i, s], normed[i, s])
            stack.moe_layer(hs[i, s], layer, hs[i + 1, s], ws, top_k=TOP_K, trace=tr,
                            router="torch" if exact else "fused")
    torch.cuda.synchronize()
    return layers, hs, ids, wts, normed


def compare(layers, hs, ids, wts, normed):
    stats = {"token_layers": TOKENS * LAYERS, "normed_rows_differ": 0, "normed_elems_differ": 0,
             "ids_differ": 0, "ids_set_differ": 0, "ids_differ_same_normed": 0, "weights_differ": 0}
    cases = []
    for i, layer in enumerate(layers):
        for s in range(TOKENS):
            ref_normed = torch_rms_norm(hs[i, s], layer.gamma)
            ref_ids, ref_w = torch_router(ref_normed, layer.gate)
            own_ids, _ = torch_router(normed[i, s], layer.gate)
            if not torch.equal(ref_w.view(torch.int16), wts[i, s].view(torch.int16)):
                logits = F.linear(ref_normed, layer.gate)
                top, _ = torch.softmax(logits.float(), dim=-1).topk(TOP_K, dim=-1)
                cases.append((logits.view(torch.int16).cpu(), top.cpu(), top.sum(-1).cpu(),
                              (top / top.sum(-1, keepdim=True)).cpu(), ref_ids.cpu(),
                              ref_w.view(torch.int16).cpu(), ids[i, s].cpu(), wts[i, s].view(torch.int16).cpu()))
            diff = int((ref_normed.view(torch.int16) != normed[i, s].view(torch.int16)).sum())
            stats["normed_elems_differ"] += diff
            stats["normed_rows_differ"] += int(diff > 0)
            if not torch.equal(ref_ids, ids[i, s]):
                stats["ids_differ"] += 1
                if not torch.equal(ref_ids.sort().values, ids[i, s].sort().values):
                    stats["ids_set_differ"] += 1
            stats["ids_differ_same_normed"] += int(not torch.equal(own_ids, ids[i, s]))
            stats["weights_differ"] += int(not torch.equal(ref_w.view(torch.int16), wts[i, s].view(torch.int16)))
    out = os.environ.get("DRAMA_B200_REPORT_DIR")
    if out and cases:
        torch.save(cases, os.path.join(out, f"router_weight_cases_{len(cases)}.pt"))
    return stats


def _report(name, stats):
    print(f"\n{name}: {json.dumps(stats)}")
    out = os.environ.get("DRAMA_B200_REPORT_DIR")
    if out:
        with open(os.path.join(out, f"router_reference_{name}.json"), "w") as f:
            json.dump(stats, f, indent=1)


def test_fused_router_against_torch_router(cuda_device):
    """Measurement: the fused layer computes RMSNorm and the router GEMV in its own fixed fp32 order."""
    stats = compare(*run_stack(cuda_device, exact=False))
    _report("fused", stats)
    # a bf16 rounding flip moves a route only at a near-tie of the top-8 boundary
    assert stats["ids_set_differ"] <= 0.02 * stats["token_layers"], stats


def test_torch_router_mode_is_exact(cuda_device):
    """With ``router="torch"`` the layer routes on torch's normalised row and logits: every id matches."""
    stats = compare(*run_stack(cuda_device, exact=True))
    _report("torch", stats)
    assert stats["normed_rows_differ"] == 0, stats
    assert stats["ids_differ"] == 0, stats
    assert stats["weights_differ"] == 0, stats


def _crafted_logits(device):
    """Router logits rows (bf16 [EXPERTS]) that stress the top-k selection:
    wide ties (the selection's candidate set overflows and the full ranking
    runs), ties among the winners (torch's sorting network orders them), ties
    across the k-th boundary, few distinct values, and -inf entries."""
    g = torch.Generator(device="cpu").manual_seed(11)
    rows = []
    rows.append(torch.zeros(EXPERTS))                                     # 128-way tie
    r = torch.randn(EXPERTS, generator=g) - 4.0
    r[torch.randperm(EXPERTS, generator=g)[:40]] = 3.0                    # 40 winners tied
    rows.append(r)
    r = torch.randn(EXPERTS, generator=g) - 4.0
    r[torch.randperm(EXPERTS, generator=g)[:TOP_K]] = 2.5                  # exactly k tied winners
    rows.append(r)
    r = torch.randn(EXPERTS, generator=g) - 4.0
    top = torch.randperm(EXPERTS, generator=g)
    r[top[:6]] = torch.tensor([5.0, 4.5, 4.0, 3.5, 3.0, 2.75])
    r[top[6:11]] = 2.5                                                    # ties across the k-th boundary
    rows.append(r)
    for _ in range(4):
        rows.append(torch.round(torch.randn(EXPERTS, generator=g) * 2.0) / 4.0)  # few distinct values
    r = torch.full((EXPERTS,), float("-inf"))
    r[torch.randperm(EXPERTS, generator=g)[:12]] = torch.randn(12, generator=g)  # all but 12 at -inf
    rows.append(r)
    r = torch.randn(EXPERTS, generator=g)
    r[5::16] = r[5]                                                       # 8 experts share one value
    rows.append(r)
    return [x.to(torch.bfloat16).to(device) for x in rows]


def _logits_layer(layer, normed, logits, hidden_in, out, ws, ids, wts):
    import ctypes

    from drama_b200 import _lib

    bank, keep = layer.bank()
    lib = _lib.library()
    lib.check(lib.dll.drama_b200_fp8_moe_layer_logits(
        ctypes.byref(bank), normed.data_ptr(), logits.data_ptr(), hidden_in.data_ptr(), out.data_ptr(), 1, TOP_K,
        ids.data_ptr(), wts.data_ptr(), None, ws.data_ptr(), ws.numel(), _lib.stream_handle(normed.device)))
    del keep


def test_crafted_ties_route_like_torch(cuda_device):
    """Tie-heavy logits through the logits-driven layer (config-1 shape): ids and
    bf16 weights equal torch's softmax -> topk -> renormalise on the same GPU."""
    from drama_b200 import stack, synthetic

    layer = stack.synthetic_stack(1, experts=EXPERTS, hidden=HIDDEN, intermediate=INTER, seed=7,
                                  device=cuda_device)[0]
    ws = stack.moe_layer_workspace(1, TOP_K, HIDDEN, INTER, EXPERTS, cuda_device)
    hidden = synthetic.hidden_states(1, HIDDEN, 5, device=cuda_device)
    normed = torch_rms_norm(hidden, layer.gamma)
    out = torch.empty_like(hidden)
    for n, logits in enumerate(_crafted_logits(cuda_device)):
        ids = torch.empty(1, TOP_K, dtype=torch.int64, device=cuda_device)
        wts = torch.empty(1, TOP_K, dtype=torch.bfloat16, device=cuda_device)
        _logits_layer(layer, normed, logits.view(1, -1), hidden, out, ws, ids, wts)
        probabilities = torch.softmax(logits.view(1, -1).float(), dim=-1)
        ref_w, ref_ids = probabilities.topk(TOP_K, dim=-1)
        ref_w = (ref_w / ref_w.sum(dim=-1, keepdim=True)).to(torch.bfloat16)
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids), (n, ids.tolist(), ref_ids.tolist())
        assert torch.equal(wts.view(torch.int16), ref_w.view(torch.int16)), (n, wts.tolist(), ref_w.tolist())
        assert torch.isfinite(out.float()).all(), n


def test_nan_logits_route_inside_the_bank(cuda_device):
    """A NaN logit makes every probability NaN; the layer still picks expert ids
    inside the bank (it reads no weight row out of bounds)."""
    from drama_b200 import stack, synthetic

    layer = stack.synthetic_stack(1, experts=EXPERTS, hidden=HIDDEN, intermediate=INTER, seed=7,
                                  device=cuda_device)[0]
    ws = stack.moe_layer_workspace(1, TOP_K, HIDDEN, INTER, EXPERTS, cuda_device)
    hidden = synthetic.hidden_states(1, HIDDEN, 5, device=cuda_device)
    normed = torch_rms_norm(hidden, layer.gamma)
    logits = torch.randn(1, EXPERTS, device=cuda_device).to(torch.bfloat16)
    logits[0, 17] = float("nan")
    ids = torch.empty(1, TOP_K, dtype=torch.int64, device=cuda_device)
    wts = torch.empty(1, TOP_K, dtype=torch.bfloat16, device=cuda_device)
    out = torch.empty_like(hidden)
    _logits_layer(layer, normed, logits, hidden, out, ws, ids, wts)
    torch.cuda.synchronize()
    assert ((ids >= 0) & (ids < EXPERTS)).all(), ids.tolist()
