"""K3 router and permutation on the B200: bit-exact against the oracle and
against the reference's own router ops (torch on CUDA)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import restate as R

pytestmark = pytest.mark.gpu


def _logit_cases():
    gen = torch.Generator().manual_seed(99)
    yield "normal", (torch.randn(1024, 128, generator=gen) * 0.905).to(torch.bfloat16), 8, True
    yield "coarse_ties", (torch.randint(-4, 5, (512, 128), generator=gen).float() / 4).to(torch.bfloat16), 8, True
    yield "all_equal", torch.zeros(8, 128, dtype=torch.bfloat16), 8, True
    yield "e256", (torch.randn(256, 256, generator=gen) * 0.9).to(torch.bfloat16), 8, True
    yield "e16_k4_raw", (torch.randint(-2, 3, (64, 16), generator=gen).float()).to(torch.bfloat16), 4, False
    yield "e1024_k32", (torch.randint(-3, 4, (32, 1024), generator=gen).float() / 3).to(torch.bfloat16), 32, True
    yield "e60_k6", torch.randn(64, 60, generator=gen).to(torch.bfloat16), 6, True
    yield "fp32_logits", torch.randn(128, 128, generator=gen) * 2, 8, True


def _reference_route(logits: torch.Tensor, top_k: int, renorm: bool, dtype):
    # backbone_graph.py:319-323, run on the GPU.
    probabilities = torch.softmax(logits.float(), dim=-1)
    w, ids = probabilities.topk(top_k, dim=-1)
    if renorm:
        w = w / w.sum(dim=-1, keepdim=True)
    return w.to(dtype), ids


@pytest.mark.parametrize("case", list(_logit_cases()), ids=lambda c: c[0])
def test_route_topk_matches_reference_ops_and_oracle(cuda_device, case):
    from drama_b200 import route_topk

    name, logits, top_k, renorm = case
    out_dtype = torch.bfloat16
    dev = logits.to(cuda_device)
    w, ids = route_topk(dev, top_k, renormalize=renorm, out_dtype=out_dtype)
    w_ref, ids_ref = _reference_route(dev, top_k, renorm, out_dtype)
    assert torch.equal(ids.cpu(), ids_ref.cpu()), f"{name}: ids differ from torch CUDA topk"
    assert torch.equal(w.cpu().view(torch.int16), w_ref.cpu().view(torch.int16)), f"{name}: weights differ"
    o_ids, o_w, _ = R.route_topk(logits.float().numpy(), top_k, renorm, "bfloat16")
    np.testing.assert_array_equal(ids.cpu().numpy(), o_ids, err_msg=name)
    diff = np.abs(R.bf16_bits(o_w).astype(np.int32) - w.cpu().view(torch.int16).numpy().view(np.uint16).astype(np.int32))
    assert diff.max() <= 1, name


def test_route_topk_int32_fp32_outputs(cuda_device):
    from drama_b200 import route_topk

    logits = (torch.randn(16, 128, generator=torch.Generator().manual_seed(5)) * 0.9).to(torch.bfloat16)
    dev = logits.to(cuda_device)
    w, ids = route_topk(dev, 8, out_dtype=torch.float32, ids_dtype=torch.int32)
    w_ref, ids_ref = _reference_route(dev, 8, True, torch.float32)
    assert ids.dtype == torch.int32 and torch.equal(ids.long().cpu(), ids_ref.cpu())
    torch.testing.assert_close(w, w_ref, rtol=2e-7, atol=0)


@pytest.mark.parametrize("experts,shape,kind", [
    (128, (1, 8), "uniform"), (128, (4, 8), "uniform"), (6, (64, 8), "dense"),
    (128, (4096, 8), "zipf"), (4, (5, 3), "single"), (1024, (300, 7), "dense"), (128, (40000, 8), "zipf"),
])
def test_permute_routes_matches_stable_argsort(cuda_device, experts, shape, kind):
    from drama_b200 import permute_routes, synthetic

    gen = torch.Generator().manual_seed(experts * 7 + shape[0])
    if kind == "uniform":
        ids = synthetic.uniform_routes(shape[0], shape[1], experts, 3)[0]
    elif kind == "zipf":
        ids = synthetic.zipf_routes(shape[0], shape[1], experts, 4)[0]
    elif kind == "single":
        ids = torch.zeros(shape, dtype=torch.int64)
    else:
        ids = torch.randint(0, experts, shape, generator=gen)
    for dtype in (torch.int64, torch.int32):
        for wide in (False, True):
            position = torch.empty(ids.numel(), dtype=torch.int64, device=cuda_device) if wide else None
            order, counts, offsets = permute_routes(ids.to(cuda_device, dtype), experts, wide=wide,
                                                    position=position)
            flat = ids.reshape(-1)
            assert torch.equal(order.cpu(), torch.argsort(flat, stable=True))
            assert torch.equal(counts.cpu(), torch.bincount(flat, minlength=experts))
            o_order, o_counts, o_offsets = R.permute_routes(flat.numpy(), experts)
            np.testing.assert_array_equal(offsets.cpu().numpy(), o_offsets)
            if wide:  # position is the inverse of order
                inv = torch.empty_like(order)
                inv[order] = torch.arange(order.numel(), device=order.device)
                assert torch.equal(position, inv)


def test_permute_routes_counts_out_of_range_ids(cuda_device):
    from drama_b200 import permute_routes

    ids = torch.tensor([3, 9, 1, -1, 3], device=cuda_device)
    for wide in (False, True):
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        position = torch.empty(5, dtype=torch.int64, device=cuda_device) if wide else None
        order, counts, offsets = permute_routes(ids, 4, status=status, wide=wide, position=position)
        assert int(status.item()) == 2
        assert counts.cpu().tolist() == [0, 1, 0, 2]
        assert order.cpu()[:3].tolist() == [2, 0, 4]
        if wide:
            assert position.cpu().tolist() == [1, -1, 0, -1, 2]
