"""K2 on tcgen05: the FP8 W8A8 contract as grouped tensor-core GEMMs.

``drama_b200_fp8_w8a8_prefill`` computes the arithmetic of the reference's
production GPU backend for many rows (``TritonExpertBackend.forward_pairs``,
``offload.py:289-341``; CPU statement ``native/src/runtime.cpp:162-237``),
which the oracle's ``w8a8_pairs`` restates and ``tests/test_oracle.py`` pins to
the reference's native core byte for byte.

* Small cases (ragged tiles, experts with no rows, dropped ids): every pair
  row against the oracle at the 2e-2 bar, the combined rows too, dropped
  pairs' rows exactly zero, a second call bit-identical.
* Config 3 (4096 tokens, top-8 of 128 experts, Zipf(1.1), hidden 2048,
  intermediate 768): every pair row against a float32 torch statement of the
  same contract on the GPU (TF32 off), and 256 pairs, half of them on the
  most-loaded expert, against the oracle.
* ``Fp8W8a8B200Backend`` dispatches such calls to this path and returns the
  same bits as the direct call.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import assert_parity, np_bank, np_f32
from oracle import restate as R

pytestmark = pytest.mark.gpu


class _Staged:
    def __init__(self, bank):
        for k, v in bank.items():
            setattr(self, k, v)


def _case(device, tokens, top_k, experts, hidden, inter, seed, zipf=False):
    from drama_b200 import synthetic

    bank = synthetic.fp8_bank(experts, hidden, inter, seed, device=device, chunk=experts)
    routes = synthetic.zipf_routes if zipf else synthetic.uniform_routes
    ids, w = routes(tokens, top_k, experts, seed + 1, device=device)
    x = synthetic.hidden_states(tokens, hidden, seed + 2, device=device)
    return bank, x, ids.to(torch.int64).contiguous(), w.to(torch.bfloat16).contiguous()


def _prefill(bank, x, ids, w):
    """(combined rows, weighted pair rows) through the C ABI."""
    from drama_b200 import _lib
    from drama_b200.backend import _fp8_bank

    lib = _lib.library()
    tokens, top_k = ids.shape
    hidden = x.shape[1]
    fp8, keep = _fp8_bank(_Staged(bank), hidden)
    assert lib.dll.drama_b200_fp8_w8a8_prefill_supported(fp8.hidden, fp8.intermediate, fp8.slots) == 1
    nbytes = lib.dll.drama_b200_fp8_w8a8_prefill_workspace_bytes(tokens, top_k, fp8.hidden, fp8.intermediate,
                                                                  fp8.slots)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    out = torch.full_like(x, float("nan"))
    pairs = torch.full((tokens * top_k, hidden), float("nan"), dtype=torch.float32, device=x.device)
    lib.check(lib.dll.drama_b200_fp8_w8a8_prefill(
        ctypes.byref(fp8), x.data_ptr(), tokens, top_k, ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype], w.data_ptr(),
        _lib.DTYPE_CODES[w.dtype], out.data_ptr(), pairs.data_ptr(), ws.data_ptr(), ws.numel(),
        _lib.stream_handle(x.device)))
    torch.cuda.synchronize()
    lead = (-ws.data_ptr()) % 1024  # the library starts its buffers on the next 1024-byte boundary
    status = ws[lead:lead + 16].view(torch.int32).tolist()
    del keep
    return out, pairs, status


def _oracle_pairs(x, ids, w, bank, tokens):
    nb = np_bank(bank)
    xs, fl, ws = np_f32(x), ids.cpu().numpy(), np_f32(w)
    rows = []
    for t in tokens:
        rows.append(R.w8a8_pairs(xs[t], fl[t], ws[t], nb))
    return np.concatenate(rows)


@pytest.mark.parametrize("tokens,top_k,experts,hidden,inter,zipf", [
    (40, 2, 4, 256, 128, False),      # the smallest case: one ragged tile per expert
    (300, 8, 16, 512, 256, True),     # Zipf: several tiles on the head expert, some experts empty
    (130, 4, 8, 768, 384, False),     # three N tiles of the down GEMM, three gate/up column tiles
])
def test_prefill_tc_matches_oracle(cuda_device, tokens, top_k, experts, hidden, inter, zipf):
    bank, x, ids, w = _case(cuda_device, tokens, top_k, experts, hidden, inter, seed=tokens + top_k, zipf=zipf)
    out, pairs, status = _prefill(bank, x, ids, w)
    assert status[0] == 0 and status[1] == 0, status
    expected = _oracle_pairs(x, ids, w, bank, range(tokens))
    label = f"tcgen05 W8A8 T={tokens} k={top_k} E={experts} {hidden}x{inter}"
    assert_parity(pairs.cpu().numpy(), expected, label=label + " pair rows")
    combined = R.combine_slots(expected, tokens, top_k, "bfloat16")
    assert_parity(np_f32(out), combined, label=label + " combined")
    again, pairs2, _ = _prefill(bank, x, ids, w)
    assert torch.equal(out.view(torch.int16), again.view(torch.int16))
    assert torch.equal(pairs, pairs2)


def test_prefill_tc_dropped_ids(cuda_device):
    """Out-of-range ids contribute zero and their pair rows are zero."""
    bank, x, ids, w = _case(cuda_device, 64, 4, 8, 256, 128, seed=5)
    bad = ids.clone()
    bad[3, 1] = -1
    bad[10, 0] = 8
    bad[11, 3] = 1 << 40
    out, pairs, status = _prefill(bank, x, bad, w)
    assert status[0] == 3
    for t, s in ((3, 1), (10, 0), (11, 3)):
        assert torch.count_nonzero(pairs[t * 4 + s]) == 0
    keep = (bad >= 0) & (bad < 8)
    expected = _oracle_pairs(x, ids, w, bank, range(64))
    expected[~keep.cpu().numpy().reshape(-1)] = 0.0
    assert_parity(pairs.cpu().numpy(), expected, label="dropped ids: pair rows")
    assert_parity(np_f32(out), R.combine_slots(expected, 64, 4, "bfloat16"), label="dropped ids: combined")


def _torch_w8a8_pairs(x, ids, w, bank):
    """The W8A8 contract in float32 torch on the GPU, batched per expert."""
    tokens, top_k = ids.shape
    hidden = x.shape[1]
    inter = bank["w2_weight"].shape[2]

    def quant(v):
        blocks = v.view(v.shape[0], -1, 128)
        scale = blocks.abs().amax(-1).clamp_min(1e-10) * (1.0 / 448.0)
        q = (blocks / scale[..., None]).to(torch.float8_e4m3fn).float()
        return q, scale

    def block_gemm(q, qs, wq, ws):
        # q [R, KB, 128], wq [N, KB, 128], qs [R, KB], ws [N/128, KB] -> [R, N]
        dots = torch.einsum("rkc,nkc->krn", q, wq)
        sb = ws.repeat_interleave(128, 0).t()           # [KB, N]
        acc = torch.zeros(q.shape[0], wq.shape[0], device=q.device)
        for kb in range(q.shape[1]):
            acc = acc + dots[kb] * (qs[:, kb, None] * sb[kb][None, :])
        return acc

    flat = ids.reshape(-1)
    pair_token = torch.arange(tokens * top_k, device=x.device) // top_k
    out = torch.zeros(tokens * top_k, hidden, device=x.device)
    xq, xs = quant(x.float())
    for e in torch.unique(flat).tolist():
        rows = torch.nonzero(flat == e).reshape(-1)
        q, qs = xq[pair_token[rows]], xs[pair_token[rows]]
        w13 = bank["w13_weight"][e].float().view(2 * inter, -1, 128)
        gu = block_gemm(q, qs, w13, bank["w13_scale_inv"][e])
        gu = gu.to(torch.bfloat16).float()
        gate, up = gu[:, :inter], gu[:, inter:]
        h = (gate / (1.0 + torch.exp(-gate))) * up
        hq, hs = quant(h)
        w2 = bank["w2_weight"][e].float().view(hidden, -1, 128)
        down = block_gemm(hq, hs, w2, bank["w2_scale_inv"][e])
        out[rows] = down * w.reshape(-1)[rows].float()[:, None]
    return out


def test_prefill_tc_config3(cuda_device):
    """4096 tokens, top-8 of 128 experts, Zipf(1.1): every pair row against the
    torch statement, 256 pairs against the oracle."""
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        bank, x, ids, w = _case(cuda_device, 4096, 8, 128, 2048, 768, seed=7, zipf=True)
        out, pairs, status = _prefill(bank, x, ids, w)
        assert status[0] == 0 and status[1] == 0, status
        ref = _torch_w8a8_pairs(x, ids, w, bank)
        torch.cuda.synchronize()
        assert_parity(pairs.cpu().numpy(), ref.cpu().numpy(), label="tcgen05 W8A8 config 3, all pair rows vs torch")
        slots = ref.view(4096, 8, -1)
        combined = slots[:, 0]
        for s in range(1, 8):  # slot order
            combined = combined + slots[:, s]
        assert_parity(np_f32(out), combined.cpu().numpy(), label="tcgen05 W8A8 config 3, combined vs torch")
        flat = ids.cpu().numpy()
        head = np.bincount(flat.reshape(-1), minlength=128).argmax()
        on_head = np.flatnonzero((flat == head).any(axis=1))
        rng = np.random.default_rng(7)
        tokens = np.concatenate([rng.choice(on_head, 16, replace=False),
                                 rng.choice(np.setdiff1d(np.arange(4096), on_head), 16, replace=False)])
        tokens.sort()
        expected = _oracle_pairs(x, ids, w, bank, tokens)
        got = pairs.view(4096, 8, -1)[torch.as_tensor(tokens, device=x.device)].reshape(-1, 2048)
        assert_parity(got.cpu().numpy(), expected, label=f"tcgen05 W8A8 config 3, 256 oracle pairs (head {head})")
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32


def test_backend_dispatches_many_pairs_to_tcgen05(cuda_device):
    from drama_b200 import Fp8W8a8B200Backend

    bank, x, ids, w = _case(cuda_device, 300, 8, 16, 512, 256, seed=11, zipf=True)
    direct, pairs, _ = _prefill(bank, x, ids, w)
    backend = Fp8W8a8B200Backend(prefill_min_pairs=512)
    got = backend.forward(x, ids, w, _Staged(bank))
    got_pairs = backend.forward_pairs(x.repeat_interleave(8, 0), ids.reshape(-1, 1), w.reshape(-1, 1),
                                      _Staged(bank))
    cells = Fp8W8a8B200Backend(prefill_min_pairs=1 << 30).forward(x, ids, w, _Staged(bank))
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), direct.view(torch.int16))
    assert torch.equal(got_pairs, pairs)
    assert_parity(np_f32(got), np_f32(cells), label="tcgen05 GEMMs vs per-pair cells, same contract")
