"""The official FP8 W8A8 contract on the B200 against the oracle.

``Fp8W8a8B200Backend`` / ``drama_b200_fp8_w8a8_decode`` compute the
arithmetic of the reference's production GPU backend (``fp8_decode.py:
114-147``; CPU statement ``native/src/runtime.cpp:162-237``), which
``oracle/restate.py`` ``w8a8_pairs`` restates and ``tests/test_oracle.py``
pins byte for byte to the reference's native core. The quantised token rows
(E4M3 bytes and block scales) must equal the oracle's exactly; the weighted
partials and the combined rows must meet the 2e-2 bar (the block dots run on
E4M3 tensor cores, whose addition order inside a block is the hardware's).
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


def _case(device, tokens, top_k, experts, hidden, inter, seed):
    from drama_b200 import synthetic

    bank = synthetic.fp8_bank(experts, hidden, inter, seed, device=device, chunk=experts)
    ids, w = synthetic.uniform_routes(tokens, top_k, experts, seed + 1, device=device)
    x = synthetic.hidden_states(tokens, hidden, seed + 2, device=device)
    return bank, x, ids.to(torch.int64).contiguous(), w.to(torch.bfloat16).contiguous()


@pytest.mark.parametrize("tokens,top_k,experts,hidden,inter", [(1, 8, 128, 2048, 768), (3, 4, 16, 512, 256),
                                                               (2, 8, 32, 1024, 384)])
def test_w8a8_matches_oracle(cuda_device, tokens, top_k, experts, hidden, inter):
    from drama_b200 import Fp8W8a8B200Backend, _lib
    from drama_b200.backend import _fp8_bank

    bank, x, ids, w = _case(cuda_device, tokens, top_k, experts, hidden, inter, seed=tokens + top_k)
    staged = _Staged(bank)
    backend = Fp8W8a8B200Backend()
    out = backend.forward(x, ids, w, staged)
    # the pair path (forward_pairs on flattened rows) and the quantised token rows
    lib = _lib.library()
    fp8, keep = _fp8_bank(staged, hidden)
    xq = torch.empty((tokens, hidden), dtype=torch.uint8, device=cuda_device)
    xs = torch.empty((tokens, hidden // 128), dtype=torch.float32, device=cuda_device)
    pairs = torch.empty((tokens * top_k, hidden), dtype=torch.float32, device=cuda_device)
    nbytes = lib.dll.drama_b200_fp8_w8a8_workspace_bytes(tokens, top_k, hidden, inter)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    lib.check(lib.dll.drama_b200_fp8_w8a8_decode(
        ctypes.byref(fp8), x.data_ptr(), tokens, top_k, ids.data_ptr(), _lib.I64, w.data_ptr(), _lib.BF16, None,
        pairs.data_ptr(), xq.data_ptr(), xs.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_handle(cuda_device)))
    torch.cuda.synchronize()
    nb = np_bank(bank)
    xn = np_f32(x)
    for t in range(tokens):
        q, s = R.quantize_fp8_activations(xn[t])
        assert np.array_equal(xq[t].cpu().numpy(), q), f"token {t}: E4M3 bytes differ from the oracle"
        assert np.array_equal(xs[t].cpu().numpy(), s), f"token {t}: block scales differ from the oracle"
    want_pairs = np.concatenate([R.w8a8_pairs(xn[t], ids[t].cpu().numpy(), np_f32(w[t]), nb)
                                 for t in range(tokens)])
    assert_parity(pairs.cpu().numpy(), want_pairs, label=f"W8A8 partials T={tokens} k={top_k} {hidden}x{inter}")
    want = R.combine_slots(want_pairs, tokens, top_k, "bfloat16")
    assert_parity(np_f32(out), want, label=f"W8A8 output T={tokens} k={top_k} {hidden}x{inter}")
    # the combined output is the slot-order sum of the same partials, rounded once
    assert np.array_equal(np_f32(out), R.combine_slots(pairs.cpu().numpy(), tokens, top_k, "bfloat16"))
    # and within the 2e-2 bar of the W16A16 dequant path as well
    dequant = R.fp8_dequant_forward(xn, ids.cpu().numpy(), np_f32(w), nb, "bfloat16")
    assert_parity(np_f32(out), dequant, rel=5e-2, label="W8A8 vs W16A16 dequant path")
    del keep


def test_w8a8_backend_protocol(cuda_device):
    from drama_b200 import Fp8W8a8B200Backend

    bank, x, ids, w = _case(cuda_device, 4, 1, 8, 256, 128, seed=3)
    staged = _Staged(bank)
    backend = Fp8W8a8B200Backend()
    pairs = backend.forward_pairs(x, ids, w, staged)
    assert pairs.dtype == torch.float32 and pairs.shape == x.shape
    assert torch.equal(pairs, backend.forward_decode_pairs(x, ids, w, staged))
    with pytest.raises(ValueError, match="outside the staging pool"):
        backend.forward(x, torch.full_like(ids, 8), w, staged)
    with pytest.raises(ValueError, match="bfloat16"):
        backend.forward(x.float(), ids, w, staged)
    assert backend.forward(x[:0], ids[:0], w[:0], staged).shape == (0, 256)
