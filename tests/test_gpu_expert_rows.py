"""Per-row expert projections on the swap-AB grouped GEMMs (``drama_b200_fp8_expert_rows``).

Against the oracle's dequant path (``fp8_dequant_pairs`` with unit route
weights: the bf16 down projection of each row), at the north_star tolerance;
rows with an out-of-range id are not written; and a row's result is the same,
bit for bit, whatever other rows share the call (the property expert
parallelism relies on to be independent of the number of GPUs).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_parity, np_bank, np_f32
from oracle import restate as R

pytestmark = pytest.mark.gpu


class Bank:
    def __init__(self, d):
        self.__dict__.update(d)


def _case(device, experts, hidden, inter, rows, seed, bad=0, hot=0):
    from drama_b200 import synthetic

    bank = synthetic.fp8_bank(experts, hidden, inter, seed, device=device, chunk=experts)
    gen = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, experts, (rows,), generator=gen)
    if hot:
        ids[:hot] = 1                                   # one expert with many rows (several 32-row chunks)
    if bad:
        ids[torch.randperm(rows, generator=gen)[:bad]] = experts + 3
    x = synthetic.hidden_states(rows, hidden, seed + 1, device=device)
    return bank, ids.to(device), x


@pytest.mark.parametrize("experts,hidden,inter,rows,bad,hot", [
    (16, 512, 256, 70, 3, 40),
    (128, 2048, 768, 300, 0, 100),
    (4, 256, 128, 5, 1, 0),
])
def test_rows_match_the_oracle(cuda_device, experts, hidden, inter, rows, bad, hot):
    from drama_b200.backend import fp8_expert_rows

    bank, ids, x = _case(cuda_device, experts, hidden, inter, rows, seed=rows, bad=bad, hot=hot)
    out = fp8_expert_rows(x, ids.to(torch.int32), Bank(bank))
    torch.cuda.synchronize()
    ids_np = ids.cpu().numpy()
    valid = np.flatnonzero((ids_np >= 0) & (ids_np < experts))
    want = R.fp8_dequant_pairs(np_f32(x)[valid], ids_np[valid], np.ones(valid.size, np.float32), np_bank(bank))
    got = np_f32(out)
    assert_parity(got[valid], want, label=f"expert rows E={experts} H={hidden} I={inter}")
    dropped = np.setdiff1d(np.arange(rows), valid)
    assert not got[dropped].any()


def test_each_row_is_independent_of_the_rest_of_the_call(cuda_device):
    from drama_b200.backend import fp8_expert_rows

    bank, ids, x = _case(cuda_device, 32, 1024, 512, 257, seed=9, hot=70)
    full = fp8_expert_rows(x, ids, Bank(bank))
    perm = torch.randperm(257, generator=torch.Generator().manual_seed(1)).to(cuda_device)
    shuffled = fp8_expert_rows(x[perm], ids[perm], Bank(bank))
    part = fp8_expert_rows(x[:37], ids[:37], Bank(bank))
    torch.cuda.synchronize()
    assert torch.equal(shuffled, full[perm])
    assert torch.equal(part, full[:37])


def test_against_the_tile_gemm(cuda_device):
    """Same rounding points as the 128-row tile GEMM of fp8_prefill (unit weights, top-1)."""
    from drama_b200.backend import fp8_expert_rows, fp8_prefill

    bank, ids, x = _case(cuda_device, 16, 2048, 768, 200, seed=4, hot=60)
    rows = fp8_expert_rows(x, ids, Bank(bank))
    tile = fp8_prefill(x, ids[:, None], torch.ones(200, 1, dtype=torch.bfloat16, device=cuda_device), Bank(bank))
    torch.cuda.synchronize()
    same = int((rows == tile).all(dim=1).sum())
    print(f"expert rows vs tile GEMM: {same} of 200 rows bit-identical")
    assert_parity(np_f32(rows), np_f32(tile), label="expert rows vs tile GEMM")


def test_tagged_rows_equal_rows_with_an_id_array(cuda_device):
    """Rows carrying their expert id after the hidden values (the exchanged layout)."""
    import ctypes

    from drama_b200 import _lib
    from drama_b200.backend import _fp8_bank, fp8_expert_rows

    bank, ids, x = _case(cuda_device, 16, 1024, 256, 90, seed=12, bad=4, hot=40)
    want = fp8_expert_rows(x, ids, Bank(bank))
    tagged = torch.zeros(90, 1024 + 8, dtype=torch.bfloat16, device=cuda_device)
    tagged[:, :1024] = x
    tagged.view(torch.int32)[:, 512] = ids.to(torch.int32)
    lib = _lib.library()
    fb, keep = _fp8_bank(Bank(bank), 1024)
    ws = torch.zeros(lib.dll.drama_b200_expert_rows_workspace_bytes(90, 1024, 256, 16), dtype=torch.uint8,
                     device=cuda_device)
    out = torch.zeros(90, 1024, dtype=torch.bfloat16, device=cuda_device)
    lib.check(lib.dll.drama_b200_fp8_expert_rows(ctypes.byref(fb), tagged.data_ptr(), 1024 + 8, 90, None, _lib.I32,
                                                 out.data_ptr(), ws.data_ptr(), ws.numel(),
                                                 _lib.stream_handle(cuda_device)))
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    del keep
