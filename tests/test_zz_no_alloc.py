"""The allocation-free FP8 decode entry point against the workspace one.

``drama_b200_fp8_decode_static`` serves callers that cannot allocate device
memory: a host binding with no device allocator of its own, or a process whose
memory manager has reserved the device and allows no further allocation. It
keeps its scratch in a static array inside the library instead of taking a
workspace. These tests call both entry points through the C ABI on the same
inputs and hold the static one to the parity bar of the other GPU tests, on
two calls in a row (the second call reuses what the first left in the array).

Both entry points run the same kernels on the same inputs, so the outputs are
compared bit for bit. The device's free memory (cudaMemGetInfo) is read around
the second static call, after the first call's set-up: it must not shrink.

The file name makes pytest collect it last, after every other test file.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import MAX_ABS_TOL, REL_TOL, assert_parity, np_f32

pytestmark = pytest.mark.gpu


def _inputs(device, tokens, top_k, hidden, inter, experts, seed):
    from drama_b200 import synthetic
    from drama_b200.backend import _fp8_bank

    bank = synthetic.fp8_bank(experts, hidden, inter, seed, device=device, chunk=experts)

    class Staged:
        w13_weight = bank["w13_weight"]
        w13_scale_inv = bank["w13_scale_inv"]
        w2_weight = bank["w2_weight"]
        w2_scale_inv = bank["w2_scale_inv"]

    fp8, keep = _fp8_bank(Staged, hidden)
    ids, w = synthetic.uniform_routes(tokens, top_k, experts, seed + 1, device=device)
    x = synthetic.hidden_states(tokens, hidden, seed + 2, device=device)
    return fp8, (bank, keep), x, ids.to(torch.int64).contiguous(), w.to(torch.bfloat16).contiguous()


def _workspace_call(lib, fp8, x, ids, w, top_k, out):
    from drama_b200 import _lib

    tokens = x.shape[0]
    nbytes = lib.dll.drama_b200_decode_workspace_bytes(tokens, top_k, fp8.hidden, fp8.intermediate)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
    lib.check(lib.dll.drama_b200_fp8_decode(
        ctypes.byref(fp8), x.data_ptr(), _lib.BF16, tokens, top_k, ids.data_ptr(), _lib.I64, w.data_ptr(),
        _lib.BF16, out.data_ptr(), None, ws.data_ptr(), ws.numel(), _lib.stream_handle(x.device)))
    return ws


def _static_call(lib, fp8, x, ids, w, top_k, out):
    from drama_b200 import _lib

    return lib.dll.drama_b200_fp8_decode_static(
        ctypes.byref(fp8), x.data_ptr(), _lib.BF16, x.shape[0], top_k, ids.data_ptr(), _lib.I64, w.data_ptr(),
        _lib.BF16, out.data_ptr(), None, _lib.stream_handle(x.device))


@pytest.mark.parametrize("tokens,top_k,hidden,inter,experts", [(1, 8, 2048, 768, 128), (5, 4, 1024, 256, 32)])
def test_static_scratch_decode_matches_workspace_decode(cuda_device, tokens, top_k, hidden, inter, experts):
    from drama_b200 import _lib

    lib = _lib.library()
    fp8, keep, x, ids, w = _inputs(cuda_device, tokens, top_k, hidden, inter, experts, seed=tokens)
    expected = torch.empty_like(x)
    ws = _workspace_call(lib, fp8, x, ids, w, top_k, expected)
    torch.cuda.synchronize()
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(cuda_device)[0]
        lib.check(_static_call(lib, fp8, x, ids, w, top_k, out))
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info(cuda_device)[0]
        if call == 1:
            assert free_after >= free_before, f"static-scratch call allocated {free_before - free_after} bytes"
        assert_parity(np_f32(out), np_f32(expected), max_abs=MAX_ABS_TOL, rel=REL_TOL,
                      label=f"static-scratch decode, call {call + 1}")
        assert torch.equal(out.view(torch.int16), expected.view(torch.int16)), f"call {call + 1} differs in bits"
    del ws, keep


def test_static_scratch_decode_rejects_oversized_calls(cuda_device):
    from drama_b200 import _lib

    lib = _lib.library()
    hidden, inter, experts, top_k = 4096, 2048, 16, 8
    cap = lib.dll.drama_b200_static_scratch_bytes()
    tokens = 1
    while lib.dll.drama_b200_decode_workspace_bytes(tokens, top_k, hidden, inter) <= cap:
        tokens += 1
    fp8, keep, x, ids, w = _inputs(cuda_device, tokens, top_k, hidden, inter, experts, seed=3)
    out = torch.empty_like(x)
    assert _static_call(lib, fp8, x, ids, w, top_k, out) == -1
    message = lib.dll.drama_b200_error().decode()
    assert "static scratch" in message and str(cap) in message
    del keep
