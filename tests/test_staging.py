"""Staging arena: packed slot layout and argument checks (CPU), and the
copy-stream staging itself against the resident bank (GPU).

``StagingArena`` replaces ``_StagingPool`` (src/drama_low_vram/offload.py:
354-704). The GPU tests stage experts from a page-locked host store, run the
expert kernels on the staged slots and require the same bytes as the resident
bank gives, bit for bit: staging moves bytes and must not change a result.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

H, I, E = 256, 128, 12


def _bank(seed=5, experts=E):
    from drama_b200 import synthetic

    return synthetic.fp8_bank(experts, H, I, seed)


def test_packed_layout_offsets_are_16_byte_aligned():
    from drama_b200.staging import expert_bytes, role_layout

    layout = role_layout(2048, 768)
    assert [r[3] for r in layout] == [0, 3145728, 3146496, 4719360]
    assert expert_bytes(2048, 768) == 4719744
    assert all(offset % 16 == 0 for _, _, _, offset, _ in layout)


def test_packed_experts_round_trip_the_role_tensors():
    from drama_b200.staging import EXPERT_BUFFER_NAMES, PackedExperts

    bank = _bank()
    packed = PackedExperts.from_bank(bank)
    for name in EXPERT_BUFFER_NAMES:
        a, b = getattr(packed, name), bank[name]
        if a.dtype == torch.float8_e4m3fn:
            a, b = a.view(torch.uint8), b.view(torch.uint8)
        assert torch.equal(a, b)
    staged = packed.staged(3, start=2)
    assert staged.count == 3
    assert torch.equal(staged.w2_scale_inv, bank["w2_scale_inv"][2:5])


def test_arena_argument_checks_without_a_gpu():
    from drama_b200.staging import PackedExperts, StagingArena

    with pytest.raises(ValueError):
        StagingArena(0)
    with pytest.raises(ValueError):
        StagingArena(4, buffers=0)
    arena = StagingArena(4)
    store = PackedExperts.from_bank(_bank())
    with pytest.raises(ValueError, match="int64 CPU"):
        arena.stage(store, torch.tensor([1, 2], dtype=torch.int32))
    with pytest.raises(ValueError, match="Cannot stage 5"):
        arena.stage(store, torch.arange(5))
    with pytest.raises(RuntimeError, match="inside a session"):
        arena.stage(store, torch.arange(2))
    with pytest.raises(ValueError):
        PackedExperts(torch.zeros(2, 10, dtype=torch.uint8), H, I)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------


def _forward(staged, x, ids, w):
    from drama_b200.backend import B200ExpertBackend

    return B200ExpertBackend(prefill_min_pairs=1 << 30).forward(x, ids, w, staged)


def _assert_slots_hold(arena, bank, ids):
    """The first len(ids) slots hold those experts' four role tensors (padding not compared)."""
    for name, t in bank.items():
        got = getattr(arena, name)[:len(ids)].cpu()
        want = t[ids]
        if want.dtype == torch.float8_e4m3fn:
            got, want = got.view(torch.uint8), want.view(torch.uint8)
        assert torch.equal(got, want), name


@pytest.mark.gpu
@pytest.mark.parametrize("store_kind", ["packed-pinned", "roles-pinned", "pageable"])
def test_staged_experts_match_the_resident_bank(cuda_device, store_kind):
    from drama_b200 import synthetic
    from drama_b200.staging import PackedExperts, StagedExperts, StagingArena

    bank = _bank()
    if store_kind == "packed-pinned":
        store = PackedExperts.from_bank(bank, pin_memory=True)
    elif store_kind == "roles-pinned":
        class Store:
            pass
        store = Store()
        for name, t in bank.items():
            setattr(store, name, t.pin_memory())
    else:
        store = PackedExperts.from_bank(bank)
    resident = StagedExperts(**{n: t.to(cuda_device) for n, t in bank.items()})
    arena = StagingArena(6)
    x = synthetic.hidden_states(5, H, 1, device=cuda_device)
    for step, chosen in enumerate(([3, 4, 5, 9], [0, 11, 7], [3, 4, 5, 9], [2])):
        ids_host = torch.tensor(chosen, dtype=torch.int64)
        local, w = synthetic.uniform_routes(5, min(2, len(chosen)), len(chosen), seed=step, device=cuda_device)
        with arena.session(store, cuda_device):
            staged = arena.stage(store, ids_host)
            got = _forward(staged, x, local, w)
        want = _forward(StagedExperts(**{n: getattr(resident, n)[ids_host.to(cuda_device)]
                                         for n in bank}), x, local, w)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"{store_kind}, step {step}"
    _assert_slots_hold(arena._sets[0].arena, bank, [3, 4, 5, 9])
    # step 2 finds its ids already in its slot set (the reuse rule, offload.py:549-560)
    assert arena.stats.expert_loads == 8 and arena.stats.expert_cache_hits == 4
    if store_kind == "pageable":
        assert arena.stats.bounce_gathers == 3
    arena.close()


@pytest.mark.gpu
def test_reuse_rule_and_combine_resident(cuda_device):
    from drama_b200.staging import PackedExperts, StagedExperts, StagingArena

    bank = _bank()
    store = PackedExperts.from_bank(bank, pin_memory=True)
    resident = PackedExperts.from_bank(bank, device=cuda_device)
    arena = StagingArena(8, buffers=1)
    ids = torch.tensor([1, 6], dtype=torch.int64)
    with arena.session(store, cuda_device):
        arena.stage(store, ids)
    with arena.session(store, cuda_device):
        arena.stage(store, ids)                     # same ids, same store, same set: no copy
        combined = arena.combine_resident(2, resident, [0, 10, 4])
    torch.cuda.synchronize()
    assert arena.stats.expert_cache_hits == 2 and arena.stats.expert_loads == 2
    assert combined.count == 5
    _assert_slots_hold(arena._sets[0].arena, bank, [1, 6, 0, 10, 4])
    with pytest.raises(ValueError, match="capacity"):
        with arena.session(store, cuda_device):
            arena.combine_resident(6, resident, [0, 1, 2])
    arena.close()


@pytest.mark.gpu
def test_stage_copies_rejects_pageable_sources_before_copying(cuda_device):
    from drama_b200 import _lib

    lib = _lib.library()
    host = torch.zeros(4096, dtype=torch.uint8)            # pageable
    dev = torch.zeros(4096, dtype=torch.uint8, device=cuda_device)
    src = (ctypes.c_void_p * 1)(host.data_ptr())
    dst = (ctypes.c_void_p * 1)(dev.data_ptr())
    n = (ctypes.c_uint64 * 1)(4096)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    assert lib.dll.drama_b200_stage_copies(src, dst, n, 1, stream, None, None) == -1
    assert b"page-locked" in lib.dll.drama_b200_error()
    pinned = torch.arange(4096, dtype=torch.int64).to(torch.uint8).pin_memory()
    src = (ctypes.c_void_p * 2)(pinned.data_ptr(), pinned.data_ptr() + 1024)
    dst = (ctypes.c_void_p * 2)(dev.data_ptr(), dev.data_ptr() + 1024)
    n = (ctypes.c_uint64 * 2)(1024, 3072)                  # contiguous pieces: merged into one copy
    lib.check(lib.dll.drama_b200_stage_copies(src, dst, n, 2, stream, None, None))
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), pinned.numpy())
