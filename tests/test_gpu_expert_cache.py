"""Expert cache as a page-locked staging source on a B200.

A registered layer window of the read-only mapping is copied by the staging
arena straight into HBM (no bounce gather); an unregistered layer still goes
through the bounce path. Both must give the bank's exact bytes and the same
expert outputs as the resident bank.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

H, I, E = 512, 256, 16


def _forward(staged, x, ids, w):
    from drama_b200.backend import B200ExpertBackend

    return B200ExpertBackend(prefill_min_pairs=1 << 30).forward(x, ids, w, staged)


def test_registered_cache_stages_without_bounce(cuda_device, tmp_path):
    from drama_b200 import synthetic
    from drama_b200.expert_cache import ExpertCacheFile, write_expert_cache
    from drama_b200.staging import StagedExperts, StagingArena, host_locked

    banks = [synthetic.fp8_bank(E, H, I, 300 + layer) for layer in range(3)]
    write_expert_cache(tmp_path / "cache", banks)
    cache = ExpertCacheFile.open(tmp_path / "cache", verify_data=True)
    locked = cache.register(0, 2)
    start, _ = cache.layer_span(0)
    off, size = cache.layer_span(1)
    assert locked >= off + size - start and cache.registered_layers == [(0, 2)]
    with pytest.raises(ValueError, match="overlap or adjoin"):
        cache.register(2, 1)  # its first page is the last page of layer 1
    assert all(host_locked(t) for t in cache.layer_buffers(1).values())
    # layer 2 starts inside the last registered page: its roles are not page-locked
    # (torch's is_pinned looks at the storage start and says they are)
    assert not any(host_locked(t) for t in cache.layer_buffers(2).values())
    assert cache.layer_buffers(2)["w13_weight"].is_pinned()
    # a copy that starts in the registered page but runs past it is refused before anything moves
    from drama_b200 import _lib

    lib = _lib.library()
    first = cache.layer_buffers(2)["w13_weight"][0]
    assert lib.host_locked(first.data_ptr(), 1)
    dev = torch.empty(first.numel(), dtype=torch.uint8, device=cuda_device)
    src = (ctypes.c_void_p * 1)(first.data_ptr())
    dst = (ctypes.c_void_p * 1)(dev.data_ptr())
    n = (ctypes.c_uint64 * 1)(first.numel())
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    assert lib.dll.drama_b200_stage_copies(src, dst, n, 1, stream, None, None) == -1
    assert b"not page-locked" in lib.dll.drama_b200_error()

    arena = StagingArena(6)
    x = synthetic.hidden_states(5, H, 1, device=cuda_device)
    chosen = [[3, 4, 5, 9], [0, 15, 7], [1, 2]]
    for layer in (0, 1, 2):
        store = cache.layer_store(layer)
        ids_host = torch.tensor(chosen[layer], dtype=torch.int64)
        local, w = synthetic.uniform_routes(5, 2, len(chosen[layer]), seed=layer, device=cuda_device)
        bounces = arena.stats.bounce_gathers
        with arena.session(store, cuda_device):
            staged = arena.stage(store, ids_host)
            got = _forward(staged, x, local, w)
            slots = {n: getattr(staged, n)[:len(chosen[layer])].clone() for n in banks[layer]}
        resident = StagedExperts(**{n: t[ids_host].to(cuda_device) for n, t in banks[layer].items()})
        want = _forward(resident, x, local, w)
        torch.cuda.synchronize()
        for name, t in banks[layer].items():
            a, b = slots[name].cpu(), t[ids_host]
            if b.dtype == torch.float8_e4m3fn:
                a, b = a.view(torch.uint8), b.view(torch.uint8)
            assert torch.equal(a, b), (layer, name)
        assert torch.equal(got, want), layer
        assert arena.stats.bounce_gathers == bounces + (1 if layer == 2 else 0), layer
    arena.close()
    cache.close()
    assert cache.registered_layers == []


def test_packed_checkpoint_stages_from_the_page_locked_file(cuda_device, tmp_path):
    """The packed safetensors checkpoint (shared_checkpoint.py's source) as an arena store."""
    from drama_b200 import synthetic
    from drama_b200.packed_checkpoint import PackedCheckpointExperts
    from drama_b200.staging import StagedExperts, StagingArena, host_locked
    from test_packed_checkpoint import write_packed

    banks = [synthetic.fp8_bank(E, H, I, 500 + layer) for layer in range(2)]
    packed = PackedCheckpointExperts.open(write_packed(tmp_path / "ckpt", banks))
    packed.register(0, 2)
    assert all(host_locked(t) for layer in range(2) for t in packed.layer_buffers(layer).values())
    arena = StagingArena(4)
    x = synthetic.hidden_states(3, H, 2, device=cuda_device)
    for layer, chosen in ((0, [2, 7, 11]), (1, [0, 15])):
        store = packed.layer_store(layer)
        ids_host = torch.tensor(chosen, dtype=torch.int64)
        local, w = synthetic.uniform_routes(3, 2, len(chosen), seed=layer, device=cuda_device)
        with arena.session(store, cuda_device):
            got = _forward(arena.stage(store, ids_host), x, local, w)
        resident = StagedExperts(**{n: t[ids_host].to(cuda_device) for n, t in banks[layer].items()})
        want = _forward(resident, x, local, w)
        torch.cuda.synchronize()
        assert torch.equal(got, want), layer
    assert arena.stats.bounce_gathers == 0
    arena.close()
    packed.close()
