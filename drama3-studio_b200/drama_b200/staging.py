"""Expert staging arena: page-locked host store -> HBM slots on a copy stream.

``StagingArena`` is a drop-in for the reference's ``_StagingPool``
(``src/drama_low_vram/offload.py:354-704``): the same ``session`` /
``stage`` / ``combine_resident`` / ``synchronize`` / ``close`` calls, the same
argument checks and error texts, the same reuse rule (same ids from the same
store -> no copy, ``offload.py:549-560``) and the same packed slot layout (one
uint8 row of ``expert_bytes`` per slot holding the four role tensors back to
back, ``offload.py:396-420``).

What differs is where the bytes move, which is the B200 part:

* The reference gathers the requested experts into one pinned host buffer and
  copies it on the compute stream (``offload.py:561-636``); the next stage
  waits on the host for that DMA (``_finish_copy``). Here a page-locked store
  (``PackedExperts.allocate(..., pin_memory=True)`` or any pinned tensors) is
  copied from directly, expert by expert, through ``drama_b200_stage_copies``
  on a dedicated copy stream, with consecutive experts merged into one DMA.
* The arena has ``buffers`` (default 2) slot sets used in turn, one per
  session. The copy stream waits only for the compute that last read the set
  it is about to overwrite, and the compute stream waits only for the copy it
  needs, so the transfer for the next layer runs while this layer computes.
* A pageable store still works: its rows are gathered into a pinned bounce
  buffer per slot set (``torch.index_select``, as the reference does) after a
  host wait for that set's previous DMA.
"""

from __future__ import annotations

import ctypes
import threading
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Iterator

import torch
from torch import Tensor

from . import _lib

EXPERT_BUFFER_NAMES = ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv")
FP8_DTYPE = torch.float8_e4m3fn
BLOCK = 128


def host_locked(t: Tensor) -> bool:
    """A host tensor whose own byte range is page-locked (torch's ``is_pinned``
    looks only at the start of the whole storage, which misleads for views into
    a partly registered mapping)."""
    if t.device.type != "cpu" or t.numel() == 0:
        return False
    if not torch.cuda.is_available():
        return t.is_pinned()
    return _lib.library().host_locked(t.data_ptr(), t.numel() * t.element_size())


def role_layout(hidden: int, intermediate: int) -> list[tuple[str, torch.dtype, tuple[int, ...], int, int]]:
    """(name, dtype, per-expert shape, byte offset, bytes) of each role in a packed slot."""
    roles = [
        ("w13_weight", FP8_DTYPE, (2 * intermediate, hidden)),
        ("w13_scale_inv", torch.float32, (2 * intermediate // BLOCK, hidden // BLOCK)),
        ("w2_weight", FP8_DTYPE, (hidden, intermediate)),
        ("w2_scale_inv", torch.float32, (hidden // BLOCK, intermediate // BLOCK)),
    ]
    out, offset = [], 0
    for name, dtype, shape in roles:
        nbytes = torch.Size(shape).numel() * torch.empty((), dtype=dtype).element_size()
        out.append((name, dtype, shape, offset, nbytes))
        offset += nbytes
    return out


def expert_bytes(hidden: int, intermediate: int) -> int:
    """Bytes of one packed slot: the four roles, padded to a multiple of 16.

    At the model's shapes the roles already sum to a multiple of 16
    (4,719,744 bytes at hidden 2048, intermediate 768), so the slot is exactly
    the reference's packed row; the padding only keeps every slot's weight
    rows on 16-byte boundaries at other shapes.
    """
    return (sum(r[4] for r in role_layout(hidden, intermediate)) + 15) // 16 * 16


@dataclass(frozen=True)
class StagedExperts:
    """The four role views of ``count`` staged slots (``offload.py:175-184``)."""

    w13_weight: Tensor
    w13_scale_inv: Tensor
    w2_weight: Tensor
    w2_scale_inv: Tensor

    @property
    def count(self) -> int:
        return self.w13_weight.shape[0]


class PackedExperts:
    """``[experts, expert_bytes]`` uint8 rows with the four role views.

    Used both for the host store (page-locked, so H2D copies can be
    asynchronous) and for the device arena. Every role starts on a 16-byte
    boundary inside a row (3,145,728 / 768 / 1,572,864 / 384 bytes at hidden
    2048, intermediate 768), which the kernels' 16-byte loads need.
    """

    def __init__(self, raw: Tensor, hidden: int, intermediate: int) -> None:
        if raw.dtype != torch.uint8 or raw.ndim != 2 or raw.shape[1] != expert_bytes(hidden, intermediate):
            raise ValueError("Packed experts must be a [experts, expert_bytes] uint8 tensor")
        if not raw.is_contiguous():
            raise ValueError("Packed experts must be contiguous")
        self.raw = raw
        self.hidden = hidden
        self.intermediate = intermediate
        self.num_experts = raw.shape[0]
        self.expert_bytes = raw.shape[1]
        self.nbytes = raw.numel()
        for name, dtype, shape, offset, nbytes in role_layout(hidden, intermediate):
            view = raw.narrow(1, offset, nbytes).view(dtype).view(self.num_experts, *shape)
            setattr(self, name, view)

    @classmethod
    def allocate(cls, experts: int, hidden: int, intermediate: int, *, device="cpu",
                 pin_memory: bool = False) -> "PackedExperts":
        dev = torch.device(device)
        options = {"pin_memory": pin_memory} if dev.type == "cpu" else {}
        raw = torch.empty((experts, expert_bytes(hidden, intermediate)), dtype=torch.uint8, device=dev, **options)
        return cls(raw, hidden, intermediate)

    @classmethod
    def from_bank(cls, bank, *, device="cpu", pin_memory: bool = False) -> "PackedExperts":
        """Pack an ``ExpertStore``-shaped bank (attributes or dict of the four roles)."""
        get = bank.__getitem__ if isinstance(bank, dict) else (lambda n: getattr(bank, n))
        experts, gate_up, hidden = get("w13_weight").shape
        packed = cls.allocate(experts, hidden, gate_up // 2, device=device, pin_memory=pin_memory)
        for name in EXPERT_BUFFER_NAMES:
            getattr(packed, name).copy_(get(name))
        return packed

    def is_pinned(self) -> bool:
        return host_locked(self.raw)

    def staged(self, count: int | None = None, start: int = 0) -> StagedExperts:
        stop = self.num_experts if count is None else start + count
        return StagedExperts(**{n: getattr(self, n)[start:stop] for n in EXPERT_BUFFER_NAMES})


@dataclass
class StagingStatistics:
    """The staging counters of ``OffloadStatistics`` (``offload.py:301-352``) this arena feeds."""

    staging_calls: int = 0
    expert_loads: int = 0
    expert_cache_hits: int = 0
    staged_bytes: int = 0
    h2d_bytes: int = 0
    h2d_copy_calls: int = 0
    bounce_gathers: int = 0
    peak_staged_experts: int = 0
    device_buffer_bytes: int = 0
    pinned_bytes: int = 0


@dataclass
class _SlotSet:
    arena: PackedExperts
    copy_done: torch.cuda.Event
    compute_done: torch.cuda.Event
    bounce: PackedExperts | None = None
    loaded_ids: Tensor | None = None
    loaded_store: int | None = None
    copy_pending: bool = False
    compute_pending: bool = False


class StagingArena:
    """``_StagingPool`` replacement with copy-stream staging into rotating slot sets."""

    def __init__(self, capacity: int, *, buffers: int = 2, copy_stream: torch.cuda.Stream | None = None,
                 stats: StagingStatistics | None = None) -> None:
        if capacity < 1:
            raise ValueError("Staging capacity must be positive")
        if buffers < 1:
            raise ValueError("A staging arena needs at least one slot set")
        self.capacity = capacity
        self.buffers = buffers
        self.stats = stats or StagingStatistics()
        self._lock = threading.Lock()
        self._sets: list[_SlotSet] = []
        self._target: torch.device | None = None
        self._shape: tuple[int, int] | None = None
        self._copy_stream = copy_stream
        self._turn = -1
        self._active: _SlotSet | None = None
        self._slot_index: dict[tuple[int, ...], Tensor] = {}
        # Set by the reference manager's configure_host_residency
        # (offload.py:1344-1345): a RAM tier that decides where each expert's
        # host bytes come from, and the layer of each store.
        self.host_residency = None
        self.host_store_layers: dict[tuple[int, ...], int] = {}

    # -- allocation -------------------------------------------------------
    def _allocate(self, hidden: int, intermediate: int, device: torch.device) -> None:
        shape = (hidden, intermediate)
        if self._target is not None:
            if self._target != device or self._shape != shape:
                raise ValueError("One offload manager supports one compute device and one expert shape")
            return
        if device.type != "cuda":
            raise RuntimeError("drama_b200 staging needs a CUDA device")
        with torch.cuda.device(device):
            if self._copy_stream is None:
                self._copy_stream = torch.cuda.Stream(device)
            for _ in range(self.buffers):
                arena = PackedExperts.allocate(self.capacity, hidden, intermediate, device=device)
                done, computed = torch.cuda.Event(), torch.cuda.Event()
                done.record(self._copy_stream)          # materialise both events
                computed.record(torch.cuda.current_stream(device))
                self._sets.append(_SlotSet(arena, done, computed))
        self._target = device
        self._shape = shape
        self.stats.device_buffer_bytes = sum(s.arena.nbytes for s in self._sets)

    # -- the _StagingPool API ----------------------------------------------
    @contextmanager
    def session(self, store, device: torch.device) -> Iterator[None]:
        """Take the next slot set for this session's ``stage`` calls.

        On exit the compute stream's position is recorded for that set, so
        the copy that next overwrites it waits for exactly this session's
        expert kernels and nothing else.
        """
        device = torch.device(device)
        with self._lock:
            hidden, intermediate = _store_shape(store)
            self._allocate(hidden, intermediate, device)
            self._turn = (self._turn + 1) % self.buffers
            slot_set = self._sets[self._turn]
            self._active = slot_set
            stream = torch.cuda.current_stream(device)
            slot_set.arena.raw.record_stream(stream)
            try:
                yield
            finally:
                slot_set.compute_done.record(stream)
                slot_set.compute_pending = True
                self._active = None

    def stage(self, store, expert_ids: Tensor) -> StagedExperts:
        """Copy ``store``'s experts ``expert_ids`` into slots ``0..n-1`` of the session's set.

        Returns the slot views; the current stream is made to wait for the
        copy, so kernels enqueued after this call see the bytes.
        """
        if expert_ids.device.type != "cpu" or expert_ids.dtype != torch.int64:
            raise ValueError("Staging IDs must be an int64 CPU tensor")
        count = expert_ids.numel()
        if not 0 < count <= self.capacity:
            raise ValueError(f"Cannot stage {count} experts in {self.capacity} slots")
        slot_set = self._active
        if slot_set is None or self._target is None:
            raise RuntimeError("Use the staging pool inside a session")
        if bool(((expert_ids < 0) | (expert_ids >= _store_experts(store))).any()):
            raise ValueError("Expert IDs are outside the host store")
        store_key = id(store)
        compute = torch.cuda.current_stream(self._target)
        if (slot_set.loaded_ids is not None and slot_set.loaded_store == store_key
                and torch.equal(slot_set.loaded_ids, expert_ids)):
            self.stats.expert_cache_hits += count
            if slot_set.copy_pending:
                compute.wait_event(slot_set.copy_done)
            return slot_set.arena.staged(count)
        src, dst, nbytes = self._plan_copies(store, expert_ids, slot_set)
        lib = _lib.library()
        n = len(src)
        arr_src = (ctypes.c_void_p * n)(*src)
        arr_dst = (ctypes.c_void_p * n)(*dst)
        arr_bytes = (ctypes.c_uint64 * n)(*nbytes)
        wait = slot_set.compute_done.cuda_event if slot_set.compute_pending else None
        lib.check(lib.dll.drama_b200_stage_copies(arr_src, arr_dst, arr_bytes, n, self._copy_stream.cuda_stream,
                                                  wait, slot_set.copy_done.cuda_event))
        slot_set.copy_pending = True
        compute.wait_event(slot_set.copy_done)
        copied = sum(nbytes)
        self.stats.staging_calls += 1
        self.stats.expert_loads += count
        self.stats.staged_bytes += copied
        self.stats.h2d_bytes += copied
        self.stats.h2d_copy_calls += 1
        self.stats.peak_staged_experts = max(self.stats.peak_staged_experts, count)
        slot_set.loaded_ids = expert_ids.clone()
        slot_set.loaded_store = store_key
        return slot_set.arena.staged(count)

    def combine_resident(self, cold_count: int, resident, resident_slots: list[int]) -> StagedExperts:
        """Append GPU-resident experts after the staged cold prefix (``offload.py:653-679``)."""
        count = cold_count + len(resident_slots)
        if cold_count < 1 or not resident_slots or count > self.capacity:
            raise ValueError("Combined expert bank must fit the staging capacity")
        slot_set = self._active
        if slot_set is None or self._target is None:
            raise RuntimeError("Stage cold experts before combining the bank")
        key = tuple(resident_slots)
        slots = self._slot_index.get(key)
        if slots is None:
            # A pageable H2D copy may wait for the device; cache the index so
            # the host keeps running ahead of the copy and compute streams.
            slots = torch.tensor(resident_slots, dtype=torch.int64, device=self._target)
            self._slot_index[key] = slots
        arena = slot_set.arena
        for name in EXPERT_BUFFER_NAMES:
            source = getattr(resident, name)
            target = getattr(arena, name)[cold_count:count]
            if source.dtype == FP8_DTYPE:
                source, target = source.view(torch.uint8), target.view(torch.uint8)
            torch.index_select(source, 0, slots, out=target)
        self.stats.peak_staged_experts = max(self.stats.peak_staged_experts, count)
        return arena.staged(count)

    def synchronize(self) -> None:
        with self._lock:
            for s in self._sets:
                s.copy_done.synchronize()
                s.compute_done.synchronize()
                s.copy_pending = s.compute_pending = False

    def close(self) -> None:
        self.synchronize()
        with self._lock:
            self._sets.clear()
            self._slot_index.clear()
            self._target = None
            self._shape = None
            self._active = None
            self.stats.device_buffer_bytes = 0
            self.stats.pinned_bytes = 0

    # -- copy planning -------------------------------------------------------
    def _plan_copies(self, store, expert_ids: Tensor, slot_set: _SlotSet):
        raw = store.raw if isinstance(store, PackedExperts) else store.w13_weight
        if raw.device.type != "cpu":
            raise ValueError("The staging store must live in host memory")
        if self.host_residency is not None and self.host_residency.enabled:
            return self._bounce(store, expert_ids, slot_set, residency=True)
        ids = expert_ids.tolist()
        arena = slot_set.arena
        packed = store if isinstance(store, PackedExperts) else getattr(store, "packed", None)
        if packed is not None and packed.is_pinned():
            base_src, base_dst, row = packed.raw.data_ptr(), arena.raw.data_ptr(), arena.expert_bytes
            return ([base_src + e * row for e in ids], [base_dst + i * row for i in range(len(ids))],
                    [row] * len(ids))
        if packed is None and all(host_locked(getattr(store, n)) for n in EXPERT_BUFFER_NAMES):
            src, dst, nbytes = [], [], []
            for name, _, _, offset, size in role_layout(arena.hidden, arena.intermediate):
                role = getattr(store, name)
                base, stride = role.data_ptr(), role.stride(0) * role.element_size()
                if not role[0].is_contiguous():
                    break
                for i, e in enumerate(ids):
                    src.append(base + e * stride)
                    dst.append(arena.raw.data_ptr() + i * arena.expert_bytes + offset)
                    nbytes.append(size)
            else:
                return src, dst, nbytes
        return self._bounce(store, expert_ids, slot_set)

    def _bounce(self, store, expert_ids: Tensor, slot_set: _SlotSet, *, residency: bool = False):
        """Gather into a pinned bounce buffer first (``offload.py:561-594``): the
        host-residency tier's own gather when one is configured, else
        ``index_select`` from a pageable store."""
        arena = slot_set.arena
        if slot_set.bounce is None:
            slot_set.bounce = PackedExperts.allocate(self.capacity, arena.hidden, arena.intermediate,
                                                     pin_memory=True)
            self.stats.pinned_bytes += slot_set.bounce.nbytes
        if slot_set.copy_pending:
            slot_set.copy_done.synchronize()     # the bounce rows are still being read by the last DMA
        count = expert_ids.numel()
        if residency:
            key = tuple(id(getattr(store, name)) for name in EXPERT_BUFFER_NAMES)
            layer = self.host_store_layers.get(key)
            if layer is None:
                raise RuntimeError("Expert buffers changed; reconfigure host residency")
            self.host_residency.copy_to(layer, expert_ids,
                                        {name: getattr(slot_set.bounce, name) for name in EXPERT_BUFFER_NAMES},
                                        observe=False)
        elif isinstance(store, PackedExperts):
            torch.index_select(store.raw, 0, expert_ids, out=slot_set.bounce.raw[:count])
        else:
            for name in EXPERT_BUFFER_NAMES:
                source = getattr(store, name)
                target = getattr(slot_set.bounce, name)[:count]
                if source.dtype == FP8_DTYPE:
                    source, target = source.view(torch.uint8), target.view(torch.uint8)
                target.copy_(torch.index_select(source, 0, expert_ids))
        self.stats.bounce_gathers += 1
        row = arena.expert_bytes
        return ([slot_set.bounce.raw.data_ptr()], [arena.raw.data_ptr()], [row * count])


def _store_shape(store) -> tuple[int, int]:
    if isinstance(store, PackedExperts):
        return store.hidden, store.intermediate
    experts, gate_up, hidden = store.w13_weight.shape
    return hidden, gate_up // 2


def _store_experts(store) -> int:
    return store.num_experts if isinstance(store, PackedExperts) else store.w13_weight.shape[0]
