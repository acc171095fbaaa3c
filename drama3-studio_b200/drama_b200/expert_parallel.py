"""Expert-parallel MoE decode over G GPUs (one process per GPU, NCCL all-to-all).

The reference runs every expert on one GPU (``ExpertOffloadManager``,
``src/drama_low_vram/offload.py:1016-1276``); here the E experts of each layer
are split into G contiguous blocks of E/G, rank r holding block r, and each
rank owns T/G of the T tokens. One layer on rank r:

1. ``drama_b200_ep_dispatch``: every (token, slot) pair's hidden row goes into
   the send block of the rank that owns its expert, tagged with the
   receiver-local expert id in its last 16 bytes (fixed ``capacity`` rows per
   destination, so nothing has to be known on the host and the step can be
   captured in a CUDA graph).
2. one all-to-all of the tagged rows (NCCL over NVLink).
3. ``drama_b200_fp8_expert_rows`` on the received rows: each row's bf16 down
   projection through the swap-AB grouped GEMMs, built for the few rows per
   expert of a decode batch (unused rows are dropped by their id).
4. all-to-all of the expert rows back to where they came from.
5. ``drama_b200_ep_combine``: route-weighted sum in slot order plus residual,
   ``h' = bf16(h + bf16(sum_s w_s * row_s))``, as one layer of the oracle's
   ``stack_layer`` with the routes given.

Every pair's arithmetic is the same whatever G is (rows are computed one by
one by the same kernels and summed in slot order by their owner), so the
result does not depend on the number of GPUs.

Two exchanges:

* ``exchange="p2p"`` (``PeerExchange``): the ranks map each other's receive and
  return buffers (CUDA IPC over NVLink). The dispatch kernel stores only the
  real rows straight into the owners' receive buffers; the second expert
  GEMM stores each result straight into the source's return buffer; epoch
  flags with bounded waits order the steps. No NCCL on the data path and no
  padding on the wire.
* ``exchange="nccl"``: fixed-capacity blocks through
  ``torch.distributed.all_to_all_single`` (a pluggable ``all_to_all(out, inp)``
  callable, which the CPU tests replace by gloo).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Sequence

import torch
from torch import Tensor

from . import _lib
from .backend import _fp8_bank

AllToAll = Callable[[Tensor, Tensor], None]
TAG = 8   # bf16 elements after each exchanged hidden row: the int32 local expert id and padding to 16 bytes


def shard_experts(experts: int, ranks: int, rank: int) -> range:
    """Global expert ids held by ``rank`` (contiguous blocks of E/G)."""
    if ranks < 1 or experts % ranks:
        raise ValueError(f"{experts} experts do not split evenly over {ranks} ranks")
    if not 0 <= rank < ranks:
        raise ValueError(f"rank {rank} outside [0, {ranks})")
    per = experts // ranks
    return range(rank * per, (rank + 1) * per)


def shard_tokens(tokens: int, ranks: int, rank: int) -> slice:
    """The token rows owned by ``rank`` (contiguous blocks of T/G)."""
    if tokens % ranks:
        raise ValueError(f"{tokens} tokens do not split evenly over {ranks} ranks")
    per = tokens // ranks
    return slice(rank * per, (rank + 1) * per)


def balanced_placement(counts: Sequence[int], ranks: int) -> list[int]:
    """Rank-major positions that even out the rows each rank receives.

    ``counts[e]`` is how many (token, slot) pairs expert e got (observed
    routes, as the reference's host-budget / hot-cache logic counts them).
    Experts are taken in decreasing count (ties by id) and each goes to the
    rank with the fewest rows so far that still has a free slot; its local id
    is its arrival order on that rank. Returns ``placement`` with
    ``placement[e] = rank * E/G + local``.
    """
    experts = len(counts)
    per = len(shard_experts(experts, ranks, 0))
    load = [0] * ranks
    fill = [0] * ranks
    placement = [0] * experts
    for e in sorted(range(experts), key=lambda x: (-int(counts[x]), x)):
        r = min((r for r in range(ranks) if fill[r] < per), key=lambda r: (load[r], r))
        placement[e] = r * per + fill[r]
        fill[r] += 1
        load[r] += int(counts[e])
    return placement


def experts_of_rank(placement: Sequence[int], ranks: int, rank: int) -> list[int]:
    """Global ids of the experts ``rank`` holds, in local-id order."""
    experts = len(placement)
    per = len(shard_experts(experts, ranks, rank))
    local = {p - rank * per: e for e, p in enumerate(placement) if p // per == rank}
    return [local[i] for i in range(per)]


class PeerExchange:
    """This rank's exchange buffers and the mapped buffers of every other rank.

    Created collectively (every rank of ``group`` at once): each rank
    allocates its receive / return / signal buffers in the library, the CUDA
    IPC handles go round with ``all_gather``, and each rank opens the others'.
    ``close`` (also collective) unmaps and frees them. Every flag wait of the
    exchange gives up after ``wait_ns`` nanoseconds (0: 2 s) and records it in
    the layer's status word 2.
    """

    def __init__(self, *, ranks: int, rank: int, capacity: int, hidden: int, experts: int, device,
                 group=None, wait_ns: int = 0) -> None:
        import torch.distributed as dist

        self.lib = lib = _lib.library()
        self.ranks, self.rank, self.group, self.device = ranks, rank, group, torch.device(device)
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        with torch.cuda.device(self.device):
            lib.check(lib.dll.drama_b200_ep_buffers_alloc(ranks, capacity, hidden, *[ctypes.byref(q) for q in ptrs]))
        self._own = [q.value for q in ptrs]
        recv, back, sig, counters = self._own
        handles = (ctypes.c_ubyte * 192)()
        for i, ptr in enumerate((recv, back, sig)):
            lib.check(lib.dll.drama_b200_ipc_handle(ptr, ctypes.addressof(handles) + 64 * i))
        mine = torch.tensor(list(bytes(handles)), dtype=torch.uint8, device=self.device)
        if ranks > 1:
            every = [torch.empty_like(mine) for _ in range(ranks)]
            dist.all_gather(every, mine, group=group)
            every = [bytes(t.cpu().tolist()) for t in every]
        else:
            every = [bytes(handles)]
        peers = _lib.EpPeers()
        peers.ranks, peers.rank, peers.capacity = ranks, rank, capacity
        peers.hidden, peers.experts = hidden, experts
        peers.wait_ns = wait_ns
        self._opened = []
        for r in range(ranks):
            if r == rank:
                peers.recv[r], peers.back[r], peers.signals[r] = recv, back, sig
                continue
            got = []
            for i in range(3):
                buf = (ctypes.c_ubyte * 64).from_buffer_copy(every[r][64 * i:64 * i + 64])
                q = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    lib.check(lib.dll.drama_b200_ipc_open(buf, ctypes.byref(q)))
                got.append(q.value)
                self._opened.append(q.value)
            peers.recv[r], peers.back[r], peers.signals[r] = got
        peers.epoch, peers.done = counters, counters + 64
        self.peers = peers

    def close(self) -> None:
        import torch.distributed as dist

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.ranks > 1:
            dist.barrier(group=self.group)      # no rank reads or writes a peer's buffers any more
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                self.lib.dll.drama_b200_ipc_close(ptr)
            if self.ranks > 1:
                dist.barrier(group=self.group)  # every mapping of this rank's buffers is gone
            self.lib.check(self.lib.dll.drama_b200_ep_buffers_free(*self._own))
        self._own = None
        self._opened = []


def nccl_all_to_all(group=None) -> AllToAll:
    """Equal-split all-to-all on ``group`` (rows travel as int32 words)."""
    import torch.distributed as dist

    def run(out: Tensor, inp: Tensor) -> None:
        dist.all_to_all_single(out, inp, group=group)

    return run


@dataclass
class ExchangeBuffers:
    """Per-rank scratch of one layer, reused by every layer and step."""

    send_rows: Tensor     # [G*cap, H + 8] bf16: hidden row, then the local expert id (int32) and padding
    pair_rows: Tensor     # [T_l*k] int32
    recv_rows: Tensor     # [G*cap, H + 8] bf16
    expert_rows: Tensor   # [G*cap, H] bf16
    back_rows: Tensor     # [G*cap, H] bf16
    status: Tensor        # [4] int32
    workspace: Tensor     # expert-rows workspace


class ExpertParallelMoE:
    """One rank's share of an expert-parallel FP8 MoE layer stack.

    ``banks[l]`` is this rank's slice of layer ``l``: an ``ExpertStore``-shaped
    FP8 bank (the four role tensors) of its E/G experts, indexed by local id:
    those ``shard_experts`` gives, or with ``placements[l]`` (int32 device
    tensor of rank-major positions, see ``balanced_placement``) those
    ``experts_of_rank`` gives.
    """

    def __init__(self, banks: Sequence, *, experts: int, top_k: int, tokens: int, ranks: int = 1, rank: int = 0,
                 all_to_all: AllToAll | None = None, capacity: int | None = None,
                 placements: Sequence[Tensor | None] | None = None, exchange: str = "nccl", group=None,
                 peer_wait_ns: int = 0, peer_exchange: PeerExchange | None = None) -> None:
        if not banks:
            raise ValueError("At least one layer bank is required")
        self.ranks, self.rank = ranks, rank
        self.experts, self.top_k = experts, top_k
        self.local_experts = len(shard_experts(experts, ranks, rank))
        self.tokens = tokens                        # tokens owned by this rank
        self.capacity = capacity if capacity is not None else tokens * top_k
        if self.capacity < 1:
            raise ValueError("Capacity must be positive")
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.exchange = exchange
        if exchange == "nccl" and ranks > 1 and all_to_all is None:
            raise ValueError("More than one rank needs an all_to_all")
        self.all_to_all = all_to_all
        first = banks[0]
        self.hidden = first.w13_weight.shape[-1]
        self.intermediate = first.w2_weight.shape[-1]
        self.device = first.w13_weight.device
        self._banks = []
        for bank in banks:
            if bank.w13_weight.shape[0] != self.local_experts:
                raise ValueError(f"Each bank must hold this rank's {self.local_experts} experts")
            self._banks.append(_fp8_bank(bank, self.hidden))
        if placements is not None and len(placements) != len(banks):
            raise ValueError("One placement (or None) per layer bank")
        self.placements = list(placements) if placements is not None else [None] * len(banks)
        for pl in self.placements:
            if pl is not None and (pl.dtype != torch.int32 or tuple(pl.shape) != (experts,)):
                raise ValueError(f"A placement is an int32 tensor of {experts} rank-major positions")
        self.lib = _lib.library()
        self.buffers = self._allocate()
        self.peer_exchange = None
        if exchange == "p2p" and peer_exchange is not None:
            # built by the caller (anything with a matching ``peers`` descriptor and ``close``)
            q = peer_exchange.peers
            if (q.ranks, q.rank, q.capacity, q.hidden, q.experts) != (ranks, rank, self.capacity, self.hidden, experts):
                raise ValueError("The peer exchange does not match this layer stack's ranks, capacity or shapes")
            self.peer_exchange = peer_exchange
        elif exchange == "p2p":
            self.peer_exchange = PeerExchange(ranks=ranks, rank=rank, capacity=self.capacity, hidden=self.hidden,
                                              experts=experts, device=self.device, group=group,
                                              wait_ns=peer_wait_ns)

    def _allocate(self) -> ExchangeBuffers:
        rows = self.ranks * self.capacity
        dev, H = self.device, self.hidden
        ws_bytes = self.lib.dll.drama_b200_expert_rows_workspace_bytes(rows, H, self.intermediate,
                                                                       self.local_experts)
        bf = dict(dtype=torch.bfloat16, device=dev)
        return ExchangeBuffers(
            send_rows=torch.zeros(rows, H + TAG, **bf),
            pair_rows=torch.empty(self.tokens * self.top_k, dtype=torch.int32, device=dev),
            recv_rows=torch.zeros(rows, H + TAG, **bf),
            expert_rows=torch.zeros(rows, H, **bf), back_rows=torch.zeros(rows, H, **bf),
            status=torch.zeros(4, dtype=torch.int32, device=dev),
            workspace=torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=dev))

    def _check_routes(self, h: Tensor, ids: Tensor, weights: Tensor) -> None:
        if h.dtype != torch.bfloat16 or tuple(h.shape) != (self.tokens, self.hidden) or not h.is_contiguous():
            raise ValueError(f"Hidden rows must be contiguous bf16 [{self.tokens}, {self.hidden}]")
        if tuple(ids.shape) != (self.tokens, self.top_k) or ids.dtype not in (torch.int32, torch.int64):
            raise ValueError(f"Expert IDs must be integer [{self.tokens}, {self.top_k}]")
        if tuple(weights.shape) != tuple(ids.shape) or not weights.is_floating_point():
            raise ValueError("Routing weights must match the expert IDs")

    def layer(self, h: Tensor, ids: Tensor, weights: Tensor, layer: int, out: Tensor | None = None) -> Tensor:
        """``bf16(h + moe(h))`` for this rank's tokens through layer ``layer``.

        ``ids`` are global expert ids, ``weights`` the route weights, both
        ``[T_l, k]`` and contiguous. ``out`` may be ``h`` (in place).
        """
        self._check_routes(h, ids, weights)
        out = torch.empty_like(h) if out is None else out
        if self.exchange == "p2p":
            return self._layer_p2p(h, ids, weights, layer, out)
        b = self.buffers
        self._dispatch(h, ids, self.placements[layer])
        if self.ranks > 1:
            self.all_to_all(b.recv_rows.view(torch.int32), b.send_rows.view(torch.int32))
            recv_rows = b.recv_rows
        else:
            recv_rows = b.send_rows
        self._run_experts(layer, recv_rows, b.expert_rows)
        if self.ranks > 1:
            self.all_to_all(b.back_rows.view(torch.int32), b.expert_rows.view(torch.int32))
            back = b.back_rows
        else:
            back = b.expert_rows
        self._combine(back, weights, h, out)
        return out

    def _layer_p2p(self, h: Tensor, ids: Tensor, weights: Tensor, layer: int, out: Tensor) -> Tensor:
        b, lib, peers = self.buffers, self.lib, ctypes.byref(self.peer_exchange.peers)
        stream = _lib.stream_handle(h.device)
        bank, _ = self._banks[layer]
        lib.check(lib.dll.drama_b200_ep_p2p_dispatch(
            peers, h.data_ptr(), self.tokens, ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype], self.top_k,
            _lib.ptr(self.placements[layer]), b.pair_rows.data_ptr(), b.status.data_ptr(), stream))
        lib.check(lib.dll.drama_b200_fp8_expert_rows_p2p(ctypes.byref(bank), peers, b.workspace.data_ptr(),
                                                         b.workspace.numel(), b.status.data_ptr(), stream))
        lib.check(lib.dll.drama_b200_ep_p2p_combine(
            peers, b.pair_rows.data_ptr(), weights.data_ptr(), _lib.DTYPE_CODES[weights.dtype], self.tokens,
            self.top_k, h.data_ptr(), out.data_ptr(), b.status.data_ptr(), stream))
        return out

    def close(self) -> None:
        """Release the peer exchange (collective across the ranks)."""
        if self.peer_exchange is not None:
            self.peer_exchange.close()
            self.peer_exchange = None

    def timed_out(self) -> bool:
        """Whether a peer wait of the layers so far gave up (synchronises)."""
        return bool(self.buffers.status[2].item())

    # The three device steps (CUDA kernels of this library).
    def _dispatch(self, h: Tensor, ids: Tensor, placement: Tensor | None = None) -> None:
        b, lib = self.buffers, self.lib
        lib.check(lib.dll.drama_b200_ep_dispatch(
            h.data_ptr(), self.tokens, self.hidden, ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype], self.top_k,
            self.experts, self.ranks, _lib.ptr(placement), self.capacity, b.send_rows.data_ptr(),
            self.hidden + TAG, None, b.pair_rows.data_ptr(), b.status.data_ptr(), _lib.stream_handle(h.device)))

    def _run_experts(self, layer: int, rows: Tensor, out: Tensor) -> None:
        """Down projections of the tagged ``rows`` (hidden values, then the local expert id)."""
        b, lib = self.buffers, self.lib
        bank, _ = self._banks[layer]
        lib.check(lib.dll.drama_b200_fp8_expert_rows(
            ctypes.byref(bank), rows.data_ptr(), self.hidden + TAG, rows.shape[0], None, _lib.I32, out.data_ptr(),
            b.workspace.data_ptr(), b.workspace.numel(), _lib.stream_handle(rows.device)))

    def _combine(self, back: Tensor, weights: Tensor, h: Tensor, out: Tensor) -> None:
        b, lib = self.buffers, self.lib
        lib.check(lib.dll.drama_b200_ep_combine(
            back.data_ptr(), back.shape[0], b.pair_rows.data_ptr(), weights.data_ptr(), _lib.DTYPE_CODES[weights.dtype],
            self.tokens, self.top_k, self.hidden, h.data_ptr(), out.data_ptr(), _lib.stream_handle(h.device)))

    def step(self, h: Tensor, routes: Sequence[tuple[Tensor, Tensor]]) -> Tensor:
        """All layers in order, in place on ``h``; ``routes[l] = (ids, weights)``."""
        for layer, (ids, weights) in enumerate(routes):
            self.layer(h, ids, weights, layer, out=h)
        return h

    def launches_per_layer(self) -> int:
        """Kernels of this library per layer."""
        # nccl: plan + pack, row prep + permute + 2 GEMMs, combine; p2p: dispatch, row prep + permute + 2 GEMMs,
        # combine
        return 6 if self.exchange == "p2p" else 7

    def dropped(self) -> tuple[int, int]:
        """(pairs with an out-of-range id, pairs over capacity) of the last layer (synchronises)."""
        s = self.buffers.status.tolist()
        return s[0], s[1]
