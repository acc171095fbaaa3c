"""Expert-parallel kernels and the EP layer stack on the GPU.

* ``drama_b200_ep_dispatch`` / ``drama_b200_ep_combine`` against CPU
  restatements of their contracts: exact (indices, bytes, and the fp32
  slot-order sum, which has one rounding order).
* One rank (G = 1) of ``ExpertParallelMoE`` against ``fp8_expert_rows`` per
  (token, slot) row with the combine restated in torch (bit for bit: the same
  kernel sees the same rows) and against the oracle's dequant path (the
  north_star tolerance).
* G = 2 and 4 emulated on one GPU (every rank's steps run in turn, the
  all-to-all done by copying blocks) and, when two GPUs are present, G = 2
  over NCCL: the result must equal G = 1 bit for bit.
* The peer exchange's bounded waits: a rank that never publishes its flags
  makes the other rank's waits give up after the limit it set, with the
  timeout recorded in the status word and no fault.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from helpers import assert_parity, np_bank, np_f32
from oracle import restate as R

pytestmark = pytest.mark.gpu

E, H, I, K, T, LAYERS = 16, 512, 256, 4, 32, 2


class Bank:
    def __init__(self, d):
        self.__dict__.update(d)


def _inputs(device):
    from drama_b200 import synthetic

    banks = [synthetic.fp8_bank(E, H, I, seed=40 + l, device=device, chunk=E) for l in range(LAYERS)]
    routes = []
    for l in range(LAYERS):
        ids, w = synthetic.zipf_routes(T, K, E, seed=50 + l, device=device)
        routes.append((ids.to(torch.int64).contiguous(), w.to(torch.bfloat16).contiguous()))
    h = synthetic.hidden_states(T, H, seed=60, device=device)
    return banks, routes, h


def _placements(routes, ranks, device):
    from drama_b200.expert_parallel import balanced_placement

    return [torch.tensor(balanced_placement(torch.bincount(ids.reshape(-1).cpu(), minlength=E).tolist(), ranks),
                         dtype=torch.int32, device=device) for ids, _ in routes]


def _model(banks, ranks=1, rank=0, tokens=T, all_to_all=None, capacity=None, placements=None, exchange="nccl",
           peer_exchange=None):
    from drama_b200.expert_parallel import ExpertParallelMoE, experts_of_rank, shard_experts

    local = []
    for l, b in enumerate(banks):
        held = experts_of_rank(placements[l].tolist(), ranks, rank) if placements is not None else \
            list(shard_experts(E, ranks, rank))
        local.append(Bank({n: v[held] for n, v in b.items()}))
    return ExpertParallelMoE(local, experts=E, top_k=K, tokens=tokens, ranks=ranks, rank=rank,
                             all_to_all=all_to_all or (lambda o, i: None), capacity=capacity, placements=placements,
                             exchange=exchange, peer_exchange=peer_exchange)


def _dispatch_restated(h, ids, experts, ranks, cap, placement=None):
    per = experts // ranks
    pos = list(range(experts)) if placement is None else placement
    send_ids = np.full(ranks * cap, per, np.int32)
    pair_rows = np.full(ids.size, -1, np.int32)
    fill = [0] * ranks
    dropped = overflow = 0
    for p, e in enumerate(ids.reshape(-1).tolist()):
        if not 0 <= e < experts:
            dropped += 1
            continue
        d = pos[e] // per
        if fill[d] >= cap:
            overflow += 1
            continue
        row = d * cap + fill[d]
        fill[d] += 1
        send_ids[row] = pos[e] - d * per
        pair_rows[p] = row
    return send_ids, pair_rows, (dropped, overflow)


@pytest.mark.parametrize("ranks,cap,permuted,tagged", [(1, 37 * 8, False, False), (2, 37 * 8, False, True),
                                                       (8, 37 * 8, False, False), (4, 20, False, True),
                                                       (4, 37 * 8, True, True)])
def test_dispatch_matches_its_restatement(cuda_device, ranks, cap, permuted, tagged):
    from drama_b200 import _lib

    lib = _lib.library()
    gen = torch.Generator().manual_seed(ranks * 100 + cap)
    tokens, top_k, experts = 37, 8, 128
    ids = torch.randint(-2, experts + 3, (tokens, top_k), generator=gen)
    h = torch.randn(tokens, 256, generator=gen).to(torch.bfloat16).to(cuda_device)
    stride = 256 + 8 if tagged else 256
    send_rows = torch.zeros(ranks * cap, stride, dtype=torch.bfloat16, device=cuda_device)
    send_ids = torch.empty(ranks * cap, dtype=torch.int32, device=cuda_device)
    pair_rows = torch.empty(tokens * top_k, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    placement = torch.randperm(experts, generator=gen).to(torch.int32) if permuted else None
    d_place = placement.to(cuda_device) if permuted else None
    for dtype in (torch.int64, torch.int32):
        d_ids = ids.to(dtype).to(cuda_device)
        lib.check(lib.dll.drama_b200_ep_dispatch(
            h.data_ptr(), tokens, 256, d_ids.data_ptr(), _lib.DTYPE_CODES[dtype], top_k, experts, ranks,
            _lib.ptr(d_place), cap, send_rows.data_ptr(), stride, None if tagged else send_ids.data_ptr(),
            pair_rows.data_ptr(), status.data_ptr(),
            _lib.stream_handle(cuda_device)))
        torch.cuda.synchronize()
        want_ids, want_rows, (dropped, overflow) = _dispatch_restated(
            h, ids.numpy(), experts, ranks, cap, placement.tolist() if permuted else None)
        got_ids = send_rows.view(torch.int32)[:, 128] if tagged else send_ids
        assert np.array_equal(got_ids.cpu().numpy(), want_ids)
        assert np.array_equal(pair_rows.cpu().numpy(), want_rows)
        assert status[:2].tolist() == [dropped, overflow]
        for p, row in enumerate(want_rows.tolist()):
            if row >= 0:
                assert torch.equal(send_rows[row, :256], h[p // top_k])


@pytest.mark.parametrize("wdtype,residual", [(torch.bfloat16, True), (torch.float32, False)])
def test_combine_matches_its_restatement(cuda_device, wdtype, residual):
    from drama_b200 import _lib

    lib = _lib.library()
    gen = torch.Generator().manual_seed(7)
    tokens, top_k, hidden, nrows = 19, 8, 512, 200
    rows = torch.randn(nrows, hidden, generator=gen).to(torch.bfloat16)
    pair_rows = torch.randint(-1, nrows, (tokens * top_k,), generator=gen, dtype=torch.int32)
    w = torch.rand(tokens, top_k, generator=gen).to(wdtype)
    h = torch.randn(tokens, hidden, generator=gen).to(torch.bfloat16)
    acc = torch.zeros(tokens, hidden)
    for s in range(top_k):
        r = pair_rows.view(tokens, top_k)[:, s].long()
        take = (r >= 0).float()[:, None]
        prod = rows[r.clamp_min(0)].float() * w[:, s].float()[:, None]
        acc = acc + prod * take                      # a skipped pair adds +0.0
    want = acc.to(torch.bfloat16)
    if residual:
        want = (h.float() + want.float()).to(torch.bfloat16)
    d = {n: t.to(cuda_device) for n, t in dict(rows=rows, pair_rows=pair_rows, w=w, h=h).items()}
    out = torch.empty(tokens, hidden, dtype=torch.bfloat16, device=cuda_device)
    lib.check(lib.dll.drama_b200_ep_combine(
        d["rows"].data_ptr(), nrows, d["pair_rows"].data_ptr(), d["w"].data_ptr(), _lib.DTYPE_CODES[wdtype], tokens,
        top_k, hidden, d["h"].data_ptr() if residual else None, out.data_ptr(), _lib.stream_handle(cuda_device)))
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), want)


def _reference_stack(banks, routes, h):
    """fp8_expert_rows per (token, slot) row, then the slot-order fp32 combine and residual in torch."""
    from drama_b200.backend import fp8_expert_rows

    x = h.clone()
    for bank, (ids, w) in zip(banks, routes):
        rows = fp8_expert_rows(x.repeat_interleave(K, dim=0), ids.reshape(-1), Bank(bank)).float()
        acc = torch.zeros(T, H, device=x.device)
        for s in range(K):
            acc = acc + rows[s::K] * w[:, s].float()[:, None]
        x = (x.float() + acc.to(torch.bfloat16).float()).to(torch.bfloat16)
    return x


def test_single_rank_matches_expert_rows_and_the_oracle(cuda_device):
    banks, routes, h = _inputs(cuda_device)
    model = _model(banks)
    x = h.clone()
    model.step(x, routes)
    torch.cuda.synchronize()
    assert model.dropped() == (0, 0)
    assert torch.equal(x, _reference_stack(banks, routes, h))
    y = np_f32(h)
    for bank, (ids, w) in zip(banks, routes):
        y = R.round_bf16(y + R.fp8_dequant_forward(y, ids.cpu().numpy(), np_f32(w), np_bank(bank)))
    assert_parity(np_f32(x), y, label="EP G=1 vs oracle stack")


def _emulated(banks, routes, h, ranks, placements=None):
    """G ranks on one GPU: each rank's device steps in turn, blocks copied for the all-to-all."""
    from drama_b200.expert_parallel import shard_tokens

    tl = T // ranks
    models = [_model(banks, ranks, r, tokens=tl, placements=placements) for r in range(ranks)]
    cap = models[0].capacity
    xs = [h[shard_tokens(T, ranks, r)].clone() for r in range(ranks)]
    for layer, (ids, w) in enumerate(routes):
        rs = [(ids[shard_tokens(T, ranks, r)].contiguous(), w[shard_tokens(T, ranks, r)].contiguous())
              for r in range(ranks)]
        for r, m in enumerate(models):
            m._dispatch(xs[r], rs[r][0], m.placements[layer])
        for r, m in enumerate(models):
            for s, src in enumerate(models):
                m.buffers.recv_rows[s * cap:(s + 1) * cap] = src.buffers.send_rows[r * cap:(r + 1) * cap]
        for m in models:
            m._run_experts(layer, m.buffers.recv_rows, m.buffers.expert_rows)
        for r, m in enumerate(models):
            for s, src in enumerate(models):
                m.buffers.back_rows[s * cap:(s + 1) * cap] = src.buffers.expert_rows[r * cap:(r + 1) * cap]
        for r, m in enumerate(models):
            m._combine(m.buffers.back_rows, rs[r][1], xs[r], xs[r])
    return torch.cat(xs)


@pytest.mark.parametrize("ranks,balanced", [(2, False), (4, False), (4, True)])
def test_emulated_ranks_equal_one_rank_bit_for_bit(cuda_device, ranks, balanced):
    banks, routes, h = _inputs(cuda_device)
    single = _model(banks)
    x = h.clone()
    single.step(x, routes)
    got = _emulated(banks, routes, h, ranks, _placements(routes, ranks, cuda_device) if balanced else None)
    torch.cuda.synchronize()
    assert torch.equal(got, x)


def test_peer_exchange_on_one_rank_equals_the_nccl_path(cuda_device):
    """The NVLink exchange (here a rank writing to itself) leaves every bit as it was."""
    banks, routes, h = _inputs(cuda_device)
    ref = _model(banks)
    x = h.clone()
    ref.step(x, routes)
    p2p = _model(banks, exchange="p2p")
    y = h.clone()
    p2p.step(y, routes)
    g_in = h.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        p2p.step(g_in, routes)
    g_in.copy_(h)
    graph.replay()
    torch.cuda.synchronize()
    assert not p2p.timed_out()
    assert torch.equal(y, x) and torch.equal(g_in, x)
    del graph
    p2p.close()


class _LoopbackExchange:
    """Every rank's exchange buffers allocated by this process on one GPU, driven as rank ``rank`` alone."""

    def __init__(self, ranks, rank, capacity, device, wait_ns):
        import ctypes

        from drama_b200 import _lib

        self.lib = lib = _lib.library()
        self.device = device
        peers = _lib.EpPeers()
        peers.ranks, peers.rank, peers.capacity, peers.hidden, peers.experts = ranks, rank, capacity, H, E
        self.sets = []
        with torch.cuda.device(device):
            for r in range(ranks):
                ptrs = [ctypes.c_void_p() for _ in range(4)]
                lib.check(lib.dll.drama_b200_ep_buffers_alloc(ranks, capacity, H, *[ctypes.byref(q) for q in ptrs]))
                self.sets.append([q.value for q in ptrs])
                peers.recv[r], peers.back[r], peers.signals[r] = self.sets[-1][:3]
        peers.epoch, peers.done = self.sets[rank][3], self.sets[rank][3] + 64
        peers.wait_ns = wait_ns
        self.peers = peers

    def close(self):
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for bufs in self.sets:
                self.lib.check(self.lib.dll.drama_b200_ep_buffers_free(*bufs))
        self.sets = []


def test_peer_waits_run_out_when_a_rank_never_publishes(cuda_device):
    """Rank 1 of two never runs: rank 0's row prep waits for rank 1's dispatch
    flag and its combine for rank 1's return flag, flags that nothing sets.
    Both waits give up after the 20 ms asked for, the kernels return, status
    word 2 records both (bit 1: row prep, bit 2: combine) and the GPU goes on
    working: the same layer on one rank afterwards gives its usual bits."""
    import ctypes
    import time

    from drama_b200 import _lib

    banks, routes, h = _inputs(cuda_device)
    tl = T // 2
    ids, w = routes[0][0][:tl].contiguous(), routes[0][1][:tl].contiguous()
    single = _model(banks)
    expected = h.clone()
    single.layer(expected, routes[0][0], routes[0][1], 0, out=expected)

    exchange = _LoopbackExchange(2, 0, tl * K, cuda_device, wait_ns=20_000_000)
    model = _model(banks, ranks=2, rank=0, tokens=tl, exchange="p2p", peer_exchange=exchange)
    x = h[:tl].clone()
    torch.cuda.synchronize()
    start = time.monotonic()
    model.layer(x, ids, w, 0, out=x)
    torch.cuda.synchronize()
    elapsed = time.monotonic() - start
    assert model.timed_out()
    assert int(model.buffers.status[2].item()) == 1 | 2
    assert elapsed < 1.5, f"the waits took {elapsed:.2f} s; the limit asked for was 20 ms (default 2 s each)"

    lib = _lib.library()
    exchange.peers.wait_ns = -1
    bad = lib.dll.drama_b200_ep_p2p_combine(
        ctypes.byref(exchange.peers), model.buffers.pair_rows.data_ptr(), w.data_ptr(), _lib.BF16, tl, K,
        x.data_ptr(), x.data_ptr(), model.buffers.status.data_ptr(), _lib.stream_handle(cuda_device))
    assert bad == -1 and "wait_ns" in lib.dll.drama_b200_error().decode()
    model.close()

    again = h.clone()
    single.layer(again, routes[0][0], routes[0][1], 0, out=again)
    torch.cuda.synchronize()
    assert torch.equal(again, expected)


def test_small_capacity_drops_and_counts_overflow(cuda_device):
    banks, routes, h = _inputs(cuda_device)
    model = _model(banks, capacity=8)
    x = h.clone()
    model.layer(x, routes[0][0], routes[0][1], 0, out=x)
    torch.cuda.synchronize()
    dropped, overflow = model.dropped()
    assert dropped == 0 and overflow == T * K - 8


def _nccl_rank(rank, world, port, out_dir):
    import torch.distributed as dist

    from drama_b200.expert_parallel import nccl_all_to_all, shard_tokens

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device, timeout=timedelta(seconds=120))
    try:
        banks, routes, h = _inputs(device)
        rows = shard_tokens(T, world, rank)
        local = [(i[rows].contiguous(), w[rows].contiguous()) for i, w in routes]
        placements = _placements(routes, world, device)
        result = {}
        for exchange in ("nccl", "p2p"):
            model = _model(banks, world, rank, tokens=T // world, all_to_all=nccl_all_to_all(),
                           placements=placements, exchange=exchange)
            x = h[rows].clone()
            model.step(x, local)                          # eager
            g_in = h[rows].clone()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                model.step(g_in, local)
            for _ in range(2):                            # replays: the epochs keep moving in lockstep
                g_in.copy_(h[rows])
                graph.replay()
            torch.cuda.synchronize()
            del graph
            if exchange == "p2p":
                assert not model.timed_out()
            model.close()
            result[exchange] = {"eager": x.cpu(), "graph": g_in.cpu()}
        torch.save(result, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_over_nccl_equal_one_rank(cuda_device, tmp_path):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    banks, routes, h = _inputs(cuda_device)
    single = _model(banks)
    x = h.clone()
    single.step(x, routes)
    torch.cuda.synchronize()
    mp.spawn(_nccl_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(2)]
    for exchange in ("nccl", "p2p"):
        assert torch.equal(torch.cat([p[exchange]["eager"] for p in parts]), x.cpu()), exchange
        assert torch.equal(torch.cat([p[exchange]["graph"] for p in parts]), x.cpu()), exchange
