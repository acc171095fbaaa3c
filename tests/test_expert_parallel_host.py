"""Expert-parallel exchange choreography on CPU: two gloo ranks, no GPU.

``ExpertParallelMoE.layer`` does the host-side work of expert parallelism:
which buffers go through which all-to-all, in which order, and how the
returned rows are matched back to their (token, slot) pairs. Here its three
device steps (dispatch, expert rows, combine) are replaced by CPU
restatements of what the CUDA kernels are specified to do, with the oracle's
dequant FFN for the expert rows, and the all-to-alls run over gloo between
two processes. The stacked result on every rank must equal, bit for bit, the
single-process oracle of the same layers (``stack_layer`` with the routes
given): the exchange may move rows but must not change any arithmetic.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from helpers import np_bank, np_f32
from oracle import restate as R

E, H, I, K, T, LAYERS = 8, 256, 128, 2, 8, 2


def _inputs():
    from drama_b200 import synthetic

    banks = [synthetic.fp8_bank(E, H, I, seed=10 + l) for l in range(LAYERS)]
    routes = []
    for l in range(LAYERS):
        ids, w = synthetic.zipf_routes(T, K, E, seed=20 + l)
        routes.append((ids.to(torch.int64).contiguous(), w.to(torch.bfloat16).contiguous()))
    h = synthetic.hidden_states(T, H, seed=30)
    return banks, routes, h


def _oracle_stack(banks, routes, h):
    x = np_f32(h)
    for bank, (ids, w) in zip(banks, routes):
        moe = R.fp8_dequant_forward(x, ids.numpy(), np_f32(w), np_bank(bank))
        x = R.round_bf16(x + moe)
    return x


def _cpu_model_class():
    from drama_b200.expert_parallel import ExpertParallelMoE

    class CpuExpertParallel(ExpertParallelMoE):
        """The three device steps restated on CPU tensors."""

        def __init__(self, banks, **kw):
            super().__init__(banks, **kw)
            self.np_banks = [np_bank(vars(b)) for b in banks]

        def _dispatch(self, h, ids, placement=None):
            b, G, cap = self.buffers, self.ranks, self.capacity
            per = self.experts // G
            pos = placement.tolist() if placement is not None else list(range(self.experts))
            tags = b.send_rows.view(torch.int32)[:, self.hidden // 2]   # the int32 after each hidden row
            tags.fill_(per)
            b.pair_rows.fill_(-1)
            fill = [0] * G
            for p, e in enumerate(ids.reshape(-1).tolist()):
                if not 0 <= e < self.experts:
                    continue
                d = pos[e] // per
                if fill[d] >= cap:
                    continue
                row = d * cap + fill[d]
                fill[d] += 1
                b.send_rows[row, :self.hidden] = h[p // self.top_k]
                tags[row] = pos[e] - d * per
                b.pair_rows[p] = row

        def _run_experts(self, layer, rows, out):
            ids = rows.view(torch.int32)[:, self.hidden // 2].clone()
            rows = rows[:, :self.hidden]
            out.zero_()
            valid = [i for i, e in enumerate(ids.tolist()) if 0 <= e < self.local_experts]
            if valid:
                y = R.fp8_dequant_pairs(np_f32(rows[valid]), ids[valid].numpy(), np.ones(len(valid), np.float32),
                                        self.np_banks[layer])
                out[valid] = torch.from_numpy(y).to(torch.bfloat16)

        def _combine(self, back, weights, h, out):
            acc = torch.zeros(self.tokens, self.hidden, dtype=torch.float32)
            pair_rows = self.buffers.pair_rows.tolist()
            for t in range(self.tokens):
                for s in range(self.top_k):
                    row = pair_rows[t * self.top_k + s]
                    if row >= 0:
                        acc[t] = acc[t] + back[row].float() * weights[t, s].float()
            out.copy_((h.float() + acc.to(torch.bfloat16).float()).to(torch.bfloat16))

    return CpuExpertParallel


def _placements(routes, world):
    from drama_b200.expert_parallel import balanced_placement

    out = []
    for ids, _ in routes:
        counts = torch.bincount(ids.reshape(-1), minlength=E).tolist()
        out.append(torch.tensor(balanced_placement(counts, world), dtype=torch.int32))
    return out


def _rank_main(rank: int, world: int, port: int, out_dir: str, balanced: bool) -> None:
    import torch.distributed as dist

    from drama_b200.expert_parallel import experts_of_rank, nccl_all_to_all, shard_experts, shard_tokens

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        banks, routes, h = _inputs()
        placements = _placements(routes, world) if balanced else None
        local = []
        for l, b in enumerate(banks):
            held = experts_of_rank(placements[l].tolist(), world, rank) if balanced else \
                list(shard_experts(E, world, rank))
            local.append({n: v[held] for n, v in b.items()})
        rows = shard_tokens(T, world, rank)

        class Bank:
            def __init__(self, d):
                self.__dict__.update(d)

        model = _cpu_model_class()([Bank(b) for b in local], experts=E, top_k=K, tokens=T // world, ranks=world,
                                   rank=rank, all_to_all=nccl_all_to_all(), placements=placements)
        x = h[rows].contiguous()
        model.step(x, [(ids[rows].contiguous(), w[rows].contiguous()) for ids, w in routes])
        torch.save(x, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("balanced", [False, True])
def test_two_gloo_ranks_match_the_single_process_oracle(tmp_path, balanced):
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path), balanced), nprocs=world, join=True)
    banks, routes, h = _inputs()
    expected = _oracle_stack(banks, routes, h)
    got = np.concatenate([np_f32(torch.load(tmp_path / f"rank{r}.pt")) for r in range(world)])
    assert np.array_equal(got, expected)


def test_single_rank_needs_no_exchange():
    banks, routes, h = _inputs()

    class Bank:
        def __init__(self, d):
            self.__dict__.update(d)

    model = _cpu_model_class()([Bank(b) for b in banks], experts=E, top_k=K, tokens=T)
    x = h.clone()
    model.step(x, routes)
    assert np.array_equal(np_f32(x), _oracle_stack(banks, routes, h))


def test_balanced_placement_evens_out_the_rows():
    from drama_b200.expert_parallel import balanced_placement, experts_of_rank

    counts = [100, 90, 10, 10, 5, 5, 1, 1]
    placement = balanced_placement(counts, 2)
    assert sorted(placement) == list(range(8))
    loads = [sum(counts[e] for e in experts_of_rank(placement, 2, r)) for r in range(2)]
    assert loads == [112, 110]                 # greedy by count, four experts per rank
    assert experts_of_rank(placement, 2, 0)[0] == 0 and experts_of_rank(placement, 2, 1)[0] == 1
    # contiguous blocks are the identity placement
    assert experts_of_rank(list(range(8)), 4, 2) == [4, 5]


def test_shard_helpers_and_argument_checks():
    from drama_b200.expert_parallel import shard_experts, shard_tokens

    assert list(shard_experts(128, 8, 3)) == list(range(48, 64))
    assert shard_tokens(256, 4, 1) == slice(64, 128)
    with pytest.raises(ValueError):
        shard_experts(128, 3, 0)
    with pytest.raises(ValueError):
        shard_experts(128, 2, 2)
    with pytest.raises(ValueError):
        shard_tokens(10, 4, 0)
    banks, routes, h = _inputs()

    class Bank:
        def __init__(self, d):
            self.__dict__.update(d)

    cls = _cpu_model_class()
    with pytest.raises(ValueError, match="all_to_all"):
        cls([Bank(b) for b in banks], experts=E, top_k=K, tokens=T // 2, ranks=2, rank=0)
    with pytest.raises(ValueError, match="experts"):
        cls([Bank(b) for b in banks], experts=E, top_k=K, tokens=T // 2, ranks=2, rank=0,
            all_to_all=lambda o, i: None)
    model = cls([Bank(b) for b in banks], experts=E, top_k=K, tokens=T)
    with pytest.raises(ValueError, match="Hidden rows"):
        model.layer(h[:3].contiguous(), routes[0][0], routes[0][1], 0)
