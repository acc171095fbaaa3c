"""The reference's own expert-offload manager driving this backend and staging arena.

``ExpertOffloadManager`` and ``install_expert_offload``
(``src/drama_low_vram/offload.py:903-1063``, ``1534-1569``) are imported
unmodified from the copy of the reference package that ``build()`` places under
``oracle/_ref`` (test infrastructure; nothing in the product imports it). The
manager keeps its own host routing, grouping and residency logic:

* ``_forward_resident`` (``offload.py:1169-1193``) when the unique experts of a
  call fit the staging slots;
* ``_forward_partitioned`` / ``_forward_pair_group`` (``1195-1276``) when they
  do not, with ``forward_pairs`` on row chunks;
* ``_forward_hot_cached`` (``1065-1134``) with a per-layer GPU hot cache of
  ``cache_experts`` slots (partial residency), both the single-token
  ``prepare`` path and the many-token ``lookup`` path.

The same manager with the reference's ``TorchExpertBackend`` (its W16A16
dequant path) is the expected value; this repository's ``B200ExpertBackend``
must agree within the 2e-2 bar. GPTQ W4A16 banks (mode 0) run the same way:
``QuantizedB200Backend(0)`` under the manager against the manager running the
reference's ``QuantizedExpertBackend(0)`` and against the oracle. A second test replaces the manager's
``_StagingPool`` with ``StagingArena`` and configures the reference's
``HostResidency`` RAM tier (``host_residency.py:53-358``) through the
manager's own ``configure_host_residency``: the residency logic decides where
each expert's host bytes come from, the arena moves them, and the outputs are
bit-identical to the same manager staging without the RAM tier.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch
from torch import nn

from helpers import assert_parity, np_f32

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
HIDDEN, INTER, EXPERTS = 512, 256, 16


def _reference():
    if not (REF / "drama_low_vram" / "offload.py").is_file():
        pytest.skip("the reference package is not under oracle/_ref (build() copies it from the reference checkout)")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import drama_low_vram.offload as off

    return off


class ExpertLayer(nn.Module):
    """A routed-expert module as the manager finds it: FP8 buffers in host memory."""

    def __init__(self, bank):
        super().__init__()
        self.fp8 = True
        for name, value in bank.items():
            self.register_buffer(name, value.contiguous())

    def forward(self, x, ids, weights):  # replaced by the manager
        raise AssertionError("the offload manager must replace the expert forward")


class Backbone(nn.Module):
    def __init__(self, layers: int, seed: int):
        super().__init__()
        from drama_b200 import synthetic

        self.layers = nn.ModuleList(
            ExpertLayer(synthetic.fp8_bank(EXPERTS, HIDDEN, INTER, seed + i, chunk=EXPERTS)) for i in range(layers))


def _inputs(device, tokens, top_k, seed):
    from drama_b200 import synthetic

    x = synthetic.hidden_states(tokens, HIDDEN, seed, device=device)
    ids, w = synthetic.uniform_routes(tokens, top_k, EXPERTS, seed + 1, device=device)
    return x, ids.to(torch.int64), w.to(torch.bfloat16)


def _run(backbone, calls):
    outs = [backbone.layers[i](x, ids, w) for i, (x, ids, w) in calls]
    torch.cuda.synchronize()
    return outs


def _calls(device):
    """(layer, inputs) in an order that crosses every manager path."""
    return [(0, _inputs(device, 1, 8, 11)), (1, _inputs(device, 1, 8, 12)), (0, _inputs(device, 6, 4, 13)),
            (1, _inputs(device, 5, 8, 14)), (0, _inputs(device, 1, 8, 15))]


@pytest.mark.parametrize("config", [
    {"max_staged_experts": 8, "max_pair_rows": 64},                      # resident, then partitioned
    {"max_staged_experts": 4, "max_pair_rows": 8},                       # partitioned, pair-row chunks
    {"max_staged_experts": 8, "max_pair_rows": 64, "cache_experts": 6},  # partial residency (hot cache)
])
def test_reference_manager_with_b200_backend(cuda_device, config):
    off = _reference()
    from drama_b200 import B200ExpertBackend

    ours = Backbone(2, seed=40)
    theirs = Backbone(2, seed=40)
    mine = off.install_expert_offload(ours, backend=B200ExpertBackend(), **config)
    ref = off.install_expert_offload(theirs, backend="torch", **config)
    calls = _calls(cuda_device)
    got, want = _run(ours, calls), _run(theirs, calls)
    for (layer, (x, ids, w)), a, b in zip(calls, got, want):
        assert a.dtype == x.dtype and a.shape == x.shape
        assert_parity(np_f32(a), np_f32(b), label=f"{config} layer {layer} tokens {x.shape[0]} top-{ids.shape[1]}")
    assert mine.stats.forward_calls == len(calls)
    if config.get("cache_experts"):
        assert mine.stats.expert_cache_hits + mine.stats.expert_loads > 0
    mine.close()
    ref.close()


class Int4Store:
    """A GPTQ W4A16 bank as the reference's ``QuantizedStore`` holds it (mode 0,
    ``quantized_model.py:27-68``): int32 nibble words [E, N, K/8], fp16 group
    scales [E, N, K/128], symmetric codes. ``quantized_model.py`` itself imports
    the full TTS stack, so the store is restated here with the members the
    manager reads (``num_experts``, ``hidden``, ``intermediate``, ``nbytes``,
    ``validate``)."""

    mode = 0

    def __init__(self, bank, hidden, inter):
        for name in ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv"):
            setattr(self, name, bank[name].contiguous())
        self.hidden, self.intermediate = hidden, inter

    @property
    def num_experts(self):
        return self.w13_weight.shape[0]

    @property
    def nbytes(self):
        return sum(getattr(self, n).numel() * getattr(self, n).element_size()
                   for n in ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv"))

    def validate(self):
        for bank, scales, n, k in ((self.w13_weight, self.w13_scale_inv, 2 * self.intermediate, self.hidden),
                                   (self.w2_weight, self.w2_scale_inv, self.hidden, self.intermediate)):
            assert bank.device.type == "cpu" and bank.dtype == torch.int32 and bank.shape[1:] == (n, k // 8)
            assert scales.dtype == torch.float16 and scales.shape[1:] == (n, k // 128)


class Int4Layer(nn.Module):
    """A routed-expert module bound to a quantized store, as ``quantized_model._bind`` leaves it."""

    def __init__(self, store):
        super().__init__()
        for name in ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv"):
            self._buffers[name] = getattr(store, name)
        self._drama_quant_store = store

    def forward(self, x, ids, weights):  # replaced by the manager
        raise AssertionError("the offload manager must replace the expert forward")


def _int4_backbone(layers, seed):
    from drama_b200 import synthetic

    backbone = nn.Module()
    backbone.layers = nn.ModuleList(
        Int4Layer(Int4Store(synthetic.int4_bank(EXPERTS, HIDDEN, INTER, seed + i, asymmetric=False,
                                                scale_dtype=torch.float16), HIDDEN, INTER))
        for i in range(layers))
    return backbone


@pytest.mark.parametrize("config", [
    {"max_staged_experts": 8, "max_pair_rows": 64},
    {"max_staged_experts": 4, "max_pair_rows": 8},
])
def test_reference_manager_with_quantized_b200_backend(cuda_device, config):
    """QuantizedB200Backend(0) under the reference's manager against the same
    manager running the reference's QuantizedExpertBackend(0)
    (``quantized_kernels.py:217-248``, default tiles) and against the oracle."""
    off = _reference()
    import numpy as np

    from drama_low_vram.quantized_kernels import QuantizedExpertBackend
    from oracle import restate as R

    from drama_b200 import QuantizedB200Backend

    theirs_backend = QuantizedExpertBackend(0)
    theirs_backend.tuned_tiles = False
    ours, theirs = _int4_backbone(2, seed=90), _int4_backbone(2, seed=90)
    mine = off.install_expert_offload(ours, backend=QuantizedB200Backend(0), **config)
    ref = off.install_expert_offload(theirs, backend=theirs_backend, **config)
    calls = _calls(cuda_device)
    got, want = _run(ours, calls), _run(theirs, calls)
    for (layer, (x, ids, w)), a, b in zip(calls, got, want):
        label = f"int4 {config} layer {layer} tokens {x.shape[0]}"
        assert a.dtype == x.dtype and a.shape == x.shape
        assert_parity(np_f32(a), np_f32(b), label=label + " vs QuantizedExpertBackend")
        store = ours.layers[layer]._drama_quant_store
        bank = {n: getattr(store, n).float().numpy() if n.endswith("scale_inv") else getattr(store, n).numpy()
                for n in ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv")}
        bank.update(w13_qzeros=None, w2_qzeros=None)
        expected = R.int4_forward(np_f32(x), ids.cpu().numpy(), np_f32(w), bank)
        assert_parity(np_f32(a), np.asarray(expected, dtype=np.float32), label=label + " vs oracle")
    assert mine.stats.forward_calls == len(calls)
    mine.close()
    ref.close()


def test_reference_manager_with_staging_arena_and_host_residency(cuda_device):
    """_StagingPool replaced by StagingArena; the reference's RAM tier picks the bytes' source."""
    off = _reference()
    from drama_b200 import B200ExpertBackend
    from drama_b200.staging import StagingArena

    config = {"max_staged_experts": 8, "max_pair_rows": 64, "cache_experts": 4}
    results = []
    for budget in (None, 6 * 1024 * 1024):
        backbone = Backbone(2, seed=70)
        manager = off.install_expert_offload(backbone, backend=B200ExpertBackend(), **config)
        manager.pool = StagingArena(config["max_staged_experts"])
        if budget is not None:
            report = manager.configure_host_residency(budget)
            assert manager.pool.host_residency is not None and manager.pool.host_residency.enabled, report
        calls = _calls(cuda_device)
        results.append(_run(backbone, calls))
        if budget is not None:
            # the residency tier saw the routes and served the gathers
            assert manager.pool.stats.bounce_gathers > 0
        manager.close()
    theirs = Backbone(2, seed=70)
    ref = off.install_expert_offload(theirs, backend="torch", **config)
    want = _run(theirs, _calls(cuda_device))
    for a, b, c in zip(results[0], results[1], want):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        assert_parity(np_f32(b), np_f32(c), label="arena + host residency vs reference manager")
    ref.close()
