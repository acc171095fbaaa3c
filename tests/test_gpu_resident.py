"""Resident-bank expert path on a B200: parity, graph capture, id checks.

``install_resident_experts`` keeps ``install_expert_offload``'s contract
(src/drama_low_vram/offload.py:1534-1569, forward checks at 1016-1063) with
every bank in HBM and no host round trip, so a decode layer's router, expert
call and residual can be captured as one CUDA graph (the reference splits the
graph around the expert call, backbone_graph.py:547-556).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import pytest
import torch
from torch import nn

from helpers import assert_parity, np_bank, np_f32
from oracle import restate as R

pytestmark = pytest.mark.gpu

H, I, E, K = 512, 256, 16, 4


class Experts(nn.Module):
    def __init__(self, bank: dict) -> None:
        super().__init__()
        self.fp8 = True
        for name, t in bank.items():
            self.register_buffer(name, t)

    def forward(self, x, ids, w):  # the upstream forward; replaced while a manager is attached
        raise AssertionError("original expert forward called")


class Layer(nn.Module):
    def __init__(self, seed: int, device) -> None:
        super().__init__()
        from drama_b200 import synthetic

        self.experts = Experts(synthetic.fp8_bank(E, H, I, seed))
        self.gate = synthetic.gate_weight(E, H, seed + 50, device=device).to(torch.bfloat16)

    def decode(self, h):
        from drama_b200.router import route_topk

        logits = h @ self.gate.t()
        w, ids = route_topk(logits, K)
        return h + self.experts(h, ids, w)


def _model(device, layers=2):
    return nn.ModuleList(Layer(100 + 10 * i, device) for i in range(layers))


def _oracle_layer(layer, h, ids, w):
    bank = {k: getattr(layer.experts, k) for k in ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv")}
    return R.fp8_dequant_forward(np_f32(h), ids.cpu().numpy(), np_f32(w), np_bank(bank), "bfloat16")


def test_resident_forward_matches_oracle_and_backend(cuda_device):
    from drama_b200 import synthetic
    from drama_b200.backend import B200ExpertBackend
    from drama_b200.resident import install_resident_experts

    model = _model(cuda_device)
    manager = install_resident_experts(model, device=cuda_device)
    try:
        assert manager.stats.resident_layers == 2
        for t, seed in ((1, 3), (7, 4), (160, 5)):  # decode rows and a prefill-sized call (640 pairs)
            x = synthetic.hidden_states(t, H, seed, device=cuda_device)
            ids, w = synthetic.uniform_routes(t, K, E, seed + 1, device=cuda_device)
            w = w.to(torch.bfloat16)
            for layer in model:
                out = layer.experts(x, ids, w)
                direct = B200ExpertBackend().forward(x, ids, w, manager.bank(layer.experts))
                torch.cuda.synchronize()
                assert torch.equal(out.view(torch.int16), direct.view(torch.int16))
                assert_parity(np_f32(out), _oracle_layer(layer, x, ids, w), label=f"resident T={t}")
    finally:
        manager.close()


def test_resident_layers_capture_as_one_graph(cuda_device):
    from drama_b200 import synthetic
    from drama_b200.resident import install_resident_experts

    model = _model(cuda_device, layers=3)
    manager = install_resident_experts(model, device=cuda_device)
    try:
        static_in = synthetic.hidden_states(1, H, 9, device=cuda_device)
        stream = torch.cuda.Stream(cuda_device)
        manager.reserve(1, K, stream=stream)
        stream.wait_stream(torch.cuda.current_stream(cuda_device))
        with torch.cuda.stream(stream):  # eager warm-up on the capture stream
            h = static_in
            for layer in model:
                h = layer.decode(h)
        torch.cuda.current_stream(cuda_device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            h = static_in
            for layer in model:
                h = layer.decode(h)
            static_out = h
        assert manager.stats.captured_calls == 3
        for seed in (21, 22, 23):
            x = synthetic.hidden_states(1, H, seed, device=cuda_device)
            static_in.copy_(x)
            graph.replay()
            eager = x
            for layer in model:
                eager = layer.decode(eager)
            torch.cuda.synchronize()
            assert torch.equal(static_out.view(torch.int16), eager.view(torch.int16))
        # one layer against the oracle, routes taken from the device router
        from drama_b200.router import route_topk

        x = synthetic.hidden_states(1, H, 31, device=cuda_device)
        w, ids = route_topk(x @ model[0].gate.t(), K)
        out = model[0].experts(x, ids, w)
        assert_parity(np_f32(out), _oracle_layer(model[0], x, ids, w), label="resident routed layer")
        del graph
    finally:
        manager.close()


def test_resident_checks_ids_like_the_manager(cuda_device):
    from drama_b200 import synthetic
    from drama_b200.resident import install_resident_experts

    model = _model(cuda_device, layers=1)
    manager = install_resident_experts(model, device=cuda_device)
    try:
        x = synthetic.hidden_states(2, H, 1, device=cuda_device)
        ids, w = synthetic.uniform_routes(2, K, E, 2, device=cuda_device)
        bad = ids.clone()
        bad[1, 2] = E
        with pytest.raises(ValueError, match=rf"Expert IDs must be in \[0, {E}\)"):
            model[0].experts(x, bad, w)
        with pytest.raises(ValueError, match="Expert IDs must have shape"):
            model[0].experts(x, ids[:1], w[:1])
        with pytest.raises(ValueError, match="Routing weights must match"):
            model[0].experts(x, ids, w[:, :2])
        assert torch.equal(model[0].experts(x[:0], ids[:0], w[:0]), x[:0])
    finally:
        manager.close()
    with pytest.raises(AssertionError, match="original expert forward"):
        model[0].experts(x, ids, w)  # forward restored by close()
    with pytest.raises(RuntimeError, match="closed"):
        manager.forward(model[0].experts, x, ids, w)


@dataclass
class _GptqStore:
    """The reference's ``QuantizedStore`` fields for mode 0 (quantized_model.py:27-35)."""

    w13_weight: torch.Tensor
    w13_scale_inv: torch.Tensor
    w2_weight: torch.Tensor
    w2_scale_inv: torch.Tensor
    hidden: int
    intermediate: int
    mode: int = 0

    def validate(self):
        assert self.w13_scale_inv.dtype == torch.float16


def test_resident_gptq_bank_matches_oracle(cuda_device):
    from drama_b200 import synthetic
    from drama_b200.resident import install_resident_experts

    bank = synthetic.int4_bank(E, H, I, 77, asymmetric=False, scale_dtype=torch.float16)
    module = Experts(synthetic.fp8_bank(1, 256, 128, 0))  # module carries a store, like quantized_model.py:110
    module._drama_quant_store = _GptqStore(bank["w13_weight"], bank["w13_scale_inv"], bank["w2_weight"],
                                           bank["w2_scale_inv"], H, I)
    manager = install_resident_experts(nn.ModuleList([module]), device=cuda_device)
    try:
        x = synthetic.hidden_states(3, H, 5, device=cuda_device)
        ids, w = synthetic.uniform_routes(3, K, E, 6, device=cuda_device)
        out = module(x, ids, w.to(torch.bfloat16))
        torch.cuda.synchronize()
        ref = R.int4_forward(np_f32(x), ids.cpu().numpy(), np_f32(w.to(torch.bfloat16)), np_bank(bank), "bfloat16")
        assert_parity(np_f32(out), ref, label="resident GPTQ")
    finally:
        manager.close()


@pytest.mark.parametrize("kind", ["fp8", "gptq", "w8a8"])
def test_batched_verification_rows_equal_per_row_calls(cuda_device, kind):
    """``backbone_block(..., batch_experts=True)`` sends 1, 2 or 4 rows through one expert call
    (src/drama_low_vram/verification.py:71-80); each row's result must not depend on the others."""
    from drama_b200 import synthetic
    from drama_b200.resident import install_resident_experts

    if kind == "fp8":
        module = Experts(synthetic.fp8_bank(E, H, I, 91))
    else:
        module = Experts(synthetic.fp8_bank(1, 256, 128, 0))
        if kind == "gptq":
            bank = synthetic.int4_bank(E, H, I, 92, asymmetric=False, scale_dtype=torch.float16)
            module._drama_quant_store = _GptqStore(bank["w13_weight"], bank["w13_scale_inv"], bank["w2_weight"],
                                                   bank["w2_scale_inv"], H, I)
        else:
            bank = synthetic.w8a8_bank(2, E, H, I, 93)
            module._drama_quant_store = _GptqStore(bank["w13_weight"], bank["w13_scale_inv"], bank["w2_weight"],
                                                   bank["w2_scale_inv"], H, I, mode=2)
            module._drama_quant_store.validate = lambda: None
    manager = install_resident_experts(nn.ModuleList([module]), device=cuda_device)
    try:
        for count in (1, 2, 4):
            x = synthetic.hidden_states(count, H, 100 + count, device=cuda_device)
            ids, w = synthetic.uniform_routes(count, K, E, 200 + count, device=cuda_device)
            w = w.to(torch.bfloat16)
            batched = module(x, ids, w)
            rows = torch.cat([module(x[r:r + 1], ids[r:r + 1], w[r:r + 1]) for r in range(count)])
            torch.cuda.synchronize()
            assert torch.equal(batched.view(torch.int16), rows.view(torch.int16)), f"{kind}, {count} rows"
    finally:
        manager.close()
