"""Resident-bank manager: store validation and discovery, checked on the host.

Every case here fails before any device memory is touched, mirroring the
checks of ``ExpertStore.validate`` (src/drama_low_vram/offload.py:139-170) and
``install_expert_offload`` (offload.py:1534-1569).
"""

from __future__ import annotations

import pytest
import torch
from torch import nn

from drama_b200 import synthetic
from drama_b200.resident import (ResidentExpertManager, _module_store, expert_modules,
                                 install_resident_experts)


class Experts(nn.Module):
    def __init__(self, bank: dict, fp8: bool = True) -> None:
        super().__init__()
        self.fp8 = fp8
        for name, t in bank.items():
            self.register_buffer(name, t)


class Backbone(nn.Module):
    def __init__(self, layers: list[nn.Module]) -> None:
        super().__init__()
        self.layers = nn.ModuleList(nn.ModuleDict({"experts": e, "gate": nn.Linear(4, 4)}) for e in layers)


def _bank(seed=0):
    return synthetic.fp8_bank(2, 256, 128, seed)


def test_discovery_finds_only_expert_banks():
    model = Backbone([Experts(_bank(0)), Experts(_bank(1))])
    names = [name for name, _ in expert_modules(model)]
    assert names == ["layers.0.experts", "layers.1.experts"]


def test_fp8_store_accepts_reference_layout():
    kind, tensors = _module_store(Experts(_bank()))
    assert kind == "fp8" and set(tensors) == {"w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv"}


@pytest.mark.parametrize("mutate,message", [
    (lambda b: b.update(w13_scale_inv=b["w13_scale_inv"].double()), "w13_scale_inv must be torch.float32"),
    (lambda b: b.update(w2_weight=b["w2_weight"].view(torch.uint8)), "w2_weight must be torch.float8_e4m3fn"),
    (lambda b: b.update(w2_weight=b["w2_weight"].transpose(1, 2)), "w2_weight must be contiguous"),
    (lambda b: b.update(w2_scale_inv=b["w2_scale_inv"][:, :1].contiguous()), "w2_scale_inv has shape"),
    (lambda b: b.update(w13_weight=b["w13_weight"][0]), "w13_weight must be a stacked three-dimensional"),
])
def test_fp8_store_rejections(mutate, message):
    bank = _bank()
    mutate(bank)
    with pytest.raises(ValueError, match=message):
        install_resident_experts(Backbone([Experts(bank)]))


def test_dense_bank_rejected():
    with pytest.raises(ValueError, match="requires FP8 buffers"):
        install_resident_experts(Backbone([Experts(_bank(), fp8=False)]))


def test_unknown_quantized_mode_rejected():
    module = Experts(_bank())

    class Store:
        mode = 7

    module._drama_quant_store = Store()
    with pytest.raises(ValueError, match="Unknown quantized bank format"):
        install_resident_experts(Backbone([module]))


def test_second_manager_refused_before_any_change():
    first, second = Experts(_bank(0)), Experts(_bank(1))
    second._drama_offload_original_forward = second.forward  # another manager got there first
    original = first.forward
    with pytest.raises(ValueError, match="already has an expert offload manager"):
        install_resident_experts(Backbone([first, second]))
    assert first.forward == original and not hasattr(first, "_drama_offload_original_forward")


def test_no_experts_and_cpu_device_refused():
    with pytest.raises(ValueError, match="no routed expert modules"):
        install_resident_experts(nn.Linear(4, 4))
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        ResidentExpertManager(device="cpu")
