"""Packed Drama3 checkpoints (``shared-model.json`` + one safetensors file) as an expert source.

The fixture is written with the public ``safetensors`` library in the layout
the reference's reader expects (``src/drama_low_vram/shared_checkpoint.py:
20-39``, ``98-145``): the four packed expert tensors of every layer plus other
model tensors around them. ``PackedCheckpointExperts`` must expose exactly the
stored bytes, agree with the reference's own ``SharedFP8Experts`` (imported
from the copy under ``oracle/_ref`` when it is there), and refuse damaged
descriptors and headers before mapping anything.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from drama_b200.packed_checkpoint import DESCRIPTOR_NAME, PACKED_ROLE_NAMES, PackedCheckpointExperts

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
E, H, I, LAYERS = 4, 256, 128, 3


def write_packed(directory: Path, banks, *, extra=True, mutate=None) -> Path:
    from safetensors.torch import save_file

    tensors = {}
    if extra:
        tensors["model.embed_tokens.weight"] = torch.arange(64 * H, dtype=torch.float32).reshape(64, H).bfloat16()
    for layer, bank in enumerate(banks):
        for role, suffix in PACKED_ROLE_NAMES.items():
            tensors[f"model.layers.{layer}.mlp.experts.{suffix}"] = bank[role].contiguous()
        if extra:
            tensors[f"model.layers.{layer}.mlp.gate.weight"] = torch.ones(E, H, dtype=torch.bfloat16)
    if mutate:
        mutate(tensors)
    directory.mkdir(parents=True, exist_ok=True)
    model = directory / "drama3-packed.safetensors"
    save_file(tensors, str(model))
    raw = model.read_bytes()
    (directory / DESCRIPTOR_NAME).write_text(json.dumps({
        "format": "drama3-packed-shared-v1", "model": model.name, "size": len(raw),
        "sha256": hashlib.sha256(raw).hexdigest()}))
    return directory


def _banks():
    from drama_b200 import synthetic

    return [synthetic.fp8_bank(E, H, I, 900 + layer) for layer in range(LAYERS)]


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t


def test_views_are_the_stored_bytes(tmp_path):
    banks = _banks()
    packed = PackedCheckpointExperts.open(write_packed(tmp_path / "ckpt", banks))
    assert (packed.num_layers, packed.num_experts, packed.hidden, packed.intermediate) == (LAYERS, E, H, I)
    for layer, bank in enumerate(banks):
        views = packed.layer_buffers(layer)
        for role, tensor in bank.items():
            assert views[role].dtype == tensor.dtype and views[role].shape == tensor.shape
            assert torch.equal(_bytes(views[role]), _bytes(tensor)), (layer, role)
        assert packed.layer_store(layer) is packed.layer_store(layer)
    with pytest.raises(IndexError):
        packed.layer_buffers(LAYERS)
    packed.close()
    with pytest.raises(RuntimeError, match="closed"):
        packed.layer_buffers(0)


def test_agrees_with_the_reference_reader(tmp_path):
    if not (REF / "drama_low_vram" / "shared_checkpoint.py").is_file():
        pytest.skip("the reference package is not under oracle/_ref (build() copies it from the reference checkout)")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from drama_low_vram.shared_checkpoint import SharedFP8Experts

    banks = _banks()
    directory = write_packed(tmp_path / "ckpt", banks)
    config = SimpleNamespace(text=SimpleNamespace(num_hidden_layers=LAYERS, num_experts=E, moe_intermediate_size=I,
                                                  hidden_size=H))
    theirs = SharedFP8Experts(directory, config)

    class Backbone(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.model = torch.nn.Module()
            self.model.layers = torch.nn.ModuleList()
            for _ in range(LAYERS):
                layer = torch.nn.Module()
                layer.mlp = torch.nn.Module()
                layer.mlp.experts = torch.nn.Module()
                self.model.layers.append(layer)

    backbone = Backbone()
    assert theirs.assign_to_backbone(backbone) == LAYERS
    ours = PackedCheckpointExperts.open(directory)
    assert ours.model_fingerprint == theirs.model_fingerprint
    for layer in range(LAYERS):
        module = backbone.model.layers[layer].mlp.experts
        for role, view in ours.layer_buffers(layer).items():
            assert torch.equal(_bytes(view), _bytes(module._buffers[role])), (layer, role)
    ours.close()


@pytest.mark.parametrize("damage,message", [
    (lambda d, banks: (d / DESCRIPTOR_NAME).write_text(json.dumps({**json.loads((d / DESCRIPTOR_NAME).read_text()),
                                                                    "format": "other"})), "format must be"),
    (lambda d, banks: (d / DESCRIPTOR_NAME).write_text(json.dumps({**json.loads((d / DESCRIPTOR_NAME).read_text()),
                                                                    "size": 10})), "size changed"),
    (lambda d, banks: (d / DESCRIPTOR_NAME).write_text(json.dumps({**json.loads((d / DESCRIPTOR_NAME).read_text()),
                                                                    "sha256": "0" * 63})), "sha256 must be"),
    (lambda d, banks: write_packed(d, banks, mutate=lambda t: t.update({
        "model.layers.1.mlp.experts.down_weight": t["model.layers.1.mlp.experts.down_weight"][:, :, :I // 2].contiguous()})),
     "layer 1 w2_weight does not have shape"),
    (lambda d, banks: write_packed(d, banks, mutate=lambda t: t.pop("model.layers.2.mlp.experts.gate_up_scale")),
     "layer 2 w13_scale_inv does not have shape"),
    (lambda d, banks: write_packed(d, banks, mutate=lambda t: t.update({
        "model.layers.0.mlp.experts.gate_up_scale": t["model.layers.0.mlp.experts.gate_up_scale"].double()})),
     "has dtype F64"),
    (lambda d, banks: write_packed(d, banks, mutate=lambda t: t.update({
        "model.layers.0.mlp.experts.bias": torch.zeros(4)})), "unexpected expert tensor"),
])
def test_damaged_checkpoints_are_refused(tmp_path, damage, message):
    banks = _banks()
    directory = write_packed(tmp_path / "ckpt", banks)
    damage(directory, banks)
    with pytest.raises(ValueError, match=message):
        PackedCheckpointExperts.open(directory)
