"""Generate the expert-cache golden fixture with the reference's own cache builder.

Run in a container that has the Drama3-Studio sources (never on the GPU box):

    python tests/golden/make_expert_cache_golden.py --reference /path/to/Drama3-Studio/src

Steps:
1. Write a tiny Fish Omni checkpoint (config.json, model.safetensors.index.json,
   one safetensors shard) whose routed-expert tensors hold the position
   patterns of ``pattern_projection`` below: every byte is a known function of
   (layer, expert, projection, kind, row, column).
2. Build the cache from it with the reference's ``build_expert_cache``
   (src/drama_low_vram/expert_cache_file.py:266-424) and copy ``manifest.json``
   and ``experts.bin`` to ``tests/golden/expert_cache/``.
3. Cross-check the other direction: a cache written by
   ``drama_b200.expert_cache.write_expert_cache`` from the same patterns must
   open with the reference's ``ExpertCacheFile`` and give identical layer
   buffers.

The fixture is 2 layers x 2 experts, hidden 128, intermediate 128 (196,656
data bytes).
"""

from __future__ import annotations

import argparse
import json
import shutil
import sys
import tempfile
from pathlib import Path

import torch

LAYERS, EXPERTS, HIDDEN, INTER = 2, 2, 128, 128
PROJECTIONS = ("gate_proj", "up_proj", "down_proj")
OUT = Path(__file__).resolve().parent / "expert_cache"


def pattern_projection(layer: int, expert: int, projection: str, kind: str) -> torch.Tensor:
    """The checkpoint tensor of one projection: fp8 bytes or fp32 scales by position."""
    p = PROJECTIONS.index(projection)
    rows, cols = (HIDDEN, INTER) if projection == "down_proj" else (INTER, HIDDEN)
    if kind == "weight":
        r = torch.arange(rows).view(-1, 1)
        c = torch.arange(cols).view(1, -1)
        byte = (layer * 37 + expert * 11 + p * 5 + r * 3 + c) % 251
        return byte.to(torch.uint8).view(torch.float8_e4m3fn)
    r = torch.arange(rows // 128).view(-1, 1).float()
    c = torch.arange(cols // 128).view(1, -1).float()
    return 1.0 + layer + 0.5 * expert + 0.25 * p + 0.125 * (r * (cols // 128) + c)


def pattern_layer(layer: int) -> dict[str, torch.Tensor]:
    """The layer's ``ExpertStore`` tensors (gate rows, then up rows, in w13)."""
    def weights(parts):  # concatenated as bytes: fp8 cat is not available on every build
        return torch.stack([torch.cat([pattern_projection(layer, e, p, "weight").view(torch.uint8) for p in parts])
                            for e in range(EXPERTS)]).view(torch.float8_e4m3fn)

    def scales(parts):
        return torch.stack([torch.cat([pattern_projection(layer, e, p, "weight_scale_inv") for p in parts])
                            for e in range(EXPERTS)])

    return {
        "w13_weight": weights(("gate_proj", "up_proj")),
        "w13_scale_inv": scales(("gate_proj", "up_proj")),
        "w2_weight": weights(("down_proj",)),
        "w2_scale_inv": scales(("down_proj",)),
    }


def _write_checkpoint(root: Path) -> None:
    root.mkdir(parents=True, exist_ok=True)
    (root / "config.json").write_text(json.dumps({
        "model_type": "fish_omni",
        "text_config": {"num_hidden_layers": LAYERS, "num_experts": EXPERTS, "hidden_size": HIDDEN,
                        "moe_intermediate_size": INTER},
    }))
    header, blobs, offset = {}, [], 0
    for layer in range(LAYERS):
        for expert in range(EXPERTS):
            for projection in PROJECTIONS:
                for kind in ("weight", "weight_scale_inv"):
                    t = pattern_projection(layer, expert, projection, kind)
                    raw = t.contiguous().view(torch.uint8).numpy().tobytes()
                    name = f"model.layers.{layer}.mlp.experts.{expert}.{projection}.{kind}"
                    header[name] = {"dtype": "F8_E4M3" if kind == "weight" else "F32", "shape": list(t.shape),
                                    "data_offsets": [offset, offset + len(raw)]}
                    blobs.append(raw)
                    offset += len(raw)
    encoded = json.dumps(header).encode()
    encoded += b" " * (-len(encoded) % 8)
    with (root / "model-00001.safetensors").open("wb") as handle:
        handle.write(len(encoded).to_bytes(8, "little"))
        handle.write(encoded)
        for raw in blobs:
            handle.write(raw)
    (root / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {name: "model-00001.safetensors" for name in header}}))


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="the reference's src directory")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, str(Path(__file__).resolve().parents[2] / "drama3-studio_b200"))
    from drama_low_vram import expert_cache_file as ref

    from drama_b200.expert_cache import write_expert_cache

    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        _write_checkpoint(tmp / "checkpoint")
        built = ref.build_expert_cache(tmp / "checkpoint", tmp / "cache")
        if OUT.exists():
            shutil.rmtree(OUT)
        OUT.mkdir(parents=True)
        for name in (ref.MANIFEST_NAME, ref.DATA_NAME):
            shutil.copyfile(built / name, OUT / name)
        # our writer -> the reference's reader
        ours = write_expert_cache(tmp / "ours", [pattern_layer(layer) for layer in range(LAYERS)])
        with ref.ExpertCacheFile.open(ours, verify_data=True) as cache:
            for layer in range(LAYERS):
                want = pattern_layer(layer)
                for name, t in cache.layer_buffers(layer).items():
                    a, b = t.view(torch.uint8) if t.dtype != torch.float32 else t, want[name]
                    b = b.view(torch.uint8) if b.dtype != torch.float32 else b
                    assert torch.equal(a, b), (layer, name)
        assert (ours / ref.DATA_NAME).read_bytes() == (OUT / ref.DATA_NAME).read_bytes()
    print(f"wrote {OUT}; the reference reads write_expert_cache output identically")


if __name__ == "__main__":
    main()
