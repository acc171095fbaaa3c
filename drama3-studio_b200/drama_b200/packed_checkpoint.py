"""Packed Drama3 checkpoints as a staging source: the expert banks in place.

The second host byte source of the reference's low-VRAM runtime
(``src/drama_low_vram/shared_checkpoint.py:98-145``, ``SharedFP8Experts``): a
directory with a ``shared-model.json`` descriptor naming one safetensors file
that holds the whole model, the routed experts of layer ``i`` as four packed
tensors

    model.layers.{i}.mlp.experts.gate_up_weight  [E, 2I, H]          F8_E4M3
    model.layers.{i}.mlp.experts.gate_up_scale   [E, 2I/128, H/128]  F32
    model.layers.{i}.mlp.experts.down_weight     [E, H, I]           F8_E4M3
    model.layers.{i}.mlp.experts.down_scale      [E, H/128, I/128]   F32

(the ``ExpertStore`` roles ``w13_weight``, ``w13_scale_inv``, ``w2_weight``,
``w2_scale_inv``, ``shared_checkpoint.py:20-23``). The descriptor records the
file's name relative to the directory, its size and SHA-256
(``shared_checkpoint.py:26-39``); the format name and fields are kept so the
same directories serve both implementations.

``PackedCheckpointExperts`` reads the safetensors header itself, checks every
layer's four expert tensors against the model geometry, maps the file private
and exposes each layer as a ``StagingArena`` store of zero-copy views. Like
``ExpertCacheFile`` it can page-lock a window of layers where it lies
(``register``), so the arena copies experts from the page cache straight into
HBM slots with no bounce gather. The other tensors of the file are never read.
"""

from __future__ import annotations

import json
import math
import re
from pathlib import Path
from typing import Any

from .expert_cache import BLOCK, MappedExperts, ROLE_DTYPES, _HEX_DIGEST, _Rule, _exactly, check_manifest
from .staging import EXPERT_BUFFER_NAMES

DESCRIPTOR_NAME = "shared-model.json"
PACKED_FORMAT = "drama3-packed-shared-v1"
# ExpertStore role -> tensor name suffix in the packed file
PACKED_ROLE_NAMES = {
    "w13_weight": "gate_up_weight",
    "w13_scale_inv": "gate_up_scale",
    "w2_weight": "down_weight",
    "w2_scale_inv": "down_scale",
}
# safetensors dtype name -> ExpertStore role dtype name
_SAFETENSORS_DTYPES = {"F8_E4M3": "float8_e4m3fn", "F32": "float32"}
_EXPERT_TENSOR = re.compile(r"model\.layers\.(\d+)\.mlp\.experts\.(\w+)")
_HEADER_LIMIT = 256 << 20

DESCRIPTOR_SCHEMA: dict[str, Any] = {
    "format": _exactly(PACKED_FORMAT),
    "model": _Rule("a file name relative to the descriptor", lambda v: isinstance(v, str) and v != ""),
    "size": _Rule("an integer >= 9", lambda v: type(v) is int and v >= 9),
    "sha256": _HEX_DIGEST,
}


def _read_safetensors_header(path: Path, size: int) -> tuple[int, dict[str, Any]]:
    """(first data byte, header object) of a safetensors file of ``size`` bytes."""
    with path.open("rb") as handle:
        prefix = handle.read(8)
        if len(prefix) != 8:
            raise ValueError(f"packed checkpoint {path}: shorter than a safetensors header")
        length = int.from_bytes(prefix, "little")
        if not 2 <= length <= min(_HEADER_LIMIT, size - 8):
            raise ValueError(f"packed checkpoint {path}: header length {length} is out of range")
        raw = handle.read(length)
    try:
        header = json.loads(raw)
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError(f"packed checkpoint {path}: header is not valid JSON") from exc
    if not isinstance(header, dict):
        raise ValueError(f"packed checkpoint {path}: header is not a JSON object")
    return 8 + length, header


class PackedCheckpointExperts(MappedExperts):
    """The routed-expert banks of a packed Drama3 checkpoint, viewed in place."""

    def __init__(self, directory: str | Path) -> None:
        self.directory = Path(directory).resolve()
        descriptor_path = self.directory / DESCRIPTOR_NAME
        if not descriptor_path.is_file():
            raise ValueError(f"packed checkpoint descriptor {descriptor_path} not found")
        try:
            descriptor = json.loads(descriptor_path.read_text(encoding="utf-8"))
        except (UnicodeDecodeError, json.JSONDecodeError) as exc:
            raise ValueError(f"packed checkpoint descriptor {descriptor_path} is not valid JSON") from exc
        fields = check_manifest(DESCRIPTOR_SCHEMA, descriptor)
        self.descriptor = descriptor
        self.model_fingerprint = fields["sha256"]
        self._data_path = (self.directory / fields["model"]).resolve()
        if not self._data_path.is_file() or self._data_path.stat().st_size != fields["size"]:
            raise ValueError(f"packed checkpoint {self._data_path} is missing or its size changed")
        self.nbytes = fields["size"]
        data_start, header = _read_safetensors_header(self._data_path, self.nbytes)
        self._roles = self._expert_roles(header, data_start)
        self._init_mapping()

    def _expert_roles(self, header: dict[str, Any], data_start: int) -> list[dict[str, tuple[int, int, tuple]]]:
        """Per layer: role -> (absolute byte offset, byte count, shape), checked
        against the geometry of layer 0 (every layer has the same banks)."""
        found: dict[int, dict[str, tuple[int, int, tuple]]] = {}
        suffix_role = {suffix: role for role, suffix in PACKED_ROLE_NAMES.items()}
        for name, entry in header.items():
            match = _EXPERT_TENSOR.fullmatch(name)
            if name == "__metadata__" or ".mlp.experts." not in name:
                continue
            if match is None or match.group(2) not in suffix_role:
                raise ValueError(f"packed checkpoint: unexpected expert tensor {name!r}")
            role = suffix_role[match.group(2)]
            if not isinstance(entry, dict) or set(entry) != {"dtype", "shape", "data_offsets"}:
                raise ValueError(f"packed checkpoint: malformed header entry for {name!r}")
            dtype = _SAFETENSORS_DTYPES.get(entry["dtype"])
            if dtype != ROLE_DTYPES[role][1]:
                raise ValueError(f"packed checkpoint: {name} has dtype {entry['dtype']}, expected {ROLE_DTYPES[role][1]}")
            shape, offsets = entry["shape"], entry["data_offsets"]
            if (not isinstance(shape, list) or len(shape) != 3 or not all(type(d) is int and d > 0 for d in shape)
                    or not isinstance(offsets, list) or len(offsets) != 2
                    or not all(type(o) is int and o >= 0 for o in offsets)):
                raise ValueError(f"packed checkpoint: malformed shape or offsets for {name!r}")
            begin, end = offsets
            if end - begin != math.prod(shape) * ROLE_DTYPES[role][2] or data_start + end > self.nbytes:
                raise ValueError(f"packed checkpoint: {name} byte range does not match its shape or the file")
            found.setdefault(int(match.group(1)), {})[role] = (data_start + begin, end - begin, tuple(shape))
        if not found:
            raise ValueError("packed checkpoint holds no routed-expert tensors")
        layers = sorted(found)
        if layers != list(range(len(layers))):
            raise ValueError(f"packed checkpoint: expert layers are not 0..{len(layers) - 1}")
        first = found[0]
        if set(first) != set(EXPERT_BUFFER_NAMES):
            raise ValueError("packed checkpoint: layer 0 lacks an expert role")
        experts, gate_up, hidden = first["w13_weight"][2]
        inter = gate_up // 2
        if gate_up % 2 or hidden % BLOCK or inter % BLOCK:
            raise ValueError("packed checkpoint: expert dimensions must be multiples of the FP8 block size")
        geometry = {
            "w13_weight": (experts, 2 * inter, hidden),
            "w13_scale_inv": (experts, 2 * inter // BLOCK, hidden // BLOCK),
            "w2_weight": (experts, hidden, inter),
            "w2_scale_inv": (experts, hidden // BLOCK, inter // BLOCK),
        }
        for layer in layers:
            roles = found[layer]
            for role, shape in geometry.items():
                if role not in roles or roles[role][2] != shape:
                    raise ValueError(f"packed checkpoint: layer {layer} {role} does not have shape {shape}")
        self.num_layers = len(layers)
        self.num_experts, self.hidden, self.intermediate = experts, hidden, inter
        return [found[layer] for layer in layers]

    def _role_records(self, layer: int) -> dict[str, tuple[int, int, tuple[int, ...]]]:
        return {name: self._roles[layer][name] for name in EXPERT_BUFFER_NAMES}

    @classmethod
    def open(cls, directory: str | Path) -> "PackedCheckpointExperts":
        return cls(directory)


__all__ = ["DESCRIPTOR_NAME", "PACKED_FORMAT", "PACKED_ROLE_NAMES", "PackedCheckpointExperts"]
