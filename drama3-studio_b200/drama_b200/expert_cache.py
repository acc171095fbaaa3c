"""Expert cache files as a staging source: read-only mmap, page-locked in place.

On-disk format (kept identical so caches move between the two implementations):
the reference's ``"drama3-official-fp8-experts"`` version 1
(src/drama_low_vram/expert_cache_file.py:28-33 names, 113-153 layout, 378-395
manifest, 426-471 reader checks). ``experts.bin`` holds, for layer 0, 1, ...
in turn, the four role tensors of ``ExpertStore`` back to back with no padding:

    w13_weight    [E, 2I, H]          float8_e4m3fn  (gate rows, then up rows)
    w13_scale_inv [E, 2I/128, H/128]  float32
    w2_weight     [E, H, I]           float8_e4m3fn
    w2_scale_inv  [E, H/128, I/128]   float32

``manifest.json`` records the model geometry, every buffer's shape, dtype,
byte offset and size, the data file's size and SHA-256, and a model
fingerprint.

What this module adds for the B200 path is ``ExpertCacheFile.register``: it
page-locks a layer window of the mapping where it lies (``drama_b200_host_register``
with ``cudaHostRegisterReadOnly``), after which the layer's role views are
page-locked tensors and ``StagingArena`` copies each requested expert straight
from the page cache into its HBM slot (four DMAs per expert, one per role,
merged where experts are adjacent). The reference reads the same mapping
through a host gather into a pinned bounce buffer before every copy
(offload.py:561-594); an unregistered cache still takes that route through the
arena's bounce path.

The file is mapped private (``MAP_PRIVATE``, copy-on-write; nothing ever
reaches the file) rather than ``PROT_READ``-only as the reference maps it:
on B200 hosts with driver 580 ``cudaHostRegister`` refuses ``PROT_READ``
mappings with or without the read-only flag, and accepts a private mapping
with it. A read-only registration pins the page-cache pages themselves (no
copy-on-write copies), so registering costs no extra RAM. The views must still
only be read.
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import math
import mmap
import re
import sys
from pathlib import Path
from typing import Any

import torch
from torch import Tensor

from . import _lib
from .staging import EXPERT_BUFFER_NAMES, StagedExperts

CACHE_FORMAT = "drama3-official-fp8-experts"
CACHE_FORMAT_VERSION = 1
MANIFEST_NAME = "manifest.json"
DATA_NAME = "experts.bin"
BLOCK = 128
_CHUNK = 1 << 20
_SHA256 = re.compile(r"[a-f0-9]{64}")
# role -> (torch dtype, manifest dtype name, element size)
ROLE_DTYPES = {
    "w13_weight": (torch.float8_e4m3fn, "float8_e4m3fn", 1),
    "w13_scale_inv": (torch.float32, "float32", 4),
    "w2_weight": (torch.float8_e4m3fn, "float8_e4m3fn", 1),
    "w2_scale_inv": (torch.float32, "float32", 4),
}


def role_shapes(num_experts: int, hidden: int, intermediate: int) -> dict[str, tuple[int, int, int]]:
    return {
        "w13_weight": (num_experts, 2 * intermediate, hidden),
        "w13_scale_inv": (num_experts, 2 * intermediate // BLOCK, hidden // BLOCK),
        "w2_weight": (num_experts, hidden, intermediate),
        "w2_scale_inv": (num_experts, hidden // BLOCK, intermediate // BLOCK),
    }


def cache_layout(num_layers: int, num_experts: int, hidden: int,
                 intermediate: int) -> tuple[list[dict[str, Any]], int]:
    """Per-layer buffer records of the manifest and the data file's size."""
    for label, value in (("num_layers", num_layers), ("num_experts", num_experts), ("hidden", hidden),
                         ("intermediate", intermediate)):
        if type(value) is not int or value < 1:
            raise ValueError(f"{label} must be a positive integer")
    if hidden % BLOCK or intermediate % BLOCK:
        raise ValueError("Expert dimensions must be divisible by the FP8 block size")
    shapes = role_shapes(num_experts, hidden, intermediate)
    layers, offset = [], 0
    for index in range(num_layers):
        buffers = {}
        for name in EXPERT_BUFFER_NAMES:
            _, dtype_name, size = ROLE_DTYPES[name]
            nbytes = math.prod(shapes[name]) * size
            buffers[name] = {"shape": list(shapes[name]), "dtype": dtype_name, "offset": offset, "nbytes": nbytes}
            offset += nbytes
        layers.append({"index": index, "buffers": buffers})
    return layers, offset


def write_expert_cache(cache_dir: str | Path, layers: list[dict[str, Tensor]], *,
                       model_fingerprint: str | None = None, source: dict[str, Any] | None = None) -> Path:
    """Write ``layers`` (one ``ExpertStore``-shaped dict per layer) as a cache directory.

    The reference builds caches from a safetensors checkpoint
    (``build_expert_cache``); this writes banks already in memory, in the same
    format. ``model_fingerprint`` defaults to the SHA-256 of the geometry.
    """
    if not layers:
        raise ValueError("An expert cache needs at least one layer")
    experts, gate_up, hidden = layers[0]["w13_weight"].shape
    inter = gate_up // 2
    records, total = cache_layout(len(layers), experts, hidden, inter)
    cache_dir = Path(cache_dir)
    cache_dir.mkdir(parents=True, exist_ok=True)
    digest = hashlib.sha256()
    written = 0
    with (cache_dir / DATA_NAME).open("wb") as handle:
        for index, bank in enumerate(layers):
            for name in EXPERT_BUFFER_NAMES:
                spec = records[index]["buffers"][name]
                t = bank[name]
                if list(t.shape) != spec["shape"] or t.dtype != ROLE_DTYPES[name][0]:
                    raise ValueError(f"layer {index} {name}: shape/dtype mismatch")
                raw = t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()
                handle.write(raw)
                digest.update(raw)
                written += len(raw)
    if written != total:
        raise ValueError(f"Expert cache byte count mismatch: {written} != {total}")
    model = {"model_type": "fish_omni", "num_layers": len(layers), "num_experts": experts, "hidden": hidden,
             "intermediate": inter, "block_size": BLOCK}
    if model_fingerprint is None:
        model_fingerprint = hashlib.sha256(json.dumps(model, sort_keys=True).encode()).hexdigest()
    manifest = {
        "format": CACHE_FORMAT,
        "format_version": CACHE_FORMAT_VERSION,
        "byte_order": "little",
        "model_fingerprint": model_fingerprint,
        "model": model,
        "source": source if source is not None else {},
        "data": {"name": DATA_NAME, "size": total, "sha256": digest.hexdigest()},
        "layers": records,
    }
    with (cache_dir / MANIFEST_NAME).open("w", encoding="utf-8", newline="\n") as handle:
        json.dump(manifest, handle, indent=2, sort_keys=True)
        handle.write("\n")
    return cache_dir


# ---------------------------------------------------------------------------
# Manifest validation: a declarative schema (field -> rule) walked by one
# generic checker, then the checks that relate fields to each other and to
# the data file.
# ---------------------------------------------------------------------------
_MISSING = object()


class _Rule:
    """One manifest value: ``accepts(value)`` and a description for errors."""

    def __init__(self, describe: str, accepts) -> None:
        self.describe = describe
        self.accepts = accepts


def _exactly(expected: Any) -> _Rule:
    return _Rule(repr(expected), lambda v: v == expected and type(v) is type(expected))


def _count(minimum: int) -> _Rule:
    return _Rule(f"an integer >= {minimum}", lambda v: type(v) is int and v >= minimum)


_HEX_DIGEST = _Rule("64 lowercase hex digits", lambda v: isinstance(v, str) and _SHA256.fullmatch(v) is not None)

MANIFEST_SCHEMA: dict[str, Any] = {
    "format": _exactly(CACHE_FORMAT),
    "format_version": _exactly(CACHE_FORMAT_VERSION),
    "byte_order": _exactly("little"),
    "model_fingerprint": _HEX_DIGEST,
    "model": {
        "model_type": _exactly("fish_omni"),
        "block_size": _exactly(BLOCK),
        "num_layers": _count(1),
        "num_experts": _count(1),
        "hidden": _count(1),
        "intermediate": _count(1),
    },
    "data": {"name": _exactly(DATA_NAME), "size": _count(1), "sha256": _HEX_DIGEST},
}


def check_manifest(schema: dict[str, Any], manifest: Any, path: str = "") -> dict[str, Any]:
    """Validate ``manifest`` against ``schema``; returns the checked values by dotted path.

    Raises ``ValueError("expert cache manifest: <path> ...")`` for the first
    field that is missing or breaks its rule.
    """
    where = path or "the manifest"
    if not isinstance(manifest, dict):
        raise ValueError(f"expert cache manifest: {where} must be a JSON object")
    values: dict[str, Any] = {}
    for key, rule in schema.items():
        field = f"{path}.{key}" if path else key
        value = manifest.get(key, _MISSING)
        if isinstance(rule, dict):
            values.update(check_manifest(rule, value if value is not _MISSING else None, field))
        elif value is _MISSING or not rule.accepts(value):
            found = "missing" if value is _MISSING else f"found {value!r}"
            raise ValueError(f"expert cache manifest: {field} must be {rule.describe} ({found})")
        else:
            values[field] = value
    return values


class MappedExperts:
    """Expert banks laid out in one file, mapped private and viewed in place.

    A subclass sets ``_data_path``, ``nbytes``, ``num_layers`` and
    ``_role_records(layer)`` (role name -> (byte offset, byte count, shape));
    this class provides the mapping, zero-copy role views, the per-layer
    staging store and page locking of layer windows.
    """

    def _init_mapping(self) -> None:
        self._mmap: mmap.mmap | None = None
        self._mapping: Tensor | None = None
        self._stores: dict[int, StagedExperts] = {}
        self._registered: list[tuple[int, int, int, int]] = []  # (base, bytes, first layer, end layer)
        self._closed = False

    def _role_records(self, layer: int) -> dict[str, tuple[int, int, tuple[int, ...]]]:
        raise NotImplementedError

    def _map(self) -> Tensor:
        if self._closed:
            raise RuntimeError("Expert source is closed")
        if self._mapping is None:
            with self._data_path.open("rb") as handle:
                self._mmap = mmap.mmap(handle.fileno(), self.nbytes, access=mmap.ACCESS_COPY)
            self._mapping = torch.frombuffer(self._mmap, dtype=torch.uint8, count=self.nbytes)
        return self._mapping

    def _check_layer(self, layer: int) -> None:
        if not isinstance(layer, int) or isinstance(layer, bool) or not 0 <= layer < self.num_layers:
            raise IndexError(f"Invalid expert layer index: {layer}")

    def layer_span(self, layer: int) -> tuple[int, int]:
        """(byte offset, byte count) of the smallest range holding one layer's four roles."""
        self._check_layer(layer)
        records = self._role_records(layer).values()
        start = min(offset for offset, _, _ in records)
        end = max(offset + size for offset, size, _ in records)
        return start, end - start

    def layer_buffers(self, layer: int) -> dict[str, Tensor]:
        """Zero-copy, read-only role views of one layer (must not be written)."""
        self._check_layer(layer)
        mapping = self._map()
        return {name: mapping.narrow(0, offset, size).view(ROLE_DTYPES[name][0]).view(shape)
                for name, (offset, size, shape) in self._role_records(layer).items()}

    def layer_store(self, layer: int) -> StagedExperts:
        """The layer as a ``StagingArena`` store; the same object for every call, so
        the arena's reuse rule (same ids from the same store) applies."""
        store = self._stores.get(layer)
        if store is None:
            store = StagedExperts(**self.layer_buffers(layer))
            self._stores[layer] = store
        return store

    def register(self, first: int = 0, count: int | None = None) -> int:
        """Page-lock the bytes of layers ``[first, first + count)`` (default: all) in place.

        Returns the number of bytes locked (the window widened to whole pages).
        A window may not overlap or adjoin one already registered.
        """
        count = self.num_layers - first if count is None else count
        self._check_layer(first)
        if count < 1 or first + count > self.num_layers:
            raise IndexError("Layer window outside the expert source")
        for _, _, a, b in self._registered:
            if first < b + 1 and a < first + count + 1:  # page widening can make neighbours touch
                raise ValueError(f"Layers [{first}, {first + count}) overlap or adjoin registered layers [{a}, {b})")
        spans = [self.layer_span(layer) for layer in range(first, first + count)]
        start = min(offset for offset, _ in spans)
        end = max(offset + size for offset, size in spans)
        mapping = self._map()
        base, size = ctypes.c_void_p(), ctypes.c_uint64()
        lib = _lib.library()
        lib.check(lib.dll.drama_b200_host_register(mapping.data_ptr() + start, end - start, 1,
                                                   ctypes.byref(base), ctypes.byref(size)))
        self._registered.append((base.value, size.value, first, first + count))
        return size.value

    @property
    def registered_layers(self) -> list[tuple[int, int]]:
        return [(a, b) for _, _, a, b in self._registered]

    def unregister(self) -> None:
        """Release every page-locked window. Copies reading them must be complete."""
        if not self._registered:
            return
        if torch.cuda.is_initialized():
            torch.cuda.synchronize()
        lib = _lib.library()
        while self._registered:
            base, _, _, _ = self._registered.pop()
            lib.check(lib.dll.drama_b200_host_unregister(base))

    def close(self) -> None:
        """Unregister and drop this object's views; tensors already handed out keep the mapping alive."""
        self.unregister()
        self._stores.clear()
        self._mapping = None
        self._mmap = None
        self._closed = True

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        self.close()


class ExpertCacheFile(MappedExperts):
    """A validated expert cache: private mapping, zero-copy role views, page locking."""

    def __init__(self, cache_dir: Path, manifest: dict[str, Any]) -> None:
        self.cache_dir = Path(cache_dir)
        self.manifest = manifest
        if sys.byteorder != "little":
            raise ValueError("expert cache files are little-endian; this host is not")
        fields = check_manifest(MANIFEST_SCHEMA, manifest)
        self.num_layers = fields["model.num_layers"]
        self.num_experts = fields["model.num_experts"]
        self.hidden = fields["model.hidden"]
        self.intermediate = fields["model.intermediate"]
        self.model_fingerprint = fields["model_fingerprint"]
        # the buffer records follow from the geometry; the manifest must repeat them exactly
        self._layers, self.nbytes = cache_layout(self.num_layers, self.num_experts, self.hidden, self.intermediate)
        if manifest.get("layers") != self._layers:
            raise ValueError("expert cache manifest: layers do not match the layout of the model geometry")
        if fields["data.size"] != self.nbytes:
            raise ValueError(f"expert cache manifest: data.size is {fields['data.size']}, the layout needs {self.nbytes}")
        self._data_path = self.cache_dir / DATA_NAME
        if not self._data_path.is_file() or self._data_path.stat().st_size != self.nbytes:
            raise ValueError(f"expert cache data file {self._data_path} is truncated or has extra data")
        self._init_mapping()

    @classmethod
    def open(cls, cache_dir: str | Path, *, verify_data: bool = False) -> "ExpertCacheFile":
        cache_dir = Path(cache_dir).resolve()
        try:
            manifest = json.loads((cache_dir / MANIFEST_NAME).read_bytes())
        except (UnicodeDecodeError, json.JSONDecodeError) as exc:
            raise ValueError(f"expert cache manifest {cache_dir / MANIFEST_NAME} is not valid JSON") from exc
        cache = cls(cache_dir, manifest)
        if verify_data:
            cache.verify_data()
        return cache

    def verify_data(self) -> None:
        """Hash the whole data file and compare with the manifest's data.sha256."""
        digest = hashlib.sha256()
        with self._data_path.open("rb") as handle:
            while chunk := handle.read(_CHUNK):
                digest.update(chunk)
        if digest.hexdigest() != self.manifest["data"]["sha256"]:
            raise ValueError("expert cache data checksum mismatch (data.sha256)")

    def _role_records(self, layer: int) -> dict[str, tuple[int, int, tuple[int, ...]]]:
        buffers = self._layers[layer]["buffers"]
        return {name: (buffers[name]["offset"], buffers[name]["nbytes"], tuple(buffers[name]["shape"]))
                for name in EXPERT_BUFFER_NAMES}


__all__ = ["CACHE_FORMAT", "CACHE_FORMAT_VERSION", "DATA_NAME", "MANIFEST_NAME", "MANIFEST_SCHEMA",
           "ExpertCacheFile", "MappedExperts", "cache_layout", "check_manifest", "write_expert_cache"]
