"""Expert cache files: the reference's on-disk format, pinned by its own builder.

``tests/golden/expert_cache`` was built by the reference's ``build_expert_cache``
(src/drama_low_vram/expert_cache_file.py:266-424) from a checkpoint whose
bytes are a known function of their position (make_expert_cache_golden.py).
"""

from __future__ import annotations

import json
import shutil
from pathlib import Path

import pytest
import torch

from drama_b200.expert_cache import (DATA_NAME, MANIFEST_NAME, ExpertCacheFile, cache_layout,
                                     write_expert_cache)
from golden.make_expert_cache_golden import EXPERTS, HIDDEN, INTER, LAYERS, pattern_layer

GOLDEN = Path(__file__).resolve().parent / "golden" / "expert_cache"


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.dtype == torch.float8_e4m3fn:
        a, b = a.view(torch.uint8), b.view(torch.uint8)
    return a.dtype == b.dtype and torch.equal(a, b)


def test_reference_built_cache_reads_back_by_position():
    with ExpertCacheFile.open(GOLDEN, verify_data=True) as cache:
        assert (cache.num_layers, cache.num_experts, cache.hidden, cache.intermediate) == \
            (LAYERS, EXPERTS, HIDDEN, INTER)
        for layer in range(LAYERS):
            want = pattern_layer(layer)
            got = cache.layer_buffers(layer)
            for name in want:
                assert _same(got[name], want[name]), (layer, name)
            assert cache.layer_store(layer) is cache.layer_store(layer)


def test_layout_matches_the_reference_manifest():
    manifest = json.loads((GOLDEN / MANIFEST_NAME).read_text())
    layers, total = cache_layout(LAYERS, EXPERTS, HIDDEN, INTER)
    assert manifest["layers"] == layers and manifest["data"]["size"] == total == 196_656


def test_writer_reproduces_the_reference_bytes(tmp_path):
    out = write_expert_cache(tmp_path / "ours", [pattern_layer(layer) for layer in range(LAYERS)])
    assert (out / DATA_NAME).read_bytes() == (GOLDEN / DATA_NAME).read_bytes()
    mine = json.loads((out / MANIFEST_NAME).read_text())
    ref = json.loads((GOLDEN / MANIFEST_NAME).read_text())
    for key in ("format", "format_version", "byte_order", "model", "data", "layers"):
        assert mine[key] == ref[key], key


def _tampered(tmp_path, edit):
    dst = tmp_path / "cache"
    shutil.copytree(GOLDEN, dst)
    manifest = json.loads((dst / MANIFEST_NAME).read_text())
    edit(manifest, dst)
    (dst / MANIFEST_NAME).write_text(json.dumps(manifest))
    return dst


@pytest.mark.parametrize("edit,error,message", [
    (lambda m, d: m.update(format="other"), ValueError, "manifest: format must be"),
    (lambda m, d: m.update(format_version=2), ValueError, "manifest: format_version must be"),
    (lambda m, d: m.update(format_version=True), ValueError, "manifest: format_version must be"),
    (lambda m, d: m.update(byte_order="big"), ValueError, "manifest: byte_order must be"),
    (lambda m, d: m["model"].update(block_size=64), ValueError, "manifest: model.block_size must be"),
    (lambda m, d: m["model"].pop("hidden"), ValueError, r"model.hidden must be an integer >= 1 \(missing\)"),
    (lambda m, d: m.update(model="fish_omni"), ValueError, "manifest: model must be a JSON object"),
    (lambda m, d: m["layers"][1]["buffers"]["w2_weight"].update(offset=0), ValueError, "layers do not match"),
    (lambda m, d: m["data"].update(size=m["data"]["size"] + 1), ValueError, "data.size is"),
    (lambda m, d: m["data"].update(sha256="xyz"), ValueError, "manifest: data.sha256 must be 64 lowercase hex"),
    (lambda m, d: m.update(model_fingerprint=None), ValueError, "manifest: model_fingerprint must be"),
    (lambda m, d: (d / DATA_NAME).write_bytes((d / DATA_NAME).read_bytes()[:-4]), ValueError, "truncated"),
])
def test_manifest_rejections(tmp_path, edit, error, message):
    with pytest.raises(error, match=message):
        ExpertCacheFile.open(_tampered(tmp_path, edit))


def test_checksum_catches_a_changed_byte(tmp_path):
    def flip(m, d):
        raw = bytearray((d / DATA_NAME).read_bytes())
        raw[1000] ^= 1
        (d / DATA_NAME).write_bytes(bytes(raw))
    path = _tampered(tmp_path, flip)
    ExpertCacheFile.open(path)  # geometry still valid
    with pytest.raises(ValueError, match="checksum mismatch"):
        ExpertCacheFile.open(path, verify_data=True)


def test_layer_and_window_checks_before_any_device_call():
    cache = ExpertCacheFile.open(GOLDEN)
    with pytest.raises(IndexError):
        cache.layer_buffers(LAYERS)
    with pytest.raises(IndexError):
        cache.register(0, LAYERS + 1)
    with pytest.raises(IndexError):
        cache.register(True)
    cache.close()
    with pytest.raises(RuntimeError, match="closed"):
        cache.layer_buffers(0)
