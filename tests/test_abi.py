"""The C-ABI library loads on any host and exports exactly what the header
declares; argument validation fails before any CUDA work (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "drama_b200.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"DRAMA_B200_API\s+[\w\s\*]+?\b(drama_b200_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    from drama_b200 import _lib

    return _lib.library()


def test_header_declares_entry_points():
    names = declared()
    assert {"drama_b200_abi", "drama_b200_error", "drama_b200_fp8_decode", "drama_b200_int4_decode",
            "drama_b200_route_topk", "drama_b200_permute_routes", "drama_b200_fp8_moe_layer"} <= names


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib.path)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (drama_b200_\w+)", out))
    assert declared() <= exported, sorted(declared() - exported)
    assert exported <= declared(), sorted(exported - declared())
    from drama_b200 import _lib

    assert set(_lib.EXPORTS) == declared()
    for name in declared():
        assert getattr(lib.dll, name) is not None


def test_abi_version(lib):
    assert lib.dll.drama_b200_abi() == 1


def test_validation_errors_before_any_launch(lib):
    d = lib.dll
    assert d.drama_b200_route_topk(None, 2, 1, 128, 8, 1, None, 4, None, 2, None) == -1
    assert b"required" in d.drama_b200_error()
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.addressof(buf)
    assert d.drama_b200_route_topk(p, 2, 1, 128, 40, 1, p + 32, 4, p + 48, 2, None) == -1
    assert b"top_k" in d.drama_b200_error()
    assert d.drama_b200_permute_routes(p, 4, 1, 0, p, p, p, None, None) == -1
    assert b"experts" in d.drama_b200_error()
    from drama_b200._lib import Fp8Bank

    bank = Fp8Bank()
    bank.hidden, bank.intermediate, bank.slots = 2048, 768, 8
    assert d.drama_b200_fp8_decode(ctypes.byref(bank), p, 2, 1, 8, p, 4, p, 2, None, None, None, 0, None) == -1
    assert b"either out or pair_out" in d.drama_b200_error()
    assert d.drama_b200_fp8_decode(ctypes.byref(bank), p, 2, 1000, 8, p, 4, p, 2, p, None, None, 0, None) == -1
    assert b"at most" in d.drama_b200_error()


def test_moe_layer_rejects_unaligned_rows(lib):
    """The fused layer reads and writes hidden rows 16 bytes at a time; an
    unaligned row is refused before any launch."""
    from drama_b200._lib import Fp8Bank

    d = lib.dll
    buf = (ctypes.c_uint8 * 512)()
    a = (ctypes.addressof(buf) + 255) & ~255  # 256-byte aligned stand-in pointers (never dereferenced)
    bank = Fp8Bank()
    bank.w13 = bank.w13_scale = bank.w2 = bank.w2_scale = a
    bank.w13_row_stride = bank.w2_row_stride = bank.w13_slot_stride = bank.w2_slot_stride = 2048
    bank.hidden, bank.intermediate, bank.slots = 2048, 768, 128

    def call(hidden_in, hidden_out, moe_out=None):
        return d.drama_b200_fp8_moe_layer(ctypes.byref(bank), ctypes.c_void_p(a), None, ctypes.c_void_p(a),
                                          ctypes.c_float(1e-6), ctypes.c_void_p(hidden_in),
                                          ctypes.c_void_p(hidden_out), ctypes.c_int64(1), 8, None, None, None,
                                          ctypes.c_void_p(moe_out), ctypes.c_void_p(a), ctypes.c_size_t(0), None)

    for args in ((a + 2, a + 256), (a, a + 258), (a, a + 256, a + 8)):
        assert call(*args) == -1
        assert b"16-byte" in d.drama_b200_error()


def test_product_code_never_imports_the_oracle():
    for path in (REPO / "drama3-studio_b200").rglob("*.py"):
        text = path.read_text()
        assert "oracle" not in re.findall(r"^\s*(?:from|import)\s+(\w+)", text, re.M), path


def test_w8a8_prefill_workspace_holds_every_region(lib):
    """The tcgen05 prefill's workspace (a host-side size, no GPU) covers what
    one call carves from it: per pair the sorted order, sorted position and
    route weight at the sorted row, the E4M3 token and SwiGLU rows with their
    1x128 scales (128 rows of tile overrun), and the fp32 pair rows."""
    size = lib.dll.drama_b200_fp8_w8a8_prefill_workspace_bytes
    tokens, top_k, hidden, inter, experts = 4096, 8, 2048, 768, 128
    pairs, rows = tokens * top_k, tokens * top_k + 128
    floor = (pairs * (8 + 8 + 4) + rows * (hidden + inter) + rows * (hidden // 128 + inter // 128) * 4
             + pairs * hidden * 4)
    assert size(tokens, top_k, hidden, inter, experts) >= floor
    sizes = [size(t, top_k, hidden, inter, experts) for t in (0, 1, 64, 4096)]
    assert sizes[0] > 0 and sizes == sorted(sizes) and len(set(sizes)) == len(sizes)
