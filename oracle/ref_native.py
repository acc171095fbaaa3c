"""ctypes handle on the reference's native CPU expert core built under oracle/_ref.

TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline; never the product).
The library is the reference's own ``native/src/*.cpp`` (ABI v1, declared in
``native/include/drama_native.h:1-90``) compiled by ``oracle/Makefile``. The
binding mirrors ``src/drama_low_vram/native_backend.py:56-173`` for the calls
used here: FP8 decode, bf16->FP8 1x128 quantisation and the W8A8 executor.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_ref" / "libdrama_native.so"


class ReferenceNative:
    def __init__(self, path: Path | str = LIB_PATH):
        path = Path(path)
        if not path.is_file():
            raise FileNotFoundError(f"reference native core not built: {path} (run make -C oracle)")
        self.dll = ctypes.CDLL(str(path))
        d = self.dll
        d.drama_native_abi.restype = ctypes.c_int
        d.drama_native_features.restype = ctypes.c_int
        d.drama_native_error.restype = ctypes.c_char_p
        d.drama_decode_fp8.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        d.drama_quantize_bf16.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int]
        d.drama_executor_create.argtypes = [ctypes.c_int] * 5
        d.drama_executor_create.restype = ctypes.c_void_p
        d.drama_executor_destroy.argtypes = [ctypes.c_void_p]
        d.drama_executor_destroy.restype = None
        d.drama_executor_forward.argtypes = (
            [ctypes.c_void_p] * 5 + [ctypes.c_int] + [ctypes.c_void_p] * 3
            + [ctypes.c_int, ctypes.c_void_p])
        if d.drama_native_abi() != 1:
            raise RuntimeError("unexpected reference native ABI")
        self.features = d.drama_native_features()

    def check(self, status: int) -> None:
        if status:
            raise RuntimeError(self.dll.drama_native_error().decode())

    def decode(self, raw: np.ndarray) -> np.ndarray:
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        out = np.empty(raw.shape, dtype=np.float32)
        self.check(self.dll.drama_decode_fp8(raw.ctypes.data, out.ctypes.data, raw.size))
        return out

    def quantize(self, bf16_bits: np.ndarray):
        v = np.ascontiguousarray(bf16_bits, dtype=np.uint16)
        q = np.empty(v.shape, dtype=np.uint8)
        s = np.empty(v.size // 128, dtype=np.float32)
        self.check(self.dll.drama_quantize_bf16(v.ctypes.data, q.ctypes.data, s.ctypes.data, v.size))
        return q, s

    def executor(self, hidden: int, intermediate: int, capacity: int = 8, threads: int = 1,
                 implementation: int = 0) -> "Executor":
        return Executor(self, hidden, intermediate, capacity, threads, implementation)


class Executor:
    """One bf16 row -> ordered fp32 weighted partials (runtime.cpp:68-276)."""

    def __init__(self, lib: ReferenceNative, hidden, intermediate, capacity, threads, implementation):
        self.lib = lib
        self.handle = lib.dll.drama_executor_create(hidden, intermediate, capacity, threads, implementation)
        if not self.handle:
            lib.check(-1)
        self.hidden = hidden

    def forward(self, bank: dict, x_bf16_bits: np.ndarray, ids: np.ndarray, weights: np.ndarray,
                out: np.ndarray | None = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int64).reshape(-1)
        weights = np.ascontiguousarray(weights, dtype=np.float32).reshape(-1)
        x = np.ascontiguousarray(x_bf16_bits, dtype=np.uint16).reshape(-1)
        if out is None:
            out = np.empty((ids.size, self.hidden), dtype=np.float32)
        arrays = [np.ascontiguousarray(bank[name]) for name in
                  ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv")]
        self.lib.check(self.lib.dll.drama_executor_forward(
            self.handle, *[a.ctypes.data for a in arrays], arrays[0].shape[0],
            x.ctypes.data, ids.ctypes.data, weights.ctypes.data, ids.size, out.ctypes.data))
        return out

    def close(self) -> None:
        if self.handle:
            self.lib.dll.drama_executor_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
