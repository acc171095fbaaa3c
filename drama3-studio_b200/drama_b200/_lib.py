"""ctypes binding of ``libdrama_b200.so`` (the C ABI in ``include/drama_b200.h``).

Mirrors the reference's binding style (``src/drama_low_vram/native_backend.py:
56-173``): argtypes declared once, every call's status checked, the thread-local
error text raised as ``RuntimeError``. There is no fallback: if the library is
missing the import of any compute entry point fails loudly.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

from .build import LIB_PATH

F32, F16, BF16, I32, I64 = 0, 1, 2, 3, 4
ABI_VERSION = 1

DTYPE_CODES = {
    torch.float32: F32,
    torch.float16: F16,
    torch.bfloat16: BF16,
    torch.int32: I32,
    torch.int64: I64,
}

EXPORTS = (
    "drama_b200_abi",
    "drama_b200_error",
    "drama_b200_device_check",
    "drama_b200_route_topk",
    "drama_b200_permute_routes",
    "drama_b200_permute_routes_wide_scratch_bytes",
    "drama_b200_permute_routes_wide",
    "drama_b200_decode_workspace_bytes",
    "drama_b200_decode_status_offset",
    "drama_b200_fp8_decode",
    "drama_b200_int4_decode",
    "drama_b200_fp8_w8a8_workspace_bytes",
    "drama_b200_fp8_w8a8_decode",
    "drama_b200_fp8_w8a8_prefill_supported",
    "drama_b200_fp8_w8a8_prefill_workspace_bytes",
    "drama_b200_fp8_w8a8_prefill",
    "drama_b200_w8a8_workspace_bytes",
    "drama_b200_w8a8_decode",
    "drama_b200_shared_expert_workspace_bytes",
    "drama_b200_shared_expert",
    "drama_b200_moe_layer_workspace_bytes",
    "drama_b200_fp8_moe_layer",
    "drama_b200_fp8_moe_layer_logits",
    "drama_b200_moe_layer_launches",
    "drama_b200_fp8_moe_router",
    "drama_b200_fp8_moe_experts",
    "drama_b200_prefill_workspace_bytes",
    "drama_b200_prefill_status_offset",
    "drama_b200_fp8_prefill",
    "drama_b200_static_scratch_bytes",
    "drama_b200_fp8_decode_static",
    "drama_b200_expert_rows_workspace_bytes",
    "drama_b200_fp8_expert_rows",
    "drama_b200_ep_dispatch",
    "drama_b200_ep_combine",
    "drama_b200_ep_buffers_alloc",
    "drama_b200_ep_buffers_free",
    "drama_b200_ipc_handle",
    "drama_b200_ipc_open",
    "drama_b200_ipc_close",
    "drama_b200_ep_p2p_dispatch",
    "drama_b200_fp8_expert_rows_p2p",
    "drama_b200_ep_p2p_combine",
    "drama_b200_stage_copies",
    "drama_b200_host_register",
    "drama_b200_host_unregister",
    "drama_b200_host_locked",
)

c_void_p, c_int, c_int64, c_size_t = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t


class Fp8Bank(ctypes.Structure):
    _fields_ = [
        ("w13", c_void_p), ("w13_scale", c_void_p), ("w2", c_void_p), ("w2_scale", c_void_p),
        ("w13_slot_stride", c_int64), ("w13_row_stride", c_int64),
        ("w13_scale_slot_stride", c_int64), ("w13_scale_row_stride", c_int64),
        ("w2_slot_stride", c_int64), ("w2_row_stride", c_int64),
        ("w2_scale_slot_stride", c_int64), ("w2_scale_row_stride", c_int64),
        ("slots", ctypes.c_int32), ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


class Int4Bank(ctypes.Structure):
    _fields_ = [
        ("w13", c_void_p), ("w13_scale", c_void_p), ("w13_zeros", c_void_p),
        ("w2", c_void_p), ("w2_scale", c_void_p), ("w2_zeros", c_void_p),
        ("w13_slot_stride", c_int64), ("w13_row_stride", c_int64),
        ("w13_scale_slot_stride", c_int64), ("w13_scale_row_stride", c_int64),
        ("w13_zeros_slot_stride", c_int64), ("w13_zeros_row_stride", c_int64),
        ("w2_slot_stride", c_int64), ("w2_row_stride", c_int64),
        ("w2_scale_slot_stride", c_int64), ("w2_scale_row_stride", c_int64),
        ("w2_zeros_slot_stride", c_int64), ("w2_zeros_row_stride", c_int64),
        ("scale_dtype", ctypes.c_int32), ("slots", ctypes.c_int32),
        ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
    ]


class W8a8Bank(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32),
        ("w13", c_void_p), ("w13_scale", c_void_p), ("w2", c_void_p), ("w2_scale", c_void_p),
        ("w13_slot_stride", c_int64), ("w13_row_stride", c_int64),
        ("w13_scale_slot_stride", c_int64), ("w13_scale_row_stride", c_int64),
        ("w2_slot_stride", c_int64), ("w2_row_stride", c_int64),
        ("w2_scale_slot_stride", c_int64), ("w2_scale_row_stride", c_int64),
        ("slots", ctypes.c_int32), ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
    ]


class SharedExpert(ctypes.Structure):
    _fields_ = [
        ("gate_proj", c_void_p), ("up_proj", c_void_p), ("down_proj", c_void_p), ("gate_weight", c_void_p),
        ("gate_row_stride", c_int64), ("up_row_stride", c_int64), ("down_row_stride", c_int64),
        ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
    ]


class EpPeers(ctypes.Structure):
    _fields_ = [
        ("ranks", ctypes.c_int32), ("rank", ctypes.c_int32), ("capacity", c_int64),
        ("hidden", ctypes.c_int32), ("experts", ctypes.c_int32),
        ("recv", c_void_p * 8), ("back", c_void_p * 8), ("signals", c_void_p * 8),
        ("epoch", c_void_p), ("done", c_void_p), ("wait_ns", c_int64),
    ]


class Library:
    """Loaded ``libdrama_b200.so`` with typed entry points."""

    def __init__(self, path: Path | str = LIB_PATH):
        self.path = Path(path).resolve()
        if not self.path.is_file():
            raise RuntimeError(
                f"drama_b200 CUDA library missing: {self.path}. Build it with "
                "drama_b200.build.build() (nvcc, sm_100a); there is no CPU fallback.")
        dll = ctypes.CDLL(str(self.path))
        self.dll = dll
        dll.drama_b200_abi.restype = c_int
        dll.drama_b200_error.restype = ctypes.c_char_p
        dll.drama_b200_device_check.argtypes = [c_int, ctypes.POINTER(c_int)]
        dll.drama_b200_route_topk.argtypes = [c_void_p, c_int, c_int64, c_int, c_int, c_int,
                                             c_void_p, c_int, c_void_p, c_int, c_void_p]
        dll.drama_b200_permute_routes.argtypes = [c_void_p, c_int, c_int64, c_int, c_void_p,
                                                 c_void_p, c_void_p, c_void_p, c_void_p]
        dll.drama_b200_decode_workspace_bytes.argtypes = [c_int64, c_int, c_int, c_int]
        dll.drama_b200_decode_workspace_bytes.restype = c_size_t
        dll.drama_b200_decode_status_offset.restype = c_size_t
        decode_args = [c_void_p, c_int, c_int64, c_int, c_void_p, c_int, c_void_p, c_int,
                       c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_fp8_decode.argtypes = [ctypes.POINTER(Fp8Bank)] + decode_args
        dll.drama_b200_int4_decode.argtypes = [ctypes.POINTER(Int4Bank)] + decode_args
        dll.drama_b200_fp8_w8a8_workspace_bytes.argtypes = [c_int64, c_int, c_int, c_int]
        dll.drama_b200_fp8_w8a8_workspace_bytes.restype = c_size_t
        dll.drama_b200_fp8_w8a8_decode.argtypes = [
            ctypes.POINTER(Fp8Bank), c_void_p, c_int64, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p,
            c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_permute_routes_wide_scratch_bytes.argtypes = [c_int64, c_int]
        dll.drama_b200_permute_routes_wide_scratch_bytes.restype = c_size_t
        dll.drama_b200_permute_routes_wide.argtypes = [c_void_p, c_int, c_int64, c_int, c_void_p, c_void_p, c_void_p,
                                                       c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]
        dll.drama_b200_permute_routes_wide.restype = c_int
        dll.drama_b200_fp8_w8a8_prefill_supported.argtypes = [c_int, c_int, c_int]
        dll.drama_b200_fp8_w8a8_prefill_supported.restype = c_int
        dll.drama_b200_fp8_w8a8_prefill_workspace_bytes.argtypes = [c_int64, c_int, c_int, c_int, c_int]
        dll.drama_b200_fp8_w8a8_prefill_workspace_bytes.restype = c_size_t
        dll.drama_b200_fp8_w8a8_prefill.argtypes = [
            ctypes.POINTER(Fp8Bank), c_void_p, c_int64, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p,
            c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_fp8_w8a8_prefill.restype = c_int
        dll.drama_b200_w8a8_decode.argtypes = [ctypes.POINTER(W8a8Bank)] + decode_args
        dll.drama_b200_w8a8_decode.restype = c_int
        dll.drama_b200_w8a8_workspace_bytes.argtypes = [c_int64, c_int, c_int, c_int]
        dll.drama_b200_w8a8_workspace_bytes.restype = c_size_t
        dll.drama_b200_shared_expert_workspace_bytes.argtypes = [c_int64, c_int, c_int]
        dll.drama_b200_shared_expert_workspace_bytes.restype = c_size_t
        dll.drama_b200_shared_expert.argtypes = [ctypes.POINTER(SharedExpert), c_void_p, c_int64, c_void_p, c_void_p,
                                                 c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_shared_expert.restype = c_int
        dll.drama_b200_moe_layer_workspace_bytes.argtypes = [c_int64, c_int, c_int, c_int, c_int]
        dll.drama_b200_moe_layer_workspace_bytes.restype = c_size_t
        dll.drama_b200_fp8_moe_layer.argtypes = [
            ctypes.POINTER(Fp8Bank), c_void_p, c_void_p, c_void_p, ctypes.c_float, c_void_p, c_void_p,
            c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_moe_layer_launches.argtypes = [c_int64, c_int, c_int, c_int, c_int]
        dll.drama_b200_moe_layer_launches.restype = c_int
        dll.drama_b200_fp8_moe_layer_logits.argtypes = [
            ctypes.POINTER(Fp8Bank), c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p,
            c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_fp8_moe_router.argtypes = [
            ctypes.POINTER(Fp8Bank), c_void_p, c_void_p, c_void_p, ctypes.c_float, c_void_p,
            c_int64, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_fp8_moe_experts.argtypes = [
            ctypes.POINTER(Fp8Bank), c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p, c_size_t,
            c_void_p]
        dll.drama_b200_prefill_workspace_bytes.argtypes = [c_int64, c_int, c_int, c_int, c_int]
        dll.drama_b200_prefill_workspace_bytes.restype = c_size_t
        dll.drama_b200_prefill_status_offset.restype = c_size_t
        dll.drama_b200_fp8_prefill.argtypes = [ctypes.POINTER(Fp8Bank), c_void_p, c_int64, c_int, c_void_p, c_int,
                                               c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_fp8_prefill.restype = c_int
        dll.drama_b200_static_scratch_bytes.restype = c_size_t
        dll.drama_b200_fp8_decode_static.argtypes = [ctypes.POINTER(Fp8Bank)] + decode_args[:10] + [c_void_p]
        dll.drama_b200_fp8_decode_static.restype = c_int
        dll.drama_b200_stage_copies.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p]
        dll.drama_b200_stage_copies.restype = c_int
        dll.drama_b200_host_register.argtypes = [c_void_p, ctypes.c_uint64, c_int, ctypes.POINTER(c_void_p),
                                                 ctypes.POINTER(ctypes.c_uint64)]
        dll.drama_b200_host_unregister.argtypes = [c_void_p]
        dll.drama_b200_host_locked.argtypes = [c_void_p, ctypes.c_uint64, ctypes.POINTER(c_int)]
        dll.drama_b200_expert_rows_workspace_bytes.argtypes = [c_int64, c_int, c_int, c_int]
        dll.drama_b200_expert_rows_workspace_bytes.restype = c_size_t
        dll.drama_b200_fp8_expert_rows.argtypes = [ctypes.POINTER(Fp8Bank), c_void_p, c_int64, c_int64, c_void_p,
                                                   c_int, c_void_p, c_void_p, c_size_t, c_void_p]
        dll.drama_b200_fp8_expert_rows.restype = c_int
        dll.drama_b200_ep_dispatch.argtypes = [c_void_p, c_int64, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                               c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                               c_void_p]
        dll.drama_b200_ep_dispatch.restype = c_int
        dll.drama_b200_ep_combine.argtypes = [c_void_p, c_int64, c_void_p, c_void_p, c_int, c_int64, c_int, c_int,
                                              c_void_p, c_void_p, c_void_p]
        dll.drama_b200_ep_combine.restype = c_int
        vpp = ctypes.POINTER(c_void_p)
        dll.drama_b200_ep_buffers_alloc.argtypes = [c_int, c_int64, c_int, vpp, vpp, vpp, vpp]
        dll.drama_b200_ep_buffers_free.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p]
        dll.drama_b200_ipc_handle.argtypes = [c_void_p, c_void_p]
        dll.drama_b200_ipc_open.argtypes = [c_void_p, vpp]
        dll.drama_b200_ipc_close.argtypes = [c_void_p]
        peers = ctypes.POINTER(EpPeers)
        dll.drama_b200_ep_p2p_dispatch.argtypes = [peers, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p,
                                                   c_void_p, c_void_p, c_void_p]
        dll.drama_b200_fp8_expert_rows_p2p.argtypes = [ctypes.POINTER(Fp8Bank), peers, c_void_p, c_size_t, c_void_p,
                                                       c_void_p]
        dll.drama_b200_ep_p2p_combine.argtypes = [peers, c_void_p, c_void_p, c_int, c_int64, c_int, c_void_p,
                                                  c_void_p, c_void_p, c_void_p]
        for name in ("drama_b200_ep_buffers_alloc", "drama_b200_ep_buffers_free", "drama_b200_ipc_handle",
                     "drama_b200_ipc_open", "drama_b200_ipc_close", "drama_b200_ep_p2p_dispatch",
                     "drama_b200_fp8_expert_rows_p2p", "drama_b200_ep_p2p_combine"):
            getattr(dll, name).restype = c_int
        for name in ("drama_b200_device_check", "drama_b200_route_topk", "drama_b200_permute_routes",
                     "drama_b200_fp8_decode", "drama_b200_int4_decode", "drama_b200_fp8_moe_layer",
                     "drama_b200_fp8_moe_router", "drama_b200_fp8_moe_experts"):
            getattr(dll, name).restype = c_int
        if dll.drama_b200_abi() != ABI_VERSION:
            raise RuntimeError("Unsupported drama_b200 ABI version")

    def check(self, status: int) -> None:
        if status:
            message = self.dll.drama_b200_error()
            raise RuntimeError(message.decode("utf-8", errors="replace") if message else "drama_b200 error")

    def host_locked(self, ptr: int, nbytes: int) -> bool:
        """Whether both ends of a host byte range are page-locked (pinned or registered)."""
        locked = c_int(0)
        self.check(self.dll.drama_b200_host_locked(ptr, nbytes, ctypes.byref(locked)))
        return bool(locked.value)

    def device_check(self, device: int) -> int:
        count = c_int(0)
        self.check(self.dll.drama_b200_device_check(device, ctypes.byref(count)))
        return count.value


_LIB: Library | None = None
_LOCK = threading.Lock()


def library() -> Library:
    global _LIB
    if _LIB is None:
        with _LOCK:
            if _LIB is None:
                _LIB = Library()
    return _LIB


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
