"""Expert backends for ``ExpertOffloadManager`` running the sm_100a kernels.

``B200ExpertBackend`` implements the reference's ``ExpertBackend`` protocol
(``src/drama_low_vram/offload.py:187-196``) for FP8 128x128 block-scaled banks
with the arithmetic of ``TorchExpertBackend`` (``offload.py:199-244``, the
PyTorch W16A16 dequant path), plus ``forward_decode_pairs``
(``offload.py:346-356``) which the manager calls for batch-1 partitions.
``QuantizedB200Backend(mode)`` replaces ``QuantizedExpertBackend(mode)``
(``src/drama_low_vram/quantized_kernels.py:217-248``): GPTQ W4A16 banks (mode
0, additionally with asymmetric uint4 zero-points) and the W8A8 INT8-ConvRot,
W6A8 and W4A8-codebook banks (modes 1-3).

Both are drop-ins: ``install_expert_offload(backbone, backend=B200ExpertBackend())``
(``offload.py:1534-1569``) needs no other change. Every call enqueues work on
``torch.cuda.current_stream`` and, apart from the optional slot-range check,
never synchronises, so the calls can sit inside a CUDA graph.
"""

from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _lib

FP8_DTYPE = torch.float8_e4m3fn
FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)
MAX_DECODE_PAIRS = 4096
PREFILL_MIN_PAIRS = 512  # below this the decode GEMVs are faster than a tensor-core tile


@dataclass(frozen=True)
class QuantizedBank:
    """INT4 bank in the reference's GPTQ layout with optional zero-points.

    ``w13_weight [S, 2I, H/8] int32``, ``w13_scale_inv [S, 2I, H/128]`` bf16 or
    fp16, ``w2_weight [S, H, I/8]``, ``w2_scale_inv [S, H, I/128]``; the
    ``*_qzeros`` tensors are ``[S, N/8, K/128] int32`` (nibble n%8 of word n/8)
    or None for the reference's implicit zero-point 8.
    """

    w13_weight: Tensor
    w13_scale_inv: Tensor
    w2_weight: Tensor
    w2_scale_inv: Tensor
    w13_qzeros: Tensor | None = None
    w2_qzeros: Tensor | None = None

    @property
    def count(self) -> int:
        return self.w13_weight.shape[0]


class _Workspace:
    """Zero-initialised device scratch, one per (device, stream), grown on demand."""

    def __init__(self) -> None:
        self._buffers: dict[tuple[int, int], Tensor] = {}
        # Buffers outgrown by a later call stay alive: a CUDA graph captured
        # while one was current keeps writing to it on every replay.
        self._retired: list[Tensor] = []
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> Tensor:
        stream = torch.cuda.current_stream(device).cuda_stream
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream)
        with self._lock:
            buf = self._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError(
                        "drama_b200 workspace must be allocated before CUDA graph capture; "
                        "run one eager call of the same size first")
                if buf is not None:
                    self._retired.append(buf)
                buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                self._buffers[key] = buf
            return buf


_WORKSPACES = _Workspace()
_PREFILL_WORKSPACES = _Workspace()


def _rows(t: Tensor) -> Tensor:
    """Innermost dimension contiguous (the kernels' only layout requirement)."""
    return t if t.stride(-1) == 1 else t.contiguous()


def _check_common(x: Tensor, ids: Tensor, weights: Tensor, count: int, hidden: int,
                  validate_ids: bool) -> None:
    if x.ndim != 2 or x.shape[-1] != hidden:
        raise ValueError(f"Expected hidden rows [N, {hidden}], got {tuple(x.shape)}")
    if not x.is_cuda:
        raise RuntimeError("drama_b200 backends need CUDA tensors on an sm_100 GPU")
    if x.dtype not in FLOAT_DTYPES:
        raise ValueError("Expert compute dtype must be float16, bfloat16 or float32")
    if ids.dtype not in (torch.int32, torch.int64):
        raise ValueError("Expert IDs must have an integer dtype")
    if not weights.is_floating_point():
        raise ValueError("Routing weights must be floating point")
    if ids.device != x.device or weights.device != x.device:
        raise ValueError("Hidden states, expert IDs and routing weights must share a device")
    if validate_ids and ids.numel() and not torch.cuda.is_current_stream_capturing():
        bad = ((ids < 0) | (ids >= count)).any()
        if bool(bad):
            first = int(ids[(ids < 0) | (ids >= count)].reshape(-1)[0])
            raise ValueError(f"Local expert slot {first} is outside the staging pool")


def _fp8_bank(staged, hidden: int) -> tuple[_lib.Fp8Bank, tuple]:
    w13 = _rows(staged.w13_weight)
    w2 = _rows(staged.w2_weight)
    s13 = _rows(staged.w13_scale_inv)
    s2 = _rows(staged.w2_scale_inv)
    for name, t, dt in (("w13_weight", w13, FP8_DTYPE), ("w2_weight", w2, FP8_DTYPE),
                        ("w13_scale_inv", s13, torch.float32), ("w2_scale_inv", s2, torch.float32)):
        if t.dtype != dt:
            raise ValueError(f"{name} must be {dt}; got {t.dtype}")
        if t.ndim != 3:
            raise ValueError(f"{name} must be a stacked three-dimensional tensor")
    slots, gate_up, h = w13.shape
    inter = gate_up // 2
    if h != hidden or tuple(w2.shape) != (slots, hidden, inter):
        raise ValueError("FP8 bank geometry does not match the hidden size")
    if tuple(s13.shape) != (slots, gate_up // 128, hidden // 128) or \
            tuple(s2.shape) != (slots, hidden // 128, inter // 128):
        raise ValueError("FP8 weight shape does not match its 128x128 block scales")
    if w13.stride(1) % 16 or w13.stride(0) % 16 or w13.data_ptr() % 16:
        w13 = w13.contiguous()
    if w2.stride(1) % 16 or w2.stride(0) % 16 or w2.data_ptr() % 16:
        w2 = w2.contiguous()
    bank = _lib.Fp8Bank(
        w13.data_ptr(), s13.data_ptr(), w2.data_ptr(), s2.data_ptr(),
        w13.stride(0), w13.stride(1), s13.stride(0), s13.stride(1),
        w2.stride(0), w2.stride(1), s2.stride(0), s2.stride(1),
        slots, hidden, inter, 0)
    return bank, (w13, w2, s13, s2)


def _int4_bank(staged, hidden: int) -> tuple[_lib.Int4Bank, tuple]:
    w13 = _rows(staged.w13_weight)
    w2 = _rows(staged.w2_weight)
    s13 = _rows(staged.w13_scale_inv)
    s2 = _rows(staged.w2_scale_inv)
    z13 = getattr(staged, "w13_qzeros", None)
    z2 = getattr(staged, "w2_qzeros", None)
    z13 = None if z13 is None else _rows(z13)
    z2 = None if z2 is None else _rows(z2)
    if w13.dtype != torch.int32 or w2.dtype != torch.int32:
        raise ValueError("Quantized weight dtype mismatch")
    if s13.dtype not in (torch.bfloat16, torch.float16) or s2.dtype != s13.dtype:
        raise ValueError("Quantized scale dtype mismatch")
    slots, gate_up, h8 = w13.shape
    inter = gate_up // 2
    if h8 * 8 != hidden or tuple(w2.shape) != (slots, hidden, inter // 8):
        raise ValueError("Quantized weight/scale geometry mismatch")
    if tuple(s13.shape) != (slots, gate_up, hidden // 128) or tuple(s2.shape) != (slots, hidden, inter // 128):
        raise ValueError("Quantized weight/scale geometry mismatch")
    for z, n, k in ((z13, gate_up, hidden), (z2, hidden, inter)):
        if z is not None and (z.dtype != torch.int32 or tuple(z.shape) != (slots, n // 8, k // 128)):
            raise ValueError("Quantized zero-point geometry mismatch")
    if w13.stride(1) % 4 or w13.stride(0) % 4 or w13.data_ptr() % 16:
        w13 = w13.contiguous()
    if w2.stride(1) % 4 or w2.stride(0) % 4 or w2.data_ptr() % 16:
        w2 = w2.contiguous()
    bank = _lib.Int4Bank(
        w13.data_ptr(), s13.data_ptr(), _lib.ptr(z13), w2.data_ptr(), s2.data_ptr(), _lib.ptr(z2),
        w13.stride(0), w13.stride(1), s13.stride(0), s13.stride(1),
        0 if z13 is None else z13.stride(0), 0 if z13 is None else z13.stride(1),
        w2.stride(0), w2.stride(1), s2.stride(0), s2.stride(1),
        0 if z2 is None else z2.stride(0), 0 if z2 is None else z2.stride(1),
        _lib.DTYPE_CODES[s13.dtype], slots, hidden, inter)
    return bank, (w13, w2, s13, s2, z13, z2)


class _DecodeBackend:
    """Shared forward / forward_pairs plumbing around one C entry point."""

    entry = ""

    def __init__(self, *, validate_ids: bool = True) -> None:
        self.validate_ids = validate_ids

    def _bank(self, staged, hidden):  # pragma: no cover - overridden
        raise NotImplementedError

    def _workspace_bytes(self, lib, tokens, top_k, hidden, intermediate) -> int:
        return lib.dll.drama_b200_decode_workspace_bytes(tokens, top_k, hidden, intermediate)

    def _run(self, x: Tensor, ids: Tensor, weights: Tensor, staged, *, combine: bool) -> Tensor:
        hidden = x.shape[-1]
        bank, keep = self._bank(staged, hidden)
        _check_common(x, ids, weights, bank.slots, hidden, self.validate_ids)
        tokens, top_k = ids.shape
        x = x.contiguous()
        ids = ids.contiguous()
        weights = weights.contiguous()
        if weights.dtype not in FLOAT_DTYPES:
            weights = weights.float()
        if tokens * top_k > MAX_DECODE_PAIRS:
            return self._chunked(x, ids, weights, staged, combine=combine)
        lib = _lib.library()
        if combine:
            out, pair_out = torch.empty_like(x), None
        else:
            out, pair_out = None, torch.empty((tokens * top_k, hidden), device=x.device, dtype=torch.float32)
        nbytes = self._workspace_bytes(lib, tokens, top_k, hidden, bank.intermediate)
        ws = _WORKSPACES.get(x.device, nbytes)
        fn = getattr(lib.dll, self.entry)
        lib.check(fn(ctypes.byref(bank), x.data_ptr(), _lib.DTYPE_CODES[x.dtype], tokens, top_k,
                     ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype], weights.data_ptr(),
                     _lib.DTYPE_CODES[weights.dtype], _lib.ptr(out), _lib.ptr(pair_out),
                     ws.data_ptr(), ws.numel(), _lib.stream_handle(x.device)))
        del keep
        return out if combine else pair_out

    def _chunked(self, x, ids, weights, staged, *, combine: bool) -> Tensor:
        tokens, top_k = ids.shape
        rows = max(1, MAX_DECODE_PAIRS // top_k)
        parts = [self._run(x[s:s + rows], ids[s:s + rows], weights[s:s + rows], staged, combine=combine)
                 for s in range(0, tokens, rows)]
        return torch.cat(parts)

    def forward(self, x: Tensor, ids: Tensor, weights: Tensor, staged) -> Tensor:
        """[T,H] expert output in x's dtype (route slots summed in slot order)."""
        if ids.ndim != 2 or ids.shape[0] != x.shape[0]:
            raise ValueError("Expert IDs must have shape [tokens, top_k]")
        if weights.shape != ids.shape:
            raise ValueError("Routing weights must match IDs and top_k must be positive")
        if x.shape[0] == 0:
            return torch.zeros_like(x)
        return self._run(x, ids, weights, staged, combine=True)

    def forward_pairs(self, x: Tensor, ids: Tensor, weights: Tensor, staged) -> Tensor:
        """Weighted [pairs, hidden] contributions in float32, before summing."""
        if ids.shape != (x.shape[0], 1) or weights.shape != ids.shape:
            raise ValueError("Pair backend expects one expert and weight per input row")
        if x.shape[0] == 0:
            return torch.empty_like(x, dtype=torch.float32)
        return self._run(x, ids, weights, staged, combine=False)

    def forward_decode_pairs(self, x: Tensor, ids: Tensor, weights: Tensor, staged) -> Tensor:
        """Small partition of one decode row (offload.py:346-356); fp32 partials."""
        return self.forward_pairs(x, ids, weights, staged)


class B200ExpertBackend(_DecodeBackend):
    """FP8 (E4M3, 128x128 block scales) experts; TorchExpertBackend arithmetic.

    ``forward`` on bf16 rows with at least ``prefill_min_pairs`` (token, slot)
    pairs runs the grouped tensor-core GEMMs (``fp8_prefill``); smaller calls and
    ``forward_pairs`` run the decode GEMV kernels.
    """

    entry = "drama_b200_fp8_decode"

    def __init__(self, *, validate_ids: bool = True, prefill_min_pairs: int = PREFILL_MIN_PAIRS) -> None:
        super().__init__(validate_ids=validate_ids)
        self.prefill_min_pairs = prefill_min_pairs

    def _bank(self, staged, hidden):
        return _fp8_bank(staged, hidden)

    def forward(self, x: Tensor, ids: Tensor, weights: Tensor, staged) -> Tensor:
        if (x.dtype == torch.bfloat16 and ids.ndim == 2 and ids.shape[0] == x.shape[0] and x.ndim == 2
                and ids.numel() >= self.prefill_min_pairs and x.shape[1] % 256 == 0
                and staged.w2_weight.shape[-1] % 128 == 0):
            if weights.shape != ids.shape:
                raise ValueError("Routing weights must match IDs and top_k must be positive")
            return fp8_prefill(x, ids, weights, staged, validate_ids=self.validate_ids)
        return super().forward(x, ids, weights, staged)


class Fp8W8a8B200Backend(_DecodeBackend):
    """FP8 experts with the official W8A8 arithmetic of ``TritonExpertBackend``.

    The reference's production GPU backend (``offload.py:247-356``) runs the
    upstream FP8 MoE kernels: token rows and SwiGLU rows quantised to E4M3 in
    1x128 blocks, E4M3 x E4M3 block dots promoted with both block scales
    (``fp8_decode.py:114-147``; CPU statement ``native/src/runtime.cpp:
    162-237``). This backend computes that contract on the same staged banks
    as ``B200ExpertBackend`` (whose arithmetic is the W16A16 dequant path of
    ``TorchExpertBackend``); rows must be bfloat16.

    From ``prefill_min_pairs`` (token, slot) pairs on, a call runs as grouped
    GEMMs on the tcgen05 tensor cores (``drama_b200_fp8_w8a8_prefill``); below
    it, as per-pair tensor-core cells (``drama_b200_fp8_w8a8_decode``).
    """

    entry = "drama_b200_fp8_w8a8_decode"

    def __init__(self, *, validate_ids: bool = True, prefill_min_pairs: int = 512) -> None:
        super().__init__(validate_ids=validate_ids)
        self.prefill_min_pairs = prefill_min_pairs

    def _prefill(self, lib, bank, x, ids, weights, out, pair_out) -> bool:
        tokens, top_k = ids.shape
        if tokens * top_k < self.prefill_min_pairs or not lib.dll.drama_b200_fp8_w8a8_prefill_supported(
                bank.hidden, bank.intermediate, bank.slots):
            return False
        nbytes = lib.dll.drama_b200_fp8_w8a8_prefill_workspace_bytes(tokens, top_k, bank.hidden, bank.intermediate,
                                                                      bank.slots)
        ws = _WORKSPACES.get(x.device, nbytes)
        lib.check(lib.dll.drama_b200_fp8_w8a8_prefill(
            ctypes.byref(bank), x.data_ptr(), tokens, top_k, ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype],
            weights.data_ptr(), _lib.DTYPE_CODES[weights.dtype], _lib.ptr(out), _lib.ptr(pair_out), ws.data_ptr(),
            ws.numel(), _lib.stream_handle(x.device)))
        return True

    def _bank(self, staged, hidden):
        return _fp8_bank(staged, hidden)

    def _workspace_bytes(self, lib, tokens, top_k, hidden, intermediate) -> int:
        return lib.dll.drama_b200_fp8_w8a8_workspace_bytes(tokens, top_k, hidden, intermediate)

    def _run(self, x: Tensor, ids: Tensor, weights: Tensor, staged, *, combine: bool,
             x_fp8: Tensor | None = None, x_scale: Tensor | None = None) -> Tensor:
        if x.dtype != torch.bfloat16:
            raise ValueError("The FP8 W8A8 backend quantises bfloat16 hidden rows")
        hidden = x.shape[-1]
        bank, keep = self._bank(staged, hidden)
        _check_common(x, ids, weights, bank.slots, hidden, self.validate_ids)
        tokens, top_k = ids.shape
        lib = _lib.library()
        prefill = (x_fp8 is None and x_scale is None and tokens * top_k >= self.prefill_min_pairs
                   and lib.dll.drama_b200_fp8_w8a8_prefill_supported(hidden, bank.intermediate, bank.slots))
        if tokens * top_k > MAX_DECODE_PAIRS and not prefill:
            return self._chunked(x, ids, weights, staged, combine=combine)
        x, ids, weights = x.contiguous(), ids.contiguous(), weights.contiguous()
        if weights.dtype not in FLOAT_DTYPES:
            weights = weights.float()
        if combine:
            out, pair_out = torch.empty_like(x), None
        else:
            out, pair_out = None, torch.empty((tokens * top_k, hidden), device=x.device, dtype=torch.float32)
        if prefill and self._prefill(lib, bank, x, ids, weights, out, pair_out):
            del keep
            return out if combine else pair_out
        nbytes = self._workspace_bytes(lib, tokens, top_k, hidden, bank.intermediate)
        ws = _WORKSPACES.get(x.device, nbytes)
        lib.check(lib.dll.drama_b200_fp8_w8a8_decode(
            ctypes.byref(bank), x.data_ptr(), tokens, top_k, ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype],
            weights.data_ptr(), _lib.DTYPE_CODES[weights.dtype], _lib.ptr(out), _lib.ptr(pair_out),
            _lib.ptr(x_fp8), _lib.ptr(x_scale), ws.data_ptr(), ws.numel(), _lib.stream_handle(x.device)))
        del keep
        return out if combine else pair_out


def fp8_prefill(x: Tensor, ids: Tensor, weights: Tensor, staged, *, validate_ids: bool = True) -> Tensor:
    """Many-token FP8 expert forward on the grouped tensor-core GEMMs.

    Same result contract as ``TorchExpertBackend.forward`` (offload.py:202-213):
    bf16 ``x [T,H]``, local slot ``ids [T,k]``, ``weights [T,k]``; returns bf16
    ``[T,H]`` with route slots summed in slot order in fp32.
    """
    if x.dtype != torch.bfloat16:
        raise ValueError("fp8_prefill runs on bf16 hidden rows")
    hidden = x.shape[-1]
    bank, keep = _fp8_bank(staged, hidden)
    _check_common(x, ids, weights, bank.slots, hidden, validate_ids)
    tokens, top_k = ids.shape
    x = x.contiguous()
    ids = ids.contiguous()
    weights = weights.contiguous()
    if weights.dtype not in FLOAT_DTYPES:
        weights = weights.float()
    out = torch.empty_like(x)
    if tokens == 0:
        return out
    lib = _lib.library()
    nbytes = lib.dll.drama_b200_prefill_workspace_bytes(tokens, top_k, hidden, bank.intermediate, bank.slots)
    ws = _PREFILL_WORKSPACES.get(x.device, nbytes)
    lib.check(lib.dll.drama_b200_fp8_prefill(
        ctypes.byref(bank), x.data_ptr(), tokens, top_k, ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype],
        weights.data_ptr(), _lib.DTYPE_CODES[weights.dtype], out.data_ptr(), ws.data_ptr(), ws.numel(),
        _lib.stream_handle(x.device)))
    del keep
    return out


def fp8_expert_rows(x: Tensor, ids: Tensor, staged) -> Tensor:
    """Per-row bf16 down projections ``[rows, H]`` of ``x [rows, H]`` through expert ``ids[rows]``.

    ``TorchExpertBackend.forward_pairs`` (offload.py:215-244) before the route
    weight, on the swap-AB grouped GEMMs: each row's result is independent of
    the other rows. Rows whose id is outside the bank are left as zeros.
    """
    if x.dtype != torch.bfloat16 or x.ndim != 2:
        raise ValueError("fp8_expert_rows runs on bf16 rows [N, H]")
    hidden = x.shape[-1]
    bank, keep = _fp8_bank(staged, hidden)
    if ids.shape != (x.shape[0],) and ids.shape != (x.shape[0], 1):
        raise ValueError("fp8_expert_rows takes one expert id per row")
    if ids.dtype not in (torch.int32, torch.int64) or ids.device != x.device:
        raise ValueError("Expert IDs must be integer tensors on the rows' device")
    x = x.contiguous()
    ids = ids.reshape(-1).contiguous()
    out = torch.zeros_like(x)
    if x.shape[0] == 0:
        return out
    lib = _lib.library()
    nbytes = lib.dll.drama_b200_expert_rows_workspace_bytes(x.shape[0], hidden, bank.intermediate, bank.slots)
    ws = _PREFILL_WORKSPACES.get(x.device, nbytes)
    lib.check(lib.dll.drama_b200_fp8_expert_rows(
        ctypes.byref(bank), x.data_ptr(), hidden, x.shape[0], ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype],
        out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_handle(x.device)))
    del keep
    return out


QUANTIZED_MODES = {0: "W4A16-GPTQ", 1: "INT8-ConvRot", 2: "W6A8", 3: "W4A8"}


class QuantizedB200Backend(_DecodeBackend):
    """``QuantizedExpertBackend(mode)`` (quantized_kernels.py:217-248) on sm_100a.

    mode 0: GPTQ W4A16, symmetric or with uint4 zero-points (f16 MMAs).
    modes 1-3: INT8-ConvRot, W6A8 and W4A8-codebook banks with ConvRot-rotated
    int8 activations on int8 tensor cores (``drama_b200_w8a8_decode``); bf16
    hidden rows, H and I multiples of 256.
    """

    entry = "drama_b200_int4_decode"

    def __init__(self, mode: int = 0, *, validate_ids: bool = True) -> None:
        if mode not in QUANTIZED_MODES:
            raise ValueError("Unknown quantized bank format")
        super().__init__(validate_ids=validate_ids)
        self.mode = mode
        self.quantized_mode = QUANTIZED_MODES[mode]
        if mode:
            self.entry = "drama_b200_w8a8_decode"

    def _bank(self, staged, hidden):
        return _int4_bank(staged, hidden) if self.mode == 0 else _w8a8_bank(staged, hidden, self.mode)

    def _workspace_bytes(self, lib, tokens, top_k, hidden, intermediate) -> int:
        if self.mode == 0:
            return super()._workspace_bytes(lib, tokens, top_k, hidden, intermediate)
        return lib.dll.drama_b200_w8a8_workspace_bytes(tokens, top_k, hidden, intermediate)

    def _run(self, x: Tensor, ids: Tensor, weights: Tensor, staged, *, combine: bool) -> Tensor:
        if self.mode and x.dtype != torch.bfloat16:
            raise ValueError(f"{self.quantized_mode} experts run on bfloat16 hidden rows")
        return super()._run(x, ids, weights, staged, combine=combine)


def _w8a8_bank(staged, hidden: int, mode: int) -> tuple[_lib.W8a8Bank, tuple]:
    """Bank descriptor for ``QuantizedStore`` modes 1-3 (quantized_model.py:45-68)."""
    w13 = _rows(staged.w13_weight)
    w2 = _rows(staged.w2_weight)
    s13 = _rows(staged.w13_scale_inv)
    s2 = _rows(staged.w2_scale_inv)
    if w13.dtype != torch.int8 or w2.dtype != torch.int8:
        raise ValueError("Quantized weight dtype mismatch")
    scale_dtype = torch.float32 if mode == 1 else torch.uint8
    if s13.dtype != scale_dtype or s2.dtype != scale_dtype:
        raise ValueError("Quantized scale dtype mismatch")
    slots, gate_up = w13.shape[0], w13.shape[1]
    inter = gate_up // 2

    def columns(k):
        return k if mode == 1 else k * 3 // 4 if mode == 2 else k // 2

    def scale_columns(k):
        return 1 if mode == 1 else k // 16 + (8 if mode == 3 else 4)

    if tuple(w13.shape) != (slots, gate_up, columns(hidden)) or tuple(w2.shape) != (slots, hidden, columns(inter)):
        raise ValueError("Quantized weight/scale geometry mismatch")
    if tuple(s13.shape) != (slots, gate_up, scale_columns(hidden)) or \
            tuple(s2.shape) != (slots, hidden, scale_columns(inter)):
        raise ValueError("Quantized weight/scale geometry mismatch")
    align = 16 if mode == 1 else 8
    if w13.stride(1) % align or w13.stride(0) % align or w13.data_ptr() % align:
        w13 = w13.contiguous()
    if w2.stride(1) % align or w2.stride(0) % align or w2.data_ptr() % align:
        w2 = w2.contiguous()
    es = s13.element_size()
    bank = _lib.W8a8Bank(
        mode, w13.data_ptr(), s13.data_ptr(), w2.data_ptr(), s2.data_ptr(),
        w13.stride(0), w13.stride(1), s13.stride(0) * es, s13.stride(1) * es,
        w2.stride(0), w2.stride(1), s2.stride(0) * es, s2.stride(1) * es,
        slots, hidden, inter)
    return bank, (w13, w2, s13, s2)
