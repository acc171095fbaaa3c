"""Resident-bank expert path: every routed expert in HBM, routing on the device.

The reference's ``ExpertOffloadManager.forward`` (src/drama_low_vram/offload.py:
1016-1063) copies the router's ids to the host on every call, ranks and stages
experts there, and refuses to run inside CUDA graph capture (offload.py:1021-
1022). ``BackboneDecodeGraph`` therefore replays a pre-expert graph, calls the
expert module eagerly and replays a post-expert graph for every layer
(src/drama_low_vram/backbone_graph.py:547-556).

When all of a layer's experts fit in HBM (the manager's ``cache_experts == E``
case: 48 x 604 MB = 29 GB for the Drama 3 FP8 stack, a sixth of one B200) the
host round trip has nothing left to decide. ``ResidentExpertManager`` keeps the
manager's attach / forward / close contract and argument errors
(offload.py:996-1063, 1456-1476), holds each module's bank in HBM, and passes
the router's global ids straight to the sm_100a kernels. Its forward enqueues
work on the current stream and never waits for the host, so it can be captured:
a layer's pre-expert graph, the expert call and the post-expert graph become
one graph.

Id range checks: outside capture (and with ``validate_ids``) an id outside
``[0, E)`` raises the reference's ``ValueError`` after one device-to-host read
of a flag. Inside capture no host read is possible; the kernels then give such
pairs zero weight, as the reference's dense path does for ids it never routes.
"""

from __future__ import annotations

import threading
import types
from contextlib import nullcontext
from dataclasses import asdict, dataclass

import torch
from torch import Tensor, nn

from . import _lib
from .backend import (FLOAT_DTYPES, FP8_DTYPE, MAX_DECODE_PAIRS, _PREFILL_WORKSPACES, _WORKSPACES,
                      B200ExpertBackend, QuantizedB200Backend)
from .staging import host_locked

EXPERT_BUFFER_NAMES = ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv")
FP8_BLOCK = 128
_ORIGINAL = "_drama_offload_original_forward"  # same marker as the reference manager (offload.py:1005)


@dataclass
class ResidentStats:
    """Counters in the spirit of ``OffloadStats`` (offload.py:62-97)."""

    forward_calls: int = 0
    captured_calls: int = 0       # calls recorded into a CUDA graph (their replays are not counted)
    validated_calls: int = 0      # eager calls whose ids were range-checked
    resident_layers: int = 0
    resident_bytes: int = 0       # bank bytes held in HBM
    cpu_expert_bytes: int = 0     # bytes of the attached host banks

    def as_dict(self) -> dict[str, int]:
        return asdict(self)


def expert_modules(backbone: nn.Module) -> list[tuple[str, nn.Module]]:
    """Routed expert modules: those holding both stacked banks (offload.py:1479-1484)."""
    return [(name, module) for name, module in backbone.named_modules()
            if hasattr(module, "w13_weight") and hasattr(module, "w2_weight")]


def _fp8_store(module: nn.Module) -> dict[str, Tensor]:
    """The four FP8 bank tensors after the checks of ``ExpertStore.validate`` (offload.py:139-170)."""
    if not getattr(module, "fp8", False):
        raise ValueError("Expert offload requires FP8 buffers, not dense BF16 weights")
    store = {name: getattr(module, name) for name in EXPERT_BUFFER_NAMES}
    for name, t in store.items():
        if t.device.type != "cpu":
            raise ValueError(f"{name} must stay in CPU memory; got {t.device}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        want = FP8_DTYPE if name.endswith("_weight") else torch.float32
        if t.dtype != want:
            raise ValueError(f"{name} must be {want}; got {t.dtype}")
        if t.ndim != 3:
            raise ValueError(f"{name} must be a stacked three-dimensional tensor")
    experts, gate_up, hidden = store["w13_weight"].shape
    if experts < 1 or gate_up % 2:
        raise ValueError("Expert bank needs at least one expert and even gate/up rows")
    inter = gate_up // 2
    if hidden % FP8_BLOCK or inter % FP8_BLOCK:
        raise ValueError("Expert dimensions must be divisible by the FP8 block size")
    shapes = {
        "w2_weight": (experts, hidden, inter),
        "w13_scale_inv": (experts, gate_up // FP8_BLOCK, hidden // FP8_BLOCK),
        "w2_scale_inv": (experts, hidden // FP8_BLOCK, inter // FP8_BLOCK),
    }
    for name, shape in shapes.items():
        if tuple(store[name].shape) != shape:
            raise ValueError(f"{name} has shape {tuple(store[name].shape)}, expected {shape}")
    return store


def _quantized_store(store) -> dict[str, Tensor]:
    """A ``QuantizedStore`` bank (modes 0-3, quantized_model.py:27-75)."""
    if getattr(store, "mode", None) not in (0, 1, 2, 3):
        raise ValueError("Unknown quantized bank format")
    if hasattr(store, "validate"):
        store.validate()
    out = {name: getattr(store, name) for name in EXPERT_BUFFER_NAMES}
    for name in ("w13_qzeros", "w2_qzeros"):
        if getattr(store, name, None) is not None:
            out[name] = getattr(store, name)
    for name, t in out.items():
        if t.device.type != "cpu" or t.ndim != 3 or not t.is_contiguous():
            raise ValueError(f"Quantized bank must be contiguous three-dimensional CPU storage: {name}")
    return out


def _module_store(module: nn.Module) -> tuple[str, dict[str, Tensor]]:
    quantized = getattr(module, "_drama_quant_store", None)
    if quantized is not None:
        return f"q{quantized.mode}", _quantized_store(quantized)
    return "fp8", _fp8_store(module)


class _ResidentBank:
    """One module's bank in HBM, with the attribute names the backends read."""

    def __init__(self, kind: str, tensors: dict[str, Tensor], device: torch.device, stream) -> None:
        self.kind = kind
        self.nbytes = 0
        with torch.cuda.stream(stream):
            for name, t in tensors.items():
                src = t if host_locked(t) else t.pin_memory()
                dev = torch.empty(t.shape, dtype=t.dtype, device=device)
                dev.copy_(src, non_blocking=True)
                setattr(self, name, dev)
                self.nbytes += dev.numel() * dev.element_size()
        for name in ("w13_qzeros", "w2_qzeros"):
            if not hasattr(self, name):
                setattr(self, name, None)
        self.num_experts = self.w13_weight.shape[0]
        self.intermediate = self.w13_weight.shape[1] // 2
        self.hidden = self.w2_weight.shape[1]


class ResidentExpertManager:
    """``ExpertOffloadManager`` for banks that stay in HBM; capturable forward.

    ``backend`` defaults to ``B200ExpertBackend`` for FP8 modules and
    ``QuantizedB200Backend(mode)`` for quantized modules (modes 0-3). Banks are copied to
    ``device`` once, at attach time, on a side stream that the caller's current
    stream then waits on.
    """

    def __init__(self, *, backend=None, device: torch.device | str | int | None = None,
                 validate_ids: bool = True) -> None:
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("The resident expert path runs on CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.validate_ids = validate_ids
        self._backend = backend
        self._fp8 = B200ExpertBackend(validate_ids=False)
        self._quantized = {mode: QuantizedB200Backend(mode, validate_ids=False) for mode in range(4)}
        self.modules: dict[str, nn.Module] = {}
        self._banks: dict[int, _ResidentBank] = {}
        self._names: dict[int, str] = {}
        self._lock = threading.Lock()
        self._closed = False
        self.stats = ResidentStats()

    # -- attach / detach ---------------------------------------------------
    def attach(self, name: str, module: nn.Module) -> None:
        if self._closed:
            raise RuntimeError("This expert offload manager has been closed")
        if hasattr(module, _ORIGINAL) or name in self.modules:
            raise ValueError(f"Expert module {name!r} already has an offload manager")
        kind, tensors = _module_store(module)
        copy_stream = torch.cuda.Stream(self.device)
        bank = _ResidentBank(kind, tensors, self.device, copy_stream)
        torch.cuda.current_stream(self.device).wait_stream(copy_stream)
        self.stats.cpu_expert_bytes += sum(t.numel() * t.element_size() for t in tensors.values())
        self.stats.resident_bytes += bank.nbytes
        self.stats.resident_layers += 1
        manager = self
        setattr(module, _ORIGINAL, module.forward)

        def forward(experts: nn.Module, x: Tensor, topk_ids: Tensor, topk_weights: Tensor) -> Tensor:
            return manager.forward(experts, x, topk_ids, topk_weights)

        module.forward = types.MethodType(forward, module)
        self.modules[name] = module
        self._banks[id(module)] = bank
        self._names[id(module)] = name

    def close(self) -> None:
        """Restore every module's forward and release the HBM banks (offload.py:1456-1476)."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        for module in self.modules.values():
            if hasattr(module, _ORIGINAL):
                module.forward = getattr(module, _ORIGINAL)
                delattr(module, _ORIGINAL)
        self.modules.clear()
        self._banks.clear()
        self._names.clear()
        self._closed = True

    def bank(self, module: nn.Module) -> _ResidentBank:
        """The HBM bank serving ``module`` (attribute names of ``ExpertStore``)."""
        try:
            return self._banks[id(module)]
        except KeyError:
            raise ValueError("Module is not attached to this manager") from None

    def _backend_for(self, bank: _ResidentBank):
        if self._backend is not None:
            return self._backend
        return self._fp8 if bank.kind == "fp8" else self._quantized[int(bank.kind[1:])]

    # -- forward -----------------------------------------------------------
    @torch.no_grad()
    def forward(self, module: nn.Module, x: Tensor, topk_ids: Tensor, topk_weights: Tensor) -> Tensor:
        if self._closed:
            raise RuntimeError("This expert offload manager has been closed")
        bank = self.bank(module)
        if x.ndim != 2 or x.shape[-1] != bank.hidden:
            raise ValueError(f"Expected hidden rows [N, {bank.hidden}], got {tuple(x.shape)}")
        if topk_ids.ndim != 2 or topk_ids.shape[0] != x.shape[0]:
            raise ValueError("Expert IDs must have shape [tokens, top_k]")
        if topk_weights.shape != topk_ids.shape or topk_ids.shape[1] < 1:
            raise ValueError("Routing weights must match IDs and top_k must be positive")
        if topk_ids.dtype not in (torch.int32, torch.int64):
            raise ValueError("Expert IDs must have an integer dtype")
        if topk_ids.device != x.device or topk_weights.device != x.device:
            raise ValueError("Hidden states, expert IDs and routing weights must share a device")
        if x.dtype not in FLOAT_DTYPES:
            raise ValueError("Expert compute dtype must be float16, bfloat16 or float32")
        if not topk_weights.is_floating_point():
            raise ValueError("Routing weights must be floating point")
        if x.device != self.device:
            raise ValueError(f"Hidden states are on {x.device}; the resident banks are on {self.device}")
        capturing = torch.cuda.is_current_stream_capturing()
        with self._lock:
            self.stats.forward_calls += 1
            self.stats.captured_calls += int(capturing)
        if x.shape[0] == 0:
            return torch.zeros_like(x)
        if self.validate_ids and not capturing:
            bad = (topk_ids < 0) | (topk_ids >= bank.num_experts)
            if bool(bad.any()):
                raise ValueError(f"Expert IDs must be in [0, {bank.num_experts})")
            with self._lock:
                self.stats.validated_calls += 1
        return self._backend_for(bank).forward(x, topk_ids, topk_weights, bank)

    # -- capture support -----------------------------------------------------
    def reserve(self, tokens: int, top_k: int, *, stream: torch.cuda.Stream | None = None) -> None:
        """Size the kernels' scratch for calls of up to ``tokens`` rows on ``stream``.

        Scratch is kept per (device, stream) and cannot grow inside capture, so
        call this for the capture stream before ``torch.cuda.graph``.
        """
        lib = _lib.library()
        ctx = torch.cuda.stream(stream) if stream is not None else nullcontext()
        rows = max(1, min(tokens, MAX_DECODE_PAIRS // max(1, top_k)))
        with ctx:
            for bank in self._banks.values():
                nbytes = self._backend_for(bank)._workspace_bytes(lib, rows, top_k, bank.hidden, bank.intermediate)
                _WORKSPACES.get(self.device, nbytes)
                if bank.kind == "fp8":
                    nbytes = lib.dll.drama_b200_prefill_workspace_bytes(tokens, top_k, bank.hidden,
                                                                        bank.intermediate, bank.num_experts)
                    _PREFILL_WORKSPACES.get(self.device, nbytes)


def install_resident_experts(backbone: nn.Module, *, backend=None,
                             device: torch.device | str | int | None = None,
                             validate_ids: bool = True) -> ResidentExpertManager:
    """Resident counterpart of ``install_expert_offload`` (offload.py:1534-1569).

    Replaces only the routed expert modules' forwards; checkpoint keys, the
    router and shared experts stay as they are. Every store is validated before
    any module changes.
    """
    experts = expert_modules(backbone)
    if not experts:
        raise ValueError("Backbone contains no routed expert modules")
    for _, module in experts:
        _module_store(module)
        if hasattr(module, _ORIGINAL):
            raise ValueError("Backbone already has an expert offload manager")
    manager = ResidentExpertManager(backend=backend, device=device, validate_ids=validate_ids)
    for name, module in experts:
        manager.attach(name, module)
    return manager
