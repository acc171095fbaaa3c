"""Shared expert + sigmoid gate, fused with the routed combine.

``BackboneDecodeGraph._shared_impl`` and ``_post_impl``
(src/drama_low_vram/backbone_graph.py:327-337) compute, per layer,
``shared = sigmoid(shared_expert_gate(x)) * shared_expert(x)`` with bf16 torch
modules and then ``after_mixer + (expert_output + shared)``. ``SharedExpertB200``
does both in two launches on the sm_100a kernels of ``shared_expert.cu``
(``drama_b200_shared_expert``): the dense bf16 weights are streamed once per
group of up to 8 tokens, and the down projection's epilogue applies the gate,
adds the routed output and the residual, so no intermediate [T, H] tensor is
written. Every rounding point of the bf16 modules is kept.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from . import _lib
from .backend import _Workspace

_SHARED_WORKSPACES = _Workspace()
MAX_TOKENS = 4096  # rows per library call


def _rowmajor(t: Tensor, name: str, shape: tuple[int, int]) -> Tensor:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16; got {t.dtype}")
    if tuple(t.shape) != shape:
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {shape}")
    if t.stride(-1) != 1 or t.stride(0) % 8 or t.data_ptr() % 16:
        t = t.contiguous()
    return t


class SharedExpertB200:
    """One layer's shared expert (gate/up/down projections) and its gate vector, on the GPU.

    ``gate_proj``/``up_proj`` are ``[I, H]``, ``down_proj`` is ``[H, I]`` and
    ``gate_weight`` is the ``[1, H]`` (or ``[H]``) weight of ``shared_expert_gate``,
    all bf16 CUDA tensors (the layouts of ``nn.Linear``).
    """

    def __init__(self, gate_proj: Tensor, up_proj: Tensor, down_proj: Tensor, gate_weight: Tensor) -> None:
        inter, hidden = gate_proj.shape
        if not gate_proj.is_cuda:
            raise RuntimeError("drama_b200 runs on CUDA tensors on an sm_100 GPU")
        self.hidden, self.intermediate = int(hidden), int(inter)
        self.gate_proj = _rowmajor(gate_proj, "gate_proj", (inter, hidden))
        self.up_proj = _rowmajor(up_proj, "up_proj", (inter, hidden))
        self.down_proj = _rowmajor(down_proj, "down_proj", (hidden, inter))
        self.gate_weight = _rowmajor(gate_weight.reshape(1, -1), "gate_weight", (1, hidden)).reshape(-1)
        devices = {t.device for t in (self.gate_proj, self.up_proj, self.down_proj, self.gate_weight)}
        if len(devices) != 1:
            raise ValueError("Shared expert weights must share a device")
        self.device = devices.pop()
        self._desc = _lib.SharedExpert(
            self.gate_proj.data_ptr(), self.up_proj.data_ptr(), self.down_proj.data_ptr(),
            self.gate_weight.data_ptr(), self.gate_proj.stride(0), self.up_proj.stride(0),
            self.down_proj.stride(0), self.hidden, self.intermediate)

    @classmethod
    def from_mlp(cls, mlp) -> "SharedExpertB200":
        """From a sparse-MoE block holding ``shared_expert`` (gate/up/down ``nn.Linear``)
        and ``shared_expert_gate`` (backbone_graph.py:329-330)."""
        se = mlp.shared_expert
        return cls(se.gate_proj.weight, se.up_proj.weight, se.down_proj.weight, mlp.shared_expert_gate.weight)

    def _rows(self, t: Tensor | None, tokens: int, name: str) -> Tensor | None:
        if t is None:
            return None
        t = t.reshape(-1, self.hidden)
        if t.shape[0] != tokens or t.dtype != torch.bfloat16 or t.device != self.device:
            raise ValueError(f"{name} must be bfloat16 [{tokens}, {self.hidden}] on {self.device}")
        return t if t.is_contiguous() and t.data_ptr() % 16 == 0 else t.contiguous()

    def _run(self, flat: Tensor, routed: Tensor | None, residual: Tensor | None, out: Tensor | None) -> Tensor:
        x = self._rows(flat, flat.reshape(-1, self.hidden).shape[0], "hidden rows")
        tokens = x.shape[0]
        routed = self._rows(routed, tokens, "expert output")
        residual = self._rows(residual, tokens, "after_mixer")
        if out is None:
            out = torch.empty_like(x)
        elif out.shape != x.shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise ValueError("out must be a contiguous bfloat16 tensor shaped like the hidden rows")
        if tokens == 0:
            return out
        if tokens > MAX_TOKENS:  # rows are independent: run in chunks
            for a in range(0, tokens, MAX_TOKENS):
                b = min(tokens, a + MAX_TOKENS)
                self._run(x[a:b], None if routed is None else routed[a:b],
                          None if residual is None else residual[a:b], out[a:b])
            return out
        lib = _lib.library()
        nbytes = lib.dll.drama_b200_shared_expert_workspace_bytes(tokens, self.hidden, self.intermediate)
        ws = _SHARED_WORKSPACES.get(self.device, nbytes)
        lib.check(lib.dll.drama_b200_shared_expert(
            ctypes.byref(self._desc), x.data_ptr(), tokens, _lib.ptr(routed), _lib.ptr(residual), out.data_ptr(),
            ws.data_ptr(), ws.numel(), _lib.stream_handle(self.device)))
        return out

    def shared(self, flat: Tensor) -> Tensor:
        """``_shared_impl`` before the reshape: ``sigmoid(gate(x)) * shared_expert(x)``, [T, H] bf16."""
        return self._run(flat, None, None, None)

    def post(self, after_mixer: Tensor, expert_output: Tensor, flat: Tensor, out: Tensor | None = None) -> Tensor:
        """``_post_impl(after_mixer, expert_output, _shared_impl(...))`` in one pass: returns
        ``after_mixer + (expert_output + shared)`` shaped like ``after_mixer``. ``out`` may be
        ``after_mixer`` or ``expert_output`` (in place)."""
        result = self._run(flat, expert_output, after_mixer, None if out is None else out.reshape(-1, self.hidden))
        return result.view_as(after_mixer)
