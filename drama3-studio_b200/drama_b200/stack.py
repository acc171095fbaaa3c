"""Device-resident decode stack of FP8 MoE layers, captured in CUDA graphs.

One layer is ``drama_b200_fp8_moe_layer``: RMSNorm -> router GEMV -> softmax /
top-k -> FP8 expert GEMVs -> combine + residual, i.e. a layer of
``BackboneDecodeGraph`` (``src/drama_low_vram/backbone_graph.py:306-337``)
without the mixer and the shared expert, with the expert call on the device
instead of ``ExpertOffloadManager``'s host routing. Because no step touches
the host, a whole multi-step decode can be one CUDA graph; this is the
all-experts-resident fast path (``cache_experts == num_experts``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _lib
from .backend import _fp8_bank


@dataclass
class MoELayer:
    """Weights of one layer: FP8 bank (ExpertStore layout), router, RMSNorm."""

    w13_weight: Tensor
    w13_scale_inv: Tensor
    w2_weight: Tensor
    w2_scale_inv: Tensor
    gate: Tensor          # bf16 [E, H]
    gamma: Tensor         # fp32 [H]
    _bank: object = field(default=None, repr=False)

    @property
    def count(self) -> int:
        return self.w13_weight.shape[0]

    def bank(self):
        if self._bank is None:
            self._bank = _fp8_bank(self, self.gate.shape[1])
        return self._bank


@dataclass
class LayerTrace:
    """Optional per-layer outputs for inspection and parity tests."""

    ids: Tensor      # int64 [T, k]
    weights: Tensor  # bf16 [T, k]
    normed: Tensor   # bf16 [T, H]
    moe: Tensor | None = None  # bf16 [T, H] expert output before the residual


def moe_layer_workspace(tokens: int, top_k: int, hidden: int, intermediate: int, experts: int,
                        device) -> Tensor:
    lib = _lib.library()
    nbytes = lib.dll.drama_b200_moe_layer_workspace_bytes(tokens, top_k, hidden, intermediate, experts)
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def torch_router_inputs(hidden_in: Tensor, layer: MoELayer, eps: float) -> tuple[Tensor, Tensor]:
    """The reference decode graph's RMSNorm and router logits, in torch ops.

    ``BackboneDecodeGraph._route_impl`` (``src/drama_low_vram/backbone_graph.py:
    316-319``): the RMSNorm in fp32 math cast to bf16, then ``moe.gate`` as a
    bf16 ``F.linear``. Returns ``(normed, logits)``, both bf16.
    """
    x = hidden_in.float()
    normed = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * layer.gamma).to(torch.bfloat16)
    return normed, F.linear(normed, layer.gate)


def moe_layer(hidden_in: Tensor, layer: MoELayer, out: Tensor, workspace: Tensor, *, top_k: int = 8,
              eps: float = 1e-6, next_gate: Tensor | None = None, trace: LayerTrace | None = None,
              layer_events: tuple | None = None, router: str = "fused") -> Tensor:
    """Enqueue one fused MoE layer on the current stream; returns ``out``.

    One hidden row runs as one launch (thread-block clusters, each streaming a
    run of one routed expert's gate/up and down rows; the last CTA to finish
    combines the slots and adds the residual); more rows run the router,
    expert-group and K1 kernels. ``layer_events=(start, end)`` records CUDA
    events around the layer's launches.

    ``router="fused"`` computes RMSNorm and the router GEMV inside the layer in
    a fixed fp32 order; ``router="torch"`` takes them from torch ops
    (``torch_router_inputs``), so the routes are those of the reference's
    decode graph bit for bit, at the cost of the extra launches.
    """
    if hidden_in.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise ValueError("The fused MoE layer runs on bf16 hidden states")
    if not hidden_in.is_contiguous() or not out.is_contiguous() or hidden_in.shape != out.shape:
        raise ValueError("hidden_in and out must be contiguous and of equal shape")
    if router not in ("fused", "torch"):
        raise ValueError("router must be 'fused' or 'torch'")
    if router == "torch":
        return _moe_layer_torch_router(hidden_in, layer, out, workspace, top_k=top_k, eps=eps, trace=trace,
                                       layer_events=layer_events)
    bank, keep = layer.bank()
    tokens = hidden_in.shape[0]
    lib = _lib.library()
    stream = _lib.stream_handle(hidden_in.device)
    traced = (_lib.ptr(trace.ids if trace else None), _lib.ptr(trace.weights if trace else None),
              _lib.ptr(trace.normed if trace else None))
    moe_out = _lib.ptr(trace.moe if trace else None)
    if layer_events is not None:
        layer_events[0].record()
    lib.check(lib.dll.drama_b200_fp8_moe_layer(
        ctypes.byref(bank), layer.gate.data_ptr(), _lib.ptr(next_gate), layer.gamma.data_ptr(),
        ctypes.c_float(eps), hidden_in.data_ptr(), out.data_ptr(), tokens, top_k, *traced, moe_out,
        workspace.data_ptr(), workspace.numel(), stream))
    if layer_events is not None:
        layer_events[1].record()
    return out


def _moe_layer_torch_router(hidden_in, layer, out, workspace, *, top_k, eps, trace, layer_events):
    if hidden_in.shape[0] != 1:
        raise ValueError("router='torch' runs one decode row per call")
    bank, keep = layer.bank()
    lib = _lib.library()
    stream = _lib.stream_handle(hidden_in.device)
    if layer_events is not None:
        layer_events[0].record()
    normed, logits = torch_router_inputs(hidden_in, layer, eps)
    lib.check(lib.dll.drama_b200_fp8_moe_layer_logits(
        ctypes.byref(bank), normed.data_ptr(), logits.data_ptr(), hidden_in.data_ptr(), out.data_ptr(), 1, top_k,
        _lib.ptr(trace.ids if trace else None), _lib.ptr(trace.weights if trace else None),
        _lib.ptr(trace.moe if trace else None), workspace.data_ptr(), workspace.numel(), stream))
    if layer_events is not None:
        layer_events[1].record()
    if trace is not None:
        trace.normed.copy_(normed)
    return out


class DecodeStack:
    """``layers`` MoE layers applied to ``tokens`` hidden rows per decode step."""

    def __init__(self, layers: list[MoELayer], *, tokens: int = 1, top_k: int = 8, eps: float = 1e-6,
                 router: str = "fused"):
        if not layers:
            raise ValueError("DecodeStack needs at least one layer")
        self.layers = layers
        self.tokens = tokens
        self.top_k = top_k
        self.eps = eps
        self.router = router
        first = layers[0]
        self.device = first.gate.device
        self.experts, self.hidden = first.gate.shape
        self.intermediate = first.w2_weight.shape[2]
        self.workspace = moe_layer_workspace(tokens, top_k, self.hidden, self.intermediate, self.experts,
                                             self.device)
        self._buffers = [torch.empty(tokens, self.hidden, dtype=torch.bfloat16, device=self.device)
                         for _ in range(2)]
        self.graph: torch.cuda.CUDAGraph | None = None

    def step(self, hidden: Tensor, out: Tensor, traces: list[LayerTrace] | None = None,
             layer_events: list[tuple] | None = None) -> Tensor:
        """Enqueue one decode step: ``out = stack(hidden)``."""
        n = len(self.layers)
        src = hidden
        for i, layer in enumerate(self.layers):
            dst = out if i == n - 1 else self._buffers[i % 2]
            nxt = self.layers[i + 1].gate if i + 1 < n else None
            moe_layer(src, layer, dst, self.workspace, top_k=self.top_k, eps=self.eps, next_gate=nxt,
                      trace=None if traces is None else traces[i],
                      layer_events=None if layer_events is None else layer_events[i], router=self.router)
            src = dst
        return out

    def capture(self, inputs: Tensor, outputs: Tensor, *, timed_steps: int = 0) -> torch.cuda.CUDAGraph:
        """One CUDA graph running ``inputs.shape[0]`` consecutive decode steps.

        ``inputs``/``outputs``: bf16 [steps, tokens, hidden]; step s reads
        inputs[s] and writes outputs[s]. Replaying the graph re-runs all steps.
        The first ``timed_steps`` steps record CUDA events around every
        layer's launches (``self.layer_events[step][layer]``).
        """
        steps = inputs.shape[0]
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            self.step(inputs[0], outputs[0])  # eager warm-up (lazy module loading)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        self.layer_events = [[(torch.cuda.Event(enable_timing=True, external=True),
                                torch.cuda.Event(enable_timing=True, external=True))
                               for _ in self.layers] for _ in range(timed_steps)]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for s in range(steps):
                self.step(inputs[s], outputs[s],
                          layer_events=self.layer_events[s] if s < timed_steps else None)
        self.graph = graph
        return graph

    def launches_per_layer(self) -> int:
        """Library kernel launches per layer (torch's RMSNorm and GEMV launches not counted)."""
        lib = _lib.library()
        return lib.dll.drama_b200_moe_layer_launches(self.tokens, self.top_k, self.hidden, self.intermediate,
                                                     self.experts)

    def layer_time_ms(self) -> float:
        """Mean duration of one layer's launches in the last replay."""
        times = [a.elapsed_time(b) for step in self.layer_events for a, b in step]
        return sum(times) / len(times)


def synthetic_stack(layers: int, *, experts: int = 128, hidden: int = 2048, intermediate: int = 768,
                    seed: int = 0, device="cuda") -> list[MoELayer]:
    """Seeded random-init layers with BASELINE's distributions (config 1)."""
    from . import synthetic

    out = []
    for i in range(layers):
        bank = synthetic.fp8_bank(experts, hidden, intermediate, seed * 1000 + i, device=device,
                                  chunk=experts if torch.device(device).type == "cuda" else 1)
        out.append(MoELayer(
            w13_weight=bank["w13_weight"], w13_scale_inv=bank["w13_scale_inv"],
            w2_weight=bank["w2_weight"], w2_scale_inv=bank["w2_scale_inv"],
            gate=synthetic.gate_weight(experts, hidden, seed * 1000 + 500 + i, device=device),
            gamma=synthetic.norm_gamma(hidden, seed * 1000 + 700 + i, device=device)))
    return out
