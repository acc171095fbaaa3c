"""K3 router and route permutation (device side, graph-capturable).

``route_topk`` replaces the routing lines of ``BackboneDecodeGraph._route_impl``
(``src/drama_low_vram/backbone_graph.py:319-323``); ``permute_routes`` replaces
the host-side stable argsort + bincount of
``ExpertOffloadManager._forward_partitioned`` (``src/drama_low_vram/offload.py:
1206-1211``). Both keep the reference's results bit-exact.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib


def route_topk(logits: Tensor, top_k: int, *, renormalize: bool = True,
               out_dtype: torch.dtype | None = None, ids_dtype: torch.dtype = torch.int64,
               ids: Tensor | None = None, weights: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """softmax(logits.float()) -> topk -> renormalise -> cast, on the GPU.

    Returns ``(topk_weights, topk_ids)`` like ``probabilities.topk`` followed by
    the reference's renormalisation and ``.to(out_dtype)`` (default: logits'
    dtype, as ``topk_weights.to(flat.dtype)`` in the reference).
    """
    if logits.ndim != 2:
        raise ValueError("Router logits must have shape [tokens, experts]")
    if not logits.is_cuda:
        raise ValueError("Router logits must be a CUDA tensor")
    tokens, experts = logits.shape
    if not 1 <= top_k <= min(32, experts):
        raise ValueError("top_k must be in [1, min(32, experts)]")
    logits = logits.contiguous()
    out_dtype = out_dtype or logits.dtype
    if ids is None:
        ids = torch.empty((tokens, top_k), device=logits.device, dtype=ids_dtype)
    if weights is None:
        weights = torch.empty((tokens, top_k), device=logits.device, dtype=out_dtype)
    lib = _lib.library()
    lib.check(lib.dll.drama_b200_route_topk(
        logits.data_ptr(), _lib.DTYPE_CODES[logits.dtype], tokens, experts, top_k,
        int(bool(renormalize)), ids.data_ptr(), _lib.DTYPE_CODES[ids.dtype], weights.data_ptr(),
        _lib.DTYPE_CODES[weights.dtype], _lib.stream_handle(logits.device)))
    return weights, ids


def permute_routes(ids: Tensor, num_experts: int, *, status: Tensor | None = None, wide: bool | None = None,
                   position: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """Stable argsort of flat route IDs plus bincount and start offsets (int64).

    ``wide`` picks the many-CTA form (default: from 4096 pairs on), which can
    also fill ``position`` (int64, each pair's sorted position or -1).
    """
    if not ids.is_cuda:
        raise ValueError("Route IDs must be a CUDA tensor")
    if ids.dtype not in (torch.int32, torch.int64):
        raise ValueError("Expert IDs must have an integer dtype")
    flat = ids.reshape(-1).contiguous()
    order = torch.empty(flat.numel(), device=ids.device, dtype=torch.int64)
    counts = torch.empty(num_experts, device=ids.device, dtype=torch.int64)
    offsets = torch.empty(num_experts + 1, device=ids.device, dtype=torch.int64)
    lib = _lib.library()
    if wide is None:
        wide = flat.numel() > 4096 or position is not None
    if wide:
        nbytes = lib.dll.drama_b200_permute_routes_wide_scratch_bytes(flat.numel(), num_experts)
        scratch = torch.empty(max(nbytes, 16), device=ids.device, dtype=torch.uint8)
        lib.check(lib.dll.drama_b200_permute_routes_wide(
            flat.data_ptr(), _lib.DTYPE_CODES[flat.dtype], flat.numel(), num_experts, order.data_ptr(),
            counts.data_ptr(), offsets.data_ptr(), _lib.ptr(position), scratch.data_ptr(), scratch.numel(),
            _lib.ptr(status), _lib.stream_handle(ids.device)))
        return order, counts, offsets
    lib.check(lib.dll.drama_b200_permute_routes(
        flat.data_ptr(), _lib.DTYPE_CODES[flat.dtype], flat.numel(), num_experts,
        order.data_ptr(), counts.data_ptr(), offsets.data_ptr(), _lib.ptr(status),
        _lib.stream_handle(ids.device)))
    return order, counts, offsets
