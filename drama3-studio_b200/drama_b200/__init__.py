"""B200-native (sm_100a) routed-expert hot path for Drama3-Studio's drama_low_vram.

Drop-in expert backends behind the reference's ``ExpertBackend`` /
``install_expert_offload`` API, a resident-bank manager whose expert calls can
be captured in CUDA graphs, the device router, and the measurement stack.
Compute runs only in ``lib/libdrama_b200.so`` (hand-written CUDA for sm_100a,
C ABI in ``include/drama_b200.h``); there is no CPU fallback.
"""

from .backend import B200ExpertBackend, Fp8W8a8B200Backend, QuantizedB200Backend, QuantizedBank  # noqa: F401
from .resident import ResidentExpertManager, install_resident_experts  # noqa: F401
from .router import permute_routes, route_topk  # noqa: F401

__all__ = [
    "B200ExpertBackend",
    "Fp8W8a8B200Backend",
    "QuantizedB200Backend",
    "QuantizedBank",
    "ResidentExpertManager",
    "install_resident_experts",
    "permute_routes",
    "route_topk",
]
