"""Test helpers: torch <-> oracle (numpy) conversion and the parity bar."""

from __future__ import annotations

import numpy as np
import torch

# north_star: "layer outputs agree within max-abs/relative error <= 2e-2 in
# bf16 (fp32 accumulation)". Both bounds are asserted.
MAX_ABS_TOL = 2e-2
REL_TOL = 2e-2


def np_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def np_bank(bank: dict) -> dict:
    out = {}
    for key, value in bank.items():
        if value is None:
            out[key] = None
        elif value.dtype == torch.float8_e4m3fn:
            out[key] = value.detach().cpu().view(torch.uint8).numpy()
        elif value.dtype in (torch.bfloat16, torch.float16):
            out[key] = value.detach().float().cpu().numpy()
        else:
            out[key] = value.detach().cpu().numpy()
    return out


def to_device(bank: dict, device) -> dict:
    return {k: (None if v is None else v.to(device)) for k, v in bank.items()}


def errors(actual: np.ndarray, expected: np.ndarray) -> tuple[float, float]:
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    max_abs = float(np.abs(actual - expected).max()) if actual.size else 0.0
    denom = float(np.linalg.norm(expected)) or 1.0
    return max_abs, float(np.linalg.norm(actual - expected)) / denom


def assert_parity(actual, expected, *, max_abs=MAX_ABS_TOL, rel=REL_TOL, label=""):
    a, r = errors(actual, expected)
    assert a <= max_abs and r <= rel, f"{label}: max_abs {a:.3e} (tol {max_abs}), rel {r:.3e} (tol {rel})"
    return a, r
