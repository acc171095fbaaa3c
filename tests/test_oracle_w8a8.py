"""W8A8 modes 1-3 restatement pinned to the reference's own Python code.

``tests/golden/convrot_w8a8.npz`` holds outputs of ``QuantizedExpertBackend``
(src/drama_low_vram/quantized_kernels.py:217-248) run on CPU tensors, the
reference test's weight-grid reconstruction (tests/test_quantized_kernels.py:
47-73) and the reference's quantized activations (make_convrot_golden.py).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from golden.make_convrot_golden import HIDDEN, INTER, bank_sha, inputs
from helpers import assert_parity, np_f32
from oracle import restate as R

GOLDEN = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "convrot_w8a8.npz")


def _case(mode):
    bank, x, ids, w = inputs(mode)
    assert bank_sha(bank) == bytes(GOLDEN[f"sha{mode}"]).decode(), "synthetic generator drifted"
    return {k: v.numpy() for k, v in bank.items()}, np_f32(x), ids.numpy(), np_f32(w)


@pytest.mark.parametrize("mode", [1, 2, 3])
def test_weight_grids_match_the_reference_reconstruction(mode):
    bank, *_ = _case(mode)
    for name, k in (("13", HIDDEN), ("2", INTER)):
        grids = np.stack([R.convrot_grid(bank[f"w{name}_weight"][e], bank[f"w{name}_scale_inv"][e], mode, k)[0]
                          for e in range(bank[f"w{name}_weight"].shape[0])])
        assert hashlib.sha256(grids.tobytes()).hexdigest() == bytes(GOLDEN[f"grid{name}_{mode}"]).decode()


@pytest.mark.parametrize("mode", [1, 2, 3])
def test_rotated_int8_activations_match_the_reference(mode):
    _, x, _, _ = _case(mode)
    q, s = R.quantize_rows_int8(R.convrot_rotate(x))
    assert np.array_equal(R.round_bf16(q.astype(np.float32) * s[:, None]), GOLDEN[f"dq{mode}"])


@pytest.mark.parametrize("mode", [1, 2, 3])
def test_forward_and_pairs_match_the_reference(mode):
    bank, x, ids, w = _case(mode)
    out = R.convrot_forward(x, ids, w, bank, mode)
    assert_parity(out, GOLDEN[f"forward{mode}"], label=f"W8A8 mode {mode} forward")
    assert (out == GOLDEN[f"forward{mode}"]).mean() >= 0.95
    pairs = R.convrot_pairs(np.repeat(x, ids.shape[1], 0), ids.reshape(-1), w.reshape(-1), bank, mode)
    assert_parity(pairs, GOLDEN[f"pairs{mode}"], label=f"W8A8 mode {mode} pairs")


def test_convrot_stages_equal_the_dense_rotation():
    rng = np.random.default_rng(3)
    x = R.round_bf16(rng.standard_normal((5, 768)).astype(np.float32) * 3)
    m = R.H4
    for _ in range(3):
        m = np.kron(m, R.H4)
    dense = (x.reshape(-1, 256).astype(np.float64) @ (m / 16.0)).reshape(x.shape)
    assert np.array_equal(R.convrot_rotate(x), R.round_from_f64(dense, "bfloat16"))


def test_round_from_f64_is_one_rounding():
    v = np.array([1 + 2 ** -8, 1 + 3 * 2 ** -8, 1 + 2 ** -8 + 2 ** -40, -(2 ** -130) * 1.5, 0.0])
    assert R.round_from_f64(v, "bfloat16").tolist() == [1.0, 1 + 2 ** -6, 1 + 2 ** -7, -(2 ** -130) * 1.5, 0.0]
