"""Pin the CPU oracle (oracle/restate.py) to the reference.

Golden vectors in tests/golden/ come from the reference's own Python code
(tests/golden/make_golden.py) and from the reference's router ops on a B200
(tests/golden/make_router_golden.py); the native C++ core is the reference's
own source built by oracle/Makefile.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from drama_b200 import synthetic
from helpers import np_bank
from oracle import restate as R

GOLDEN = Path(__file__).resolve().parent / "golden"
DT = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _cases(npz):
    return sorted({k.split("/")[0] for k in npz.files if "/" in k})


def _digest(t: torch.Tensor) -> str:
    a = t.detach().cpu().contiguous()
    if a.dtype == torch.float8_e4m3fn:
        a = a.view(torch.uint8)
    elif a.dtype == torch.bfloat16:
        a = a.view(torch.int16)
    return hashlib.sha256(a.numpy().tobytes()).hexdigest()


def _decode_bits(bits: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return R.from_bf16_bits(bits)
    if dtype == "float16":
        return bits.view(np.float16).astype(np.float32)
    return bits


@pytest.fixture(scope="module")
def native():
    from oracle.ref_native import LIB_PATH, ReferenceNative

    if not LIB_PATH.is_file():
        pytest.skip("reference native core not built (make -C oracle)")
    return ReferenceNative()


def test_fp8_table_matches_torch_e4m3fn():
    raw = torch.arange(256, dtype=torch.int64).to(torch.uint8)
    expected = raw.view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(R.FP8_TABLE, expected)


def test_fp8_table_matches_reference_native(native):
    raw = np.arange(256, dtype=np.uint8)
    np.testing.assert_array_equal(R.decode_fp8(raw), native.decode(raw))
    assert np.signbit(R.decode_fp8(np.uint8(128)))


@pytest.mark.parametrize("kind", ["random", "zero", "tiny", "saturated"])
def test_activation_quantisation_exact_bytes(native, kind):
    # Restates tests/test_native_backend.py:41-56 against the restatement.
    x = torch.randn(16, 128, generator=torch.Generator().manual_seed(22))
    if kind == "zero":
        x.zero_()
    elif kind == "tiny":
        x *= 1e-20
    elif kind == "saturated":
        x *= 1e20
    bits = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    q_ref, s_ref = native.quantize(bits.reshape(-1))
    q, s = R.quantize_fp8_activations(R.from_bf16_bits(bits).reshape(-1))
    np.testing.assert_array_equal(q.reshape(-1), q_ref)
    np.testing.assert_array_equal(s, s_ref)


def test_bf16_rounding_matches_torch():
    x = torch.randn(4096, generator=torch.Generator().manual_seed(3)) * 1e3
    x[:4] = torch.tensor([float("inf"), -0.0, 1e-40, 65504.0])
    ours = R.round_bf16(x.numpy())
    np.testing.assert_array_equal(ours, x.to(torch.bfloat16).float().numpy())


def test_fp8_dequant_path_matches_reference_goldens():
    g = np.load(GOLDEN / "fp8_dequant.npz")
    for name in _cases(g):
        hidden, inter, experts, tokens, top_k, seed = (int(v) for v in g[f"{name}/params"])
        dtype = str(g[f"{name}/dtype"])
        bank = synthetic.fp8_bank(experts, hidden, inter, seed)
        x = synthetic.hidden_states(tokens, hidden, seed + 500, dtype=DT[dtype])
        for key, t in bank.items():
            assert _digest(t) == str(g[f"{name}/sha_{key}"]), f"generator drift in {name}/{key}"
        assert _digest(x) == str(g[f"{name}/sha_x"])
        ids, w = g[f"{name}/ids"], g[f"{name}/weights"]
        xs = x.float().numpy()
        pairs = R.fp8_dequant_pairs(np.repeat(xs, top_k, 0), ids.reshape(-1), w.reshape(-1),
                                    np_bank(bank), dtype)
        ref = g[f"{name}/pairs"]
        assert np.abs(pairs - ref).max() <= 1e-3, name
        assert np.linalg.norm(pairs - ref) <= 1e-3 * np.linalg.norm(ref), name
        y = R.combine_slots(pairs, tokens, top_k, dtype)
        y_ref = _decode_bits(g[f"{name}/forward"], dtype)
        assert np.abs(y - y_ref).max() <= 1e-3, name


def test_int4_symmetric_matches_reference_goldens():
    g = np.load(GOLDEN / "int4_sym.npz")
    for name in _cases(g):
        hidden, inter, experts, tokens, top_k, seed = (int(v) for v in g[f"{name}/params"])
        bank = synthetic.int4_bank(experts, hidden, inter, seed, asymmetric=False,
                                   scale_dtype=torch.float16)
        for key in ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv"):
            assert _digest(bank[key]) == str(g[f"{name}/sha_{key}"]), f"generator drift {name}/{key}"
        x = synthetic.hidden_states(tokens, hidden, seed + 500)
        y = R.int4_forward(x.float().numpy(), g[f"{name}/ids"], g[f"{name}/weights"], np_bank(bank))
        y_ref = R.from_bf16_bits(g[f"{name}/forward"])
        assert np.abs(y - y_ref).max() <= 1e-3, name


def test_int4_zero_point_8_equals_implicit():
    bank = synthetic.int4_bank(2, 256, 128, 5, asymmetric=False, scale_dtype=torch.bfloat16)
    nb = np_bank(bank)
    rows = nb["w13_weight"].shape[1]
    explicit = dict(nb)
    explicit["w13_qzeros"] = np.stack([R.pack_zeros(np.full((rows, 2), 8))] * 2)
    explicit["w2_qzeros"] = np.stack([R.pack_zeros(np.full((256, 1), 8))] * 2)
    x = synthetic.hidden_states(1, 256, 9).float().numpy()
    ids, w = np.array([[1, 0]]), np.array([[0.6, 0.4]], dtype=np.float32)
    np.testing.assert_array_equal(R.int4_forward(x, ids, w, nb), R.int4_forward(x, ids, w, explicit))


def test_int4_pack_roundtrip():
    rng = np.random.default_rng(1)
    codes = rng.integers(0, 16, size=(3, 16, 256))
    np.testing.assert_array_equal(R.unpack_int4(R.pack_int4(codes), 256), codes)
    zeros = rng.integers(0, 16, size=(16, 6))
    np.testing.assert_array_equal(R.unpack_zeros(R.pack_zeros(zeros), 16), zeros)
    torch_words = synthetic.pack_int4_rows(torch.from_numpy(codes))
    np.testing.assert_array_equal(torch_words.numpy(), R.pack_int4(codes))
    torch_zeros = synthetic.pack_int4_zeros(torch.from_numpy(zeros))
    np.testing.assert_array_equal(torch_zeros.numpy(), R.pack_zeros(zeros))


def test_w8a8_matches_reference_python_goldens():
    g = np.load(GOLDEN / "w8a8.npz")
    for name in _cases(g):
        hidden, inter, experts, jobs, seed = (int(v) for v in g[f"{name}/params"])
        bank = np_bank(synthetic.fp8_bank(experts, hidden, inter, seed))
        x = synthetic.hidden_states(1, hidden, seed + 500).float().numpy()[0]
        pairs = R.w8a8_pairs(x, g[f"{name}/ids"], g[f"{name}/weights"], bank)
        np.testing.assert_allclose(pairs, g[f"{name}/pairs"], rtol=1e-5, atol=2e-6)


def test_w8a8_matches_reference_native_executor(native):
    bank = synthetic.fp8_bank(4, 256, 128, 77)
    nb = np_bank(bank)
    x = synthetic.hidden_states(1, 256, 78)
    ids = np.array([3, 1, 3, 0])
    w = np.array([0.4, 0.2, 0.3, 0.1], dtype=np.float32)
    bits = x.view(torch.int16).numpy().view(np.uint16)[0]
    with native.executor(256, 128, capacity=8, threads=1) as ex:
        ref = ex.forward(nb, bits, ids, w)
    ours = R.w8a8_pairs(x.float().numpy()[0], ids, w, nb)
    np.testing.assert_allclose(ours, ref, rtol=1e-5, atol=2e-6)


def test_permutation_matches_reference_goldens():
    g = np.load(GOLDEN / "permute.npz")
    for name in _cases(g):
        order, counts, offsets = R.permute_routes(g[f"{name}/ids"], int(g[f"{name}/experts"]))
        np.testing.assert_array_equal(order, g[f"{name}/order"])
        np.testing.assert_array_equal(counts, g[f"{name}/counts"])
        assert offsets[-1] == g[f"{name}/ids"].size


def test_router_oracle_selects_top_values():
    rng = np.random.default_rng(7)
    logits = R.round_bf16(rng.normal(0, 0.9, size=(64, 128)).astype(np.float32))
    ids, w, probs = R.route_topk(logits, 8, True, "float32")
    for r in range(64):
        chosen = probs[r, ids[r]]
        assert np.all(np.diff(chosen) <= 0)  # descending
        assert chosen.min() >= np.sort(probs[r])[-8]
        assert len(set(ids[r].tolist())) == 8
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)


def test_router_oracle_matches_cuda_goldens():
    path = GOLDEN / "router_cuda.npz"
    if not path.is_file():
        pytest.skip("router CUDA goldens not generated yet (tests/golden/make_router_golden.py)")
    g = np.load(path)
    for name in _cases(g):
        logits = R.from_bf16_bits(g[f"{name}/logits_bits"])
        top_k = int(g[f"{name}/top_k"])
        ids, w, probs = R.route_topk(logits, top_k, bool(g[f"{name}/renorm"]), "bfloat16")
        np.testing.assert_array_equal(ids, g[f"{name}/ids"], err_msg=name)
        # numpy's exp may differ from CUDA's expf in the last fp32 bit, which
        # can move a renormalised weight by one bf16 step.
        diff = np.abs(R.bf16_bits(w).astype(np.int32) - g[f"{name}/weights_bits"].astype(np.int32))
        assert diff.max() <= 1, name
