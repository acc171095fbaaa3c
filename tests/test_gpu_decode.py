"""K1 decode kernels on the B200 against the oracle and the reference goldens.

Bar (north_star): max-abs and relative-L2 error <= 2e-2 against the
reference's PyTorch dequant path, per quant format.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import assert_parity, np_bank, np_f32, to_device
from oracle import restate as R

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DT = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
DTN = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}


class Staged:
    def __init__(self, bank: dict):
        for k, v in bank.items():
            setattr(self, k, v)

    @property
    def count(self):
        return self.w13_weight.shape[0]


def _routes(tokens, top_k, experts, seed, dup=False):
    from drama_b200 import synthetic

    if dup:
        ids = torch.tensor([[3, 1, 3, 0, 2, 7, 1, 5][:top_k]] * tokens)
        w = torch.softmax(torch.randn(tokens, top_k, generator=torch.Generator().manual_seed(seed)), -1)
        return ids, w
    return synthetic.uniform_routes(tokens, top_k, experts, seed)


@pytest.mark.parametrize("hidden,inter,experts,tokens,top_k,dtype,dup", [
    (256, 128, 4, 1, 4, torch.bfloat16, False),
    (256, 256, 8, 1, 8, torch.bfloat16, True),
    (256, 128, 4, 3, 3, torch.float16, False),
    (256, 128, 4, 2, 3, torch.float32, False),
    (2048, 768, 8, 1, 8, torch.bfloat16, False),
    (2048, 768, 16, 4, 8, torch.bfloat16, False),
    (2048, 768, 32, 16, 8, torch.bfloat16, False),
    (1024, 512, 4, 20, 4, torch.bfloat16, False),
])
def test_fp8_decode_forward_matches_dequant_oracle(cuda_device, hidden, inter, experts, tokens, top_k, dtype, dup):
    from drama_b200 import B200ExpertBackend, synthetic

    bank = synthetic.fp8_bank(experts, hidden, inter, 100 + tokens)
    x = synthetic.hidden_states(tokens, hidden, 200 + tokens, dtype=dtype)
    ids, w = _routes(tokens, top_k, experts, 300 + tokens, dup)
    w = w.to(dtype)
    backend = B200ExpertBackend()
    staged = Staged(to_device(bank, cuda_device))
    y = backend.forward(x.to(cuda_device), ids.to(cuda_device), w.to(cuda_device), staged)
    assert y.dtype == dtype and y.shape == x.shape
    expected = R.fp8_dequant_forward(np_f32(x), ids.numpy(), np_f32(w), np_bank(bank), DTN[dtype])
    assert_parity(np_f32(y), expected, label=f"fp8 forward {hidden}x{inter} T={tokens}")
    # repeat: workspace counters must be left clean and results deterministic
    y2 = backend.forward(x.to(cuda_device), ids.to(cuda_device), w.to(cuda_device), staged)
    assert torch.equal(y.view(torch.uint8) if y.dtype != torch.float32 else y, y2.view(torch.uint8) if y.dtype != torch.float32 else y2)


@pytest.mark.parametrize("pairs", [1, 7, 8, 33])
def test_fp8_forward_pairs_fp32_partials(cuda_device, pairs):
    from drama_b200 import B200ExpertBackend, synthetic

    hidden, inter, experts = 512, 256, 6
    bank = synthetic.fp8_bank(experts, hidden, inter, 7)
    x = synthetic.hidden_states(pairs, hidden, 8)
    ids = torch.randint(0, experts, (pairs, 1), generator=torch.Generator().manual_seed(pairs))
    w = torch.rand(pairs, 1, generator=torch.Generator().manual_seed(pairs + 1)).to(torch.bfloat16)
    out = B200ExpertBackend().forward_pairs(x.to(cuda_device), ids.to(cuda_device), w.to(cuda_device),
                                            Staged(to_device(bank, cuda_device)))
    assert out.dtype == torch.float32 and out.shape == (pairs, hidden)
    expected = R.fp8_dequant_pairs(np_f32(x), ids.numpy(), np_f32(w), np_bank(bank), "bfloat16")
    assert_parity(out.cpu().numpy(), expected, label="forward_pairs")


def test_fp8_decode_matches_reference_goldens(cuda_device):
    from drama_b200 import B200ExpertBackend, synthetic

    g = np.load(GOLDEN / "fp8_dequant.npz")
    backend = B200ExpertBackend()
    for name in sorted({k.split("/")[0] for k in g.files}):
        hidden, inter, experts, tokens, top_k, seed = (int(v) for v in g[f"{name}/params"])
        dtype = str(g[f"{name}/dtype"])
        bank = to_device(synthetic.fp8_bank(experts, hidden, inter, seed), cuda_device)
        x = synthetic.hidden_states(tokens, hidden, seed + 500, dtype=DT[dtype]).to(cuda_device)
        ids = torch.from_numpy(g[f"{name}/ids"]).to(cuda_device)
        w = torch.from_numpy(g[f"{name}/weights"]).to(DT[dtype]).to(cuda_device)
        y = backend.forward(x, ids, w, Staged(bank))
        bits = g[f"{name}/forward"]
        ref = R.from_bf16_bits(bits) if dtype == "bfloat16" else (
            bits.view(np.float16).astype(np.float32) if dtype == "float16" else bits)
        assert_parity(np_f32(y), ref, label=f"golden {name}")
        pairs = backend.forward_pairs(x.repeat_interleave(top_k, 0), ids.reshape(-1, 1), w.reshape(-1, 1), Staged(bank))
        assert_parity(pairs.cpu().numpy(), g[f"{name}/pairs"], label=f"golden pairs {name}")


def test_fp8_decode_packed_arena_strided_views(cuda_device):
    """Role views of one packed uint8 arena (offload.py:396-421) have expert
    strides larger than the role size; the kernels read them in place."""
    from drama_b200 import B200ExpertBackend, synthetic

    hidden, inter, experts = 256, 128, 4
    bank = synthetic.fp8_bank(experts, hidden, inter, 41)
    names = ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv")
    role = {n: bank[n][0].numel() * bank[n].element_size() for n in names}
    arena = torch.empty((experts, sum(role.values())), dtype=torch.uint8, device=cuda_device)
    views, offset = {}, 0
    for n in names:
        src = bank[n].to(cuda_device)
        v = arena.narrow(1, offset, role[n]).view(src.dtype).view(experts, *src.shape[1:])
        v.copy_(src)
        views[n] = v
        offset += role[n]
    x = synthetic.hidden_states(1, hidden, 42).to(cuda_device)
    ids = torch.tensor([[2, 0, 3]], device=cuda_device)
    w = torch.tensor([[0.5, 0.3, 0.2]], device=cuda_device).to(torch.bfloat16)
    y = B200ExpertBackend().forward(x, ids, w, Staged(views))
    expected = R.fp8_dequant_forward(np_f32(x), ids.cpu().numpy(), np_f32(w), np_bank(bank))
    assert_parity(np_f32(y), expected, label="packed arena")


def test_invalid_slot_raises_like_reference(cuda_device):
    from drama_b200 import B200ExpertBackend, synthetic

    bank = to_device(synthetic.fp8_bank(2, 256, 128, 1), cuda_device)
    x = synthetic.hidden_states(1, 256, 2).to(cuda_device)
    with pytest.raises(ValueError, match="outside the staging pool"):
        B200ExpertBackend().forward(x, torch.tensor([[0, 5]], device=cuda_device),
                                    torch.ones(1, 2, device=cuda_device), Staged(bank))


@pytest.mark.parametrize("tokens", [1, 4, 16])
@pytest.mark.parametrize("asym", [True, False])
def test_int4_decode_matches_oracle(cuda_device, tokens, asym):
    from drama_b200 import QuantizedB200Backend, QuantizedBank, synthetic

    hidden, inter, experts = 2048, 768, 32
    bank = synthetic.int4_bank(experts, hidden, inter, 60 + tokens, asymmetric=asym)
    x = synthetic.hidden_states(tokens, hidden, 61 + tokens)
    ids, w = synthetic.uniform_routes(tokens, 8, experts, 62 + tokens)
    w = w.to(torch.bfloat16)
    dev = to_device(bank, cuda_device)
    qb = QuantizedBank(dev["w13_weight"], dev["w13_scale_inv"], dev["w2_weight"], dev["w2_scale_inv"],
                       dev["w13_qzeros"], dev["w2_qzeros"])
    y = QuantizedB200Backend(0).forward(x.to(cuda_device), ids.to(cuda_device), w.to(cuda_device), qb)
    expected = R.int4_forward(np_f32(x), ids.numpy(), np_f32(w), np_bank(bank))
    assert_parity(np_f32(y), expected, label=f"int4 T={tokens} asym={asym}")


def _int4_config2(device, seed, experts=128, scale_dtype=torch.bfloat16):
    """The config-2 shape (hidden 2048, intermediate 768, top-8), asymmetric,
    the one-launch layer's envelope for one bfloat16 row."""
    from drama_b200 import QuantizedBank, synthetic

    bank = synthetic.int4_bank(experts, 2048, 768, seed, asymmetric=True, scale_dtype=scale_dtype)
    dev = to_device(bank, device)
    qb = QuantizedBank(dev["w13_weight"], dev["w13_scale_inv"], dev["w2_weight"], dev["w2_scale_inv"],
                       dev["w13_qzeros"], dev["w2_qzeros"])
    return bank, qb


@pytest.mark.parametrize("scale_dtype", [torch.bfloat16, torch.float16])
def test_int4_one_row_layer_out_and_pairs(cuda_device, scale_dtype):
    """One row at the config-2 shape takes the one-launch layer; with both
    outputs given it writes the weighted partial of every route slot
    (pair_out) and their slot-order sum (out), repeated slots included."""
    import ctypes

    from drama_b200 import _lib, synthetic
    from drama_b200.backend import _int4_bank

    bank, qb = _int4_config2(cuda_device, 71, scale_dtype=scale_dtype)
    x = synthetic.hidden_states(1, 2048, 72)
    ids = torch.tensor([[5, 17, 5, 90, 127, 0, 64, 33]], dtype=torch.int32)
    w = torch.softmax(torch.randn(1, 8, generator=torch.Generator().manual_seed(73)), -1).to(torch.bfloat16)
    lib = _lib.library()
    desc, keep = _int4_bank(qb, 2048)
    xd, idd, wd = x.to(cuda_device), ids.to(cuda_device), w.to(cuda_device)
    out = torch.empty_like(xd)
    pairs = torch.empty(8, 2048, device=cuda_device, dtype=torch.float32)
    nbytes = lib.dll.drama_b200_decode_workspace_bytes(1, 8, 2048, 768)
    ws = torch.zeros(nbytes, device=cuda_device, dtype=torch.uint8)  # zero-filled, as the ABI requires
    lib.check(lib.dll.drama_b200_int4_decode(
        ctypes.byref(desc), xd.data_ptr(), _lib.DTYPE_CODES[xd.dtype], 1, 8, idd.data_ptr(),
        _lib.DTYPE_CODES[idd.dtype], wd.data_ptr(), _lib.DTYPE_CODES[wd.dtype], out.data_ptr(), pairs.data_ptr(),
        ws.data_ptr(), ws.numel(), _lib.stream_handle(xd.device)))
    torch.cuda.synchronize(cuda_device)
    del keep
    nb = np_bank(bank)
    want_pairs = R.int4_dequant_pairs(np.repeat(np_f32(x), 8, axis=0), ids.numpy().reshape(-1),
                                      np_f32(w).reshape(-1), nb)
    assert_parity(np_f32(pairs), want_pairs, label="int4 layer pair_out")
    assert_parity(np_f32(out), R.combine_slots(want_pairs, 1, 8, "bfloat16"), label="int4 layer out")
    # the pair rows are the slot partials the sum is made of, added in slot order
    total = np.zeros(2048, dtype=np.float32)
    for j in range(8):
        total = (total + np_f32(pairs)[j]).astype(np.float32)
    np.testing.assert_array_equal(np_f32(out)[0], R.round_bf16(total))


def test_int4_one_row_layer_after_larger_batches(cuda_device):
    """The layer's arrival tickets share the workspace with the grouped
    schedule of larger batches: one row after 16 and 4 rows (and again) on
    the same workspace still matches the oracle."""
    from drama_b200 import QuantizedB200Backend, synthetic

    bank, qb = _int4_config2(cuda_device, 81, experts=64)
    nb = np_bank(bank)
    backend = QuantizedB200Backend(0)
    for step, tokens in enumerate((16, 1, 4, 1, 1)):
        x = synthetic.hidden_states(tokens, 2048, 82 + step)
        ids, w = synthetic.uniform_routes(tokens, 8, 64, 83 + step)
        w = w.to(torch.bfloat16)
        y = backend.forward(x.to(cuda_device), ids.to(cuda_device), w.to(cuda_device), qb)
        assert_parity(np_f32(y), R.int4_forward(np_f32(x), ids.numpy(), np_f32(w), nb),
                      label=f"int4 step {step} T={tokens}")


def test_int4_decode_matches_reference_goldens(cuda_device):
    from drama_b200 import QuantizedB200Backend, QuantizedBank, synthetic

    g = np.load(GOLDEN / "int4_sym.npz")
    backend = QuantizedB200Backend(0)
    for name in sorted({k.split("/")[0] for k in g.files}):
        hidden, inter, experts, tokens, top_k, seed = (int(v) for v in g[f"{name}/params"])
        bank = to_device(synthetic.int4_bank(experts, hidden, inter, seed, asymmetric=False,
                                             scale_dtype=torch.float16), cuda_device)
        x = synthetic.hidden_states(tokens, hidden, seed + 500).to(cuda_device)
        ids = torch.from_numpy(g[f"{name}/ids"]).to(cuda_device)
        w = torch.from_numpy(g[f"{name}/weights"]).to(torch.bfloat16).to(cuda_device)
        qb = QuantizedBank(bank["w13_weight"], bank["w13_scale_inv"], bank["w2_weight"], bank["w2_scale_inv"])
        y = backend.forward(x, ids, w, qb)
        assert_parity(np_f32(y), R.from_bf16_bits(g[f"{name}/forward"]), label=f"int4 golden {name}")
