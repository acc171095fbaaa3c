"""Generate golden vectors by running the reference's own Python code on CPU.

Run in a container that has the Drama3-Studio sources (never on the GPU box):

    python tests/golden/make_golden.py --reference /path/to/Drama3-Studio/src

Inputs come from the seeded generators in ``drama_b200.synthetic``; each
fixture stores the generator parameters, a SHA-256 of every generated input
(so a test detects generator drift) and the reference outputs:

* ``fp8_dequant.npz`` - ``TorchExpertBackend.forward`` / ``forward_pairs``
  (``src/drama_low_vram/offload.py:199-244``), the PyTorch dequant path.
* ``int4_sym.npz``    - ``QuantizedExpertBackend(0)`` with ``tuned_tiles=False``
  (``src/drama_low_vram/quantized_kernels.py:217-248``), symmetric zp=8,
  fp16 scales (the reference's only INT4 form).
* ``w8a8.npz``        - ``fp8_cpu_reference.expert_pairs``
  (``src/drama_low_vram/fp8_cpu_reference.py:37-52``).
* ``permute.npz``     - ``torch.argsort(flat, stable=True)`` + ``bincount`` as
  ``ExpertOffloadManager._forward_partitioned`` runs them (offload.py:1206-1211).
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "drama3-studio_b200"))

from drama_b200 import synthetic  # noqa: E402

FP8_CASES = [
    # name, hidden, intermediate, experts, tokens, top_k, dtype, seed
    ("small_bf16", 256, 128, 4, 1, 4, "bfloat16", 11),
    ("small_t3_bf16", 256, 256, 8, 3, 8, "bfloat16", 12),
    ("small_fp16", 256, 128, 4, 2, 3, "float16", 13),
    ("small_fp32", 256, 128, 4, 2, 3, "float32", 14),
    ("dup_routes", 256, 128, 8, 1, 8, "bfloat16", 15),
    ("baseline_b1", 2048, 768, 8, 1, 8, "bfloat16", 16),
]

INT4_CASES = [
    ("small_b1", 256, 128, 4, 1, 4, 21),
    ("small_b3", 256, 256, 8, 3, 8, 22),
    ("baseline_b1", 2048, 768, 8, 1, 8, 23),
    ("baseline_b4", 2048, 768, 16, 4, 8, 24),
]

W8A8_CASES = [
    ("small", 256, 128, 4, 4, 31),
    ("baseline", 2048, 768, 8, 8, 32),
]

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def digest(t: torch.Tensor) -> str:
    a = t.detach().cpu().contiguous()
    if a.dtype in (torch.bfloat16, torch.float8_e4m3fn):
        a = a.view(torch.uint8 if a.dtype == torch.float8_e4m3fn else torch.int16)
    return hashlib.sha256(a.numpy().tobytes()).hexdigest()


def routes_for(name: str, tokens: int, top_k: int, experts: int, seed: int):
    if name == "dup_routes":
        ids = torch.tensor([[3, 1, 3, 0, 2, 7, 1, 5]])
        w = torch.softmax(torch.randn(1, 8, generator=torch.Generator().manual_seed(seed)), -1)
        return ids, w
    return synthetic.uniform_routes(tokens, top_k, experts, seed + 1000)


def as_bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.numpy().view(np.uint16)
    return t.numpy()


def make_fp8(ref) -> dict:
    out = {}
    for name, hidden, inter, experts, tokens, top_k, dtype, seed in FP8_CASES:
        bank = synthetic.fp8_bank(experts, hidden, inter, seed)
        staged = ref.StagedExperts(**bank)
        x = synthetic.hidden_states(tokens, hidden, seed + 500, dtype=DTYPES[dtype])
        ids, w = routes_for(name, tokens, top_k, experts, seed)
        w = w.to(DTYPES[dtype])
        backend = ref.TorchExpertBackend()
        y = backend.forward(x, ids, w, staged)
        pairs = backend.forward_pairs(x.repeat_interleave(top_k, 0), ids.reshape(-1, 1),
                                      w.reshape(-1, 1), staged)
        out[f"{name}/params"] = np.array([hidden, inter, experts, tokens, top_k, seed])
        out[f"{name}/dtype"] = np.array(dtype)
        for key, t in bank.items():
            out[f"{name}/sha_{key}"] = np.array(digest(t))
        out[f"{name}/sha_x"] = np.array(digest(x))
        out[f"{name}/ids"] = ids.numpy()
        out[f"{name}/weights"] = w.float().numpy()
        out[f"{name}/forward"] = as_bits(y)
        out[f"{name}/pairs"] = pairs.numpy()
    return out


def make_int4(ref_q, ref_o) -> dict:
    out = {}
    for name, hidden, inter, experts, tokens, top_k, seed in INT4_CASES:
        bank = synthetic.int4_bank(experts, hidden, inter, seed, asymmetric=False,
                                   scale_dtype=torch.float16)
        staged = ref_o.StagedExperts(bank["w13_weight"], bank["w13_scale_inv"],
                                     bank["w2_weight"], bank["w2_scale_inv"])
        x = synthetic.hidden_states(tokens, hidden, seed + 500)
        ids, w = synthetic.uniform_routes(tokens, top_k, experts, seed + 1000)
        w = w.to(torch.bfloat16)
        backend = ref_q.QuantizedExpertBackend(0)
        backend.tuned_tiles = False
        with torch.inference_mode():
            y = backend.forward(x, ids, w, staged)
        out[f"{name}/params"] = np.array([hidden, inter, experts, tokens, top_k, seed])
        for key in ("w13_weight", "w13_scale_inv", "w2_weight", "w2_scale_inv"):
            out[f"{name}/sha_{key}"] = np.array(digest(bank[key]))
        out[f"{name}/sha_x"] = np.array(digest(x))
        out[f"{name}/ids"] = ids.numpy()
        out[f"{name}/weights"] = w.float().numpy()
        out[f"{name}/forward"] = as_bits(y)
    return out


def make_w8a8(ref_f, ref_o) -> dict:
    out = {}
    for name, hidden, inter, experts, jobs, seed in W8A8_CASES:
        bank = synthetic.fp8_bank(experts, hidden, inter, seed)
        store = ref_o.ExpertStore(**bank)
        x = synthetic.hidden_states(1, hidden, seed + 500)[0]
        ids = torch.tensor([(3 * j + 1) % experts for j in range(jobs)])
        w = torch.softmax(torch.randn(jobs, generator=torch.Generator().manual_seed(seed)), -1)
        pairs = ref_f.expert_pairs(store, x, ids, w)
        out[f"{name}/params"] = np.array([hidden, inter, experts, jobs, seed])
        for key, t in bank.items():
            out[f"{name}/sha_{key}"] = np.array(digest(t))
        out[f"{name}/sha_x"] = np.array(digest(x))
        out[f"{name}/ids"] = ids.numpy()
        out[f"{name}/weights"] = w.numpy()
        out[f"{name}/pairs"] = pairs.numpy()
    return out


def make_permute() -> dict:
    out = {}
    cases = {
        "decode_b1": synthetic.uniform_routes(1, 8, 128, 41)[0],
        "verify_b4": synthetic.uniform_routes(4, 8, 128, 42)[0],
        "dense_dups": torch.randint(0, 6, (64, 8), generator=torch.Generator().manual_seed(43)),
        "zipf_4096": synthetic.zipf_routes(4096, 8, 128, 44)[0],
        "single_expert": torch.zeros(5, 3, dtype=torch.int64),
    }
    experts = {"decode_b1": 128, "verify_b4": 128, "dense_dups": 6, "zipf_4096": 128,
               "single_expert": 4}
    for name, ids in cases.items():
        flat = ids.reshape(-1)
        out[f"{name}/ids"] = ids.numpy()
        out[f"{name}/experts"] = np.array(experts[name])
        out[f"{name}/order"] = torch.argsort(flat, stable=True).numpy()
        out[f"{name}/counts"] = torch.bincount(flat, minlength=experts[name]).numpy()
    return out


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=str(Path(__file__).resolve().parents[3] / "reference" / "src"))
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    torch.manual_seed(0)
    from drama_low_vram import fp8_cpu_reference as ref_f
    from drama_low_vram import offload as ref_o
    from drama_low_vram import quantized_kernels as ref_q

    np.savez_compressed(HERE / "fp8_dequant.npz", **make_fp8(ref_o))
    np.savez_compressed(HERE / "int4_sym.npz", **make_int4(ref_q, ref_o))
    np.savez_compressed(HERE / "w8a8.npz", **make_w8a8(ref_f, ref_o))
    np.savez_compressed(HERE / "permute.npz", **make_permute())
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
