"""Golden vectors for W8A8 modes 1-3 from the reference's own Python code.

Run in a container that has the Drama3-Studio sources (never on the GPU box):

    python tests/golden/make_convrot_golden.py --reference /path/to/Drama3-Studio/src

For each mode (1 INT8-ConvRot, 2 W6A8, 3 W4A8 codebook) the bank comes from
``drama_b200.synthetic.w8a8_bank`` (numpy PCG64, seed recorded with a SHA-256
of its bytes), the hidden rows and routes from a seeded numpy stream. Stored:

* ``grid13_{m}``, ``grid2_{m}`` - SHA-256 of the int8 weight grids of all
                  experts as the reference's own test reconstructs them
                  (tests/test_quantized_kernels.py:47-73):
                  ``clamp(round(level * relative), +-127)``; mode 1 the weights.
* ``forward{m}``- ``QuantizedExpertBackend(m).forward`` (quantized_kernels.py:
                  217-229) on CPU tensors, i.e. through ``projection_torch``
                  (48-112), the reference's bounded fallback; ``tuned_tiles``
                  off (a tile choice only).
* ``pairs{m}``  - ``forward_pairs`` of the same call (weighted fp32 partials).
* ``dq{m}``     - ``projection_torch(x, ., identity bank, mode=1)``: the
                  reference's rotated-and-quantized activations, dequantized
                  and rounded to bf16.
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HIDDEN, INTER, EXPERTS, TOKENS, TOP_K = 256, 256, 3, 4, 2
OUT = Path(__file__).resolve().parent / "convrot_w8a8.npz"


def inputs(mode: int):
    from drama_b200 import synthetic

    bank = synthetic.w8a8_bank(mode, EXPERTS, HIDDEN, INTER, seed=400 + mode)
    rng = np.random.default_rng(500 + mode)
    x = torch.from_numpy(rng.standard_normal((TOKENS, HIDDEN)).astype(np.float32)).to(torch.bfloat16)
    ids = torch.from_numpy(np.stack([rng.permutation(EXPERTS)[:TOP_K] for _ in range(TOKENS)]).astype(np.int64))
    w = torch.from_numpy(rng.random((TOKENS, TOP_K)).astype(np.float32)).to(torch.bfloat16)
    return bank, x, ids, w


def bank_sha(bank) -> str:
    h = hashlib.sha256()
    for name in sorted(bank):
        h.update(bank[name].contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def explicit_grid(weight, scales, mode: int, k: int) -> torch.Tensor:
    """The reconstruction of tests/test_quantized_kernels.py:47-73, from packed bytes."""
    if mode == 1:
        return weight.clone()
    raw = weight.view(torch.uint8).long()
    low = raw[..., :k // 2]
    codes = torch.stack((low & 15, low >> 4), -1).reshape(*raw.shape[:-1], k)
    if mode == 2:
        high = raw[..., k // 2:k // 2 + k // 4]
        top = torch.stack([(high >> (2 * i)) & 3 for i in range(4)], -1).reshape(*raw.shape[:-1], k)
        levels = (codes | (top << 4)).float() - 32
    else:
        tables = scales[..., :16, k // 16 + 4:k // 16 + 8].contiguous().view(torch.float32).reshape(-1, 16)
        levels = torch.stack([tables[i][codes[i]] for i in range(codes.shape[0])])
    relative = scales[..., :k // 16].contiguous().view(torch.float8_e4m3fn).float()
    grid = levels * relative.repeat_interleave(16, dim=-1)
    return grid.round().clamp(-127, 127).to(torch.int8)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="the reference's src directory")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, str(Path(__file__).resolve().parents[2] / "drama3-studio_b200"))
    from drama_low_vram.quantized_kernels import QuantizedExpertBackend, projection_torch

    out = {}
    for mode in (1, 2, 3):
        bank, x, ids, w = inputs(mode)
        out[f"sha{mode}"] = np.frombuffer(bank_sha(bank).encode(), dtype=np.uint8)
        for name, k in (("13", HIDDEN), ("2", INTER)):
            grid = explicit_grid(bank[f"w{name}_weight"], bank[f"w{name}_scale_inv"], mode, k)
            digest = hashlib.sha256(grid.numpy().tobytes()).hexdigest()
            out[f"grid{name}_{mode}"] = np.frombuffer(digest.encode(), dtype=np.uint8)
        backend = QuantizedExpertBackend(mode)
        backend.tuned_tiles = False
        staged = SimpleNamespace(**bank)
        with torch.inference_mode():
            out[f"forward{mode}"] = backend.forward(x, ids, w, staged).float().numpy()
            out[f"pairs{mode}"] = backend.forward_pairs(
                x.repeat_interleave(TOP_K, 0), ids.reshape(-1, 1), w.reshape(-1, 1), staged).float().numpy()
            eye = torch.eye(HIDDEN, dtype=torch.int8)[None]
            ones = torch.ones((1, HIDDEN, 1), dtype=torch.float32)
            out[f"dq{mode}"] = projection_torch(x, torch.zeros(TOKENS, dtype=torch.int64), None, eye, ones,
                                                mode=1).float().numpy()
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
