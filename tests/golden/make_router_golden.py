"""Router golden vectors from the reference's own router ops, run on a B200.

The reference routes with torch ops inside its decode graph
(src/drama_low_vram/backbone_graph.py:319-323):

    probabilities = torch.softmax(logits.float(), dim=-1)
    topk_weights, topk_ids = probabilities.topk(top_k, dim=-1)
    topk_weights = topk_weights / topk_weights.sum(dim=-1, keepdim=True)
    topk_weights = topk_weights.to(dtype)

This script runs exactly those ops on CUDA (tie order is device-specific) on
seeded bf16 logits and writes tests/golden/router_cuda.npz:

    python tests/golden/make_router_golden.py --out tests/golden/router_cuda.npz
"""

from __future__ import annotations

import argparse

import numpy as np
import torch


def cases():
    gen = torch.Generator().manual_seed(2026)
    normal = (torch.randn(512, 128, generator=gen) * 0.905).to(torch.bfloat16)
    coarse = (torch.randint(-4, 5, (256, 128), generator=gen).float() / 4).to(torch.bfloat16)
    narrow = (torch.randn(256, 128, generator=gen) * 0.02).to(torch.bfloat16)
    equal = torch.zeros(4, 128, dtype=torch.bfloat16)
    wide = (torch.randn(128, 256, generator=gen) * 0.9).to(torch.bfloat16)
    wide_ties = (torch.randint(-2, 3, (128, 256), generator=gen).float() / 2).to(torch.bfloat16)
    small = (torch.randint(-2, 3, (64, 16), generator=gen).float()).to(torch.bfloat16)
    big = (torch.randint(-3, 4, (32, 1024), generator=gen).float() / 3).to(torch.bfloat16)
    odd = (torch.randn(64, 60, generator=gen)).to(torch.bfloat16)
    return [
        ("normal_e128_k8", normal, 8, True),
        ("coarse_ties_e128_k8", coarse, 8, True),
        ("narrow_e128_k8", narrow, 8, True),
        ("all_equal_e128_k8", equal, 8, True),
        ("e256_k8", wide, 8, True),
        ("ties_e256_k8", wide_ties, 8, True),
        ("ties_e16_k4_norenorm", small, 4, False),
        ("ties_e1024_k32", big, 32, True),
        ("odd_e60_k6", odd, 6, True),
    ]


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--out", default="tests/golden/router_cuda.npz")
    args = parser.parse_args()
    out = {"device": np.array(torch.cuda.get_device_name()), "torch": np.array(torch.__version__)}
    for name, logits, top_k, renorm in cases():
        dev = logits.cuda()
        probabilities = torch.softmax(dev.float(), dim=-1)
        w, ids = probabilities.topk(top_k, dim=-1)
        if renorm:
            w = w / w.sum(dim=-1, keepdim=True)
        w = w.to(logits.dtype)
        out[f"{name}/logits_bits"] = logits.view(torch.int16).numpy().view(np.uint16)
        out[f"{name}/top_k"] = np.array(top_k)
        out[f"{name}/renorm"] = np.array(renorm)
        out[f"{name}/ids"] = ids.cpu().numpy()
        out[f"{name}/weights_bits"] = w.cpu().view(torch.int16).numpy().view(np.uint16)
        out[f"{name}/probs"] = probabilities.cpu().numpy()
    np.savez_compressed(args.out, **out)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
