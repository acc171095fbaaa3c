"""Seeded synthetic expert banks, hidden rows and routes (the benchmark inputs).

The reference measures nothing on a public dataset; its checkpoints are not
available here, so every bank is generated from a seed with the shapes and
value distributions of the benchmark configurations:

* FP8: weights N(0, 0.02) quantised to E4M3 with an fp32 scale per 128x128
  block (scale = block amax / 448), the layout of ``ExpertStore``
  (``src/drama_low_vram/offload.py:101-172``).
* INT4 W4A16: the GPTQ mode-0 layout of ``QuantizedStore``
  (``src/drama_low_vram/quantized_model.py:26-68``): ``[E, N, K/8]`` int32 with
  nibble ``k % 8`` at bit ``4*(k % 8)``, group 128 along K, plus (asymmetric)
  ``[E, N/8, K/128]`` int32 zero-points, nibble ``n % 8`` at bit ``4*(n % 8)``.
* W8A8 modes 1-3 (INT8-ConvRot, W6A8, W4A8 codebook): the ``QuantizedStore``
  layouts of ``quantized_model.py:45-68, 114-151`` with the value ranges of the
  reference's own kernel test (``tests/test_quantized_kernels.py:47-69``):
  uniform int8 / 6-bit / 4-bit codes, FP8 relative scales in [1, 2), fp32
  channel scales sized so a projection's outputs are O(1).
* Activations bf16 N(0, 1); router weight bf16 N(0, 0.02); RMSNorm gamma
  1 + N(0, 0.01).

Everything runs on any torch device, so the same code builds a 29 GB resident
bank on the GPU for the benchmark and a small bank on the CPU for a test.
"""

from __future__ import annotations

import math

import numpy as np
import torch

FP8 = torch.float8_e4m3fn
BLOCK = 128


def _generator(seed: int, device) -> torch.Generator:
    gen = torch.Generator(device=torch.device(device))
    gen.manual_seed(int(seed))
    return gen


def quantize_fp8_blocks(weight: torch.Tensor):
    """[.., R, C] float -> (E4M3 [.., R, C], fp32 scales [.., R/128, C/128])."""
    *lead, rows, cols = weight.shape
    blocks = weight.float().reshape(*lead, rows // BLOCK, BLOCK, cols // BLOCK, BLOCK)
    amax = blocks.abs().amax(dim=(-3, -1)).clamp_min(1e-12)
    scale = amax / 448.0
    q = (blocks / scale[..., :, None, :, None]).clamp(-448, 448).to(FP8)
    return q.reshape(weight.shape), scale.contiguous()


def fp8_bank(experts: int, hidden: int, intermediate: int, seed: int, *, device="cpu",
             std: float = 0.02, chunk: int = 1) -> dict[str, torch.Tensor]:
    """An ``ExpertStore``-shaped FP8 bank, generated ``chunk`` experts at a time.

    The random stream depends on ``chunk``; tests use the default (1).
    """
    dev = torch.device(device)
    gen = _generator(seed, dev)
    bank = {
        "w13_weight": torch.empty(experts, 2 * intermediate, hidden, dtype=FP8, device=dev),
        "w13_scale_inv": torch.empty(experts, 2 * intermediate // BLOCK, hidden // BLOCK, device=dev),
        "w2_weight": torch.empty(experts, hidden, intermediate, dtype=FP8, device=dev),
        "w2_scale_inv": torch.empty(experts, hidden // BLOCK, intermediate // BLOCK, device=dev),
    }
    for e in range(0, experts, chunk):
        n = min(chunk, experts - e)
        for name, rows, cols in (("w13", 2 * intermediate, hidden), ("w2", hidden, intermediate)):
            w = torch.randn(n, rows, cols, generator=gen, device=dev) * std
            q, s = quantize_fp8_blocks(w)
            bank[f"{name}_weight"][e:e + n].copy_(q)
            bank[f"{name}_scale_inv"][e:e + n].copy_(s)
            del w, q, s
    return bank


def pack_int4_rows(codes: torch.Tensor) -> torch.Tensor:
    """[.., K] codes 0..15 -> [.., K/8] int32, nibble k%8 at bit 4*(k%8)."""
    *lead, k = codes.shape
    c = codes.to(torch.int64).reshape(*lead, k // 8, 8)
    shifts = torch.arange(8, device=codes.device, dtype=torch.int64) * 4
    words = (c << shifts).sum(-1)
    return (words - ((words >> 31) << 32)).to(torch.int32)


def pack_int4_zeros(zeros: torch.Tensor) -> torch.Tensor:
    """[.., N, G] zero-points -> [.., N/8, G] int32, nibble n%8 at bit 4*(n%8)."""
    *lead, n, g = zeros.shape
    z = zeros.to(torch.int64).reshape(*lead, n // 8, 8, g)
    shifts = (torch.arange(8, device=zeros.device, dtype=torch.int64) * 4)[:, None]
    words = (z << shifts).sum(-2)
    return (words - ((words >> 31) << 32)).to(torch.int32)


def quantize_int4_groups(weight: torch.Tensor, *, asymmetric: bool = True,
                         scale_dtype=torch.bfloat16):
    """Group-128 W4 quantisation: returns (words, scales, qzeros or None)."""
    rows, cols = weight.shape[-2:]
    lead = weight.shape[:-2]
    g = weight.float().reshape(*lead, rows, cols // BLOCK, BLOCK)
    if asymmetric:
        lo = g.amin(-1).clamp(max=0.0)
        hi = g.amax(-1).clamp(min=0.0)
        scale = ((hi - lo) / 15.0).clamp_min(1e-8).to(scale_dtype).float()
        zero = torch.round(-lo / scale).clamp(0, 15)
    else:
        scale = (g.abs().amax(-1) / 7.0).clamp_min(1e-8).to(scale_dtype).float()
        zero = torch.full_like(scale, 8.0)
    codes = torch.round(g / scale[..., None] + zero[..., None]).clamp(0, 15)
    words = pack_int4_rows(codes.reshape(*lead, rows, cols))
    qzeros = pack_int4_zeros(zero.to(torch.int64)) if asymmetric else None
    return words, scale.to(scale_dtype), qzeros


def int4_bank(experts: int, hidden: int, intermediate: int, seed: int, *, device="cpu",
              std: float = 0.02, asymmetric: bool = True,
              scale_dtype=torch.bfloat16) -> dict[str, torch.Tensor | None]:
    dev = torch.device(device)
    gen = _generator(seed, dev)
    out: dict[str, list] = {k: [] for k in ("w13_weight", "w13_scale_inv", "w13_qzeros",
                                            "w2_weight", "w2_scale_inv", "w2_qzeros")}
    for _ in range(experts):
        for name, rows, cols in (("w13", 2 * intermediate, hidden), ("w2", hidden, intermediate)):
            w = torch.randn(rows, cols, generator=gen, device=dev) * std
            words, scales, zeros = quantize_int4_groups(w, asymmetric=asymmetric,
                                                        scale_dtype=scale_dtype)
            out[f"{name}_weight"].append(words)
            out[f"{name}_scale_inv"].append(scales)
            out[f"{name}_qzeros"].append(zeros)
    bank = {}
    for key, parts in out.items():
        bank[key] = None if parts[0] is None else torch.stack(parts).contiguous()
    return bank


def hidden_states(tokens: int, hidden: int, seed: int, *, device="cpu",
                  dtype=torch.bfloat16) -> torch.Tensor:
    gen = _generator(seed, device)
    return torch.randn(tokens, hidden, generator=gen, device=device).to(dtype)


def gate_weight(experts: int, hidden: int, seed: int, *, device="cpu", std: float = 0.02):
    gen = _generator(seed, device)
    return (torch.randn(experts, hidden, generator=gen, device=device) * std).to(torch.bfloat16)


def norm_gamma(hidden: int, seed: int, *, device="cpu", std: float = 0.01):
    gen = _generator(seed, device)
    return (1.0 + torch.randn(hidden, generator=gen, device=device) * std).float()


def uniform_routes(tokens: int, top_k: int, experts: int, seed: int, *, device="cpu"):
    """``top_k`` distinct experts per token, uniform; softmax route weights."""
    gen = _generator(seed, "cpu")
    keys = torch.rand(tokens, experts, generator=gen)
    ids = keys.topk(top_k, dim=-1).indices
    w = torch.softmax(torch.randn(tokens, top_k, generator=gen), -1)
    return ids.to(device), w.to(device)


def zipf_routes(tokens: int, top_k: int, experts: int, seed: int, *, s: float = 1.1,
                device="cpu"):
    """``top_k`` distinct experts per token drawn proportional to rank^-s.

    Gumbel-top-k sampling without replacement over a seeded permutation of
    expert ranks; route weights are a softmax of N(0,1) logits.
    """
    gen = _generator(seed, "cpu")
    perm = torch.randperm(experts, generator=gen)
    logp = -s * torch.log(torch.arange(1, experts + 1, dtype=torch.float64))
    logp = logp[torch.argsort(perm)]
    u = torch.rand(tokens, experts, generator=gen, dtype=torch.float64).clamp_min(1e-300)
    gumbel = -torch.log(-torch.log(u))
    ids = (logp[None, :] + gumbel).topk(top_k, dim=-1).indices
    w = torch.softmax(torch.randn(tokens, top_k, generator=gen), -1)
    return ids.to(device), w.to(device)


def expert_nbytes_fp8(hidden: int, intermediate: int) -> int:
    """Bytes of one FP8 expert: weights + fp32 block scales (4,719,744 at 2048/768)."""
    w = 3 * hidden * intermediate
    s = 4 * (2 * intermediate // BLOCK * hidden // BLOCK + hidden // BLOCK * intermediate // BLOCK)
    return w + s


def expert_nbytes_int4(hidden: int, intermediate: int) -> int:
    """Bytes of one asymmetric W4A16 expert (2,451,456 at 2048/768)."""
    n13, n2 = 2 * intermediate, hidden
    words = 4 * (n13 * hidden // 8 + n2 * intermediate // 8)
    scales = 2 * (n13 * hidden // BLOCK + n2 * intermediate // BLOCK)
    zeros = 4 * (n13 // 8 * hidden // BLOCK + n2 // 8 * math.ceil(intermediate / BLOCK))
    return words + scales + zeros


def w8a8_bank(mode: int, experts: int, hidden: int, intermediate: int, seed: int) -> dict[str, torch.Tensor]:
    """A ``QuantizedStore``-shaped CPU bank for W8A8 mode 1, 2 or 3 (numpy PCG64 stream).

    mode 1: ``[E, N, K]`` int8 weights, ``[E, N, 1]`` fp32 channel scales.
    mode 2: ``[E, N, 3K/4]`` int8 (K/2 bytes of low nibbles, column 2j in the
            low nibble of byte j; then K/4 bytes of top-two bits, column 4j+i
            at bits 2i of byte j); ``[E, N, K/16 + 4]`` uint8 scales (FP8
            relative scale per 16 columns, then the fp32 channel scale).
    mode 3: ``[E, N, K/2]`` int8 4-bit codes; ``[E, N, K/16 + 8]`` uint8 (as
            mode 2, plus one fp32 codebook entry in bytes K/16+4.. of rows 0-15).
    """
    if mode not in (1, 2, 3):
        raise ValueError("W8A8 banks are modes 1, 2 and 3")
    rng = np.random.default_rng(seed)
    typical = {1: 64.0, 2: 24.0, 3: 10.0}[mode]  # mean |grid value| of the mode
    bank = {}
    for name, n, k in (("w13", 2 * intermediate, hidden), ("w2", hidden, intermediate)):
        channel = (rng.random((experts, n, 1)) / (typical * math.sqrt(k))).astype(np.float32)
        if mode == 1:
            bank[f"{name}_weight"] = torch.from_numpy(rng.integers(-127, 128, (experts, n, k), dtype=np.int8))
            bank[f"{name}_scale_inv"] = torch.from_numpy(channel)
            continue
        codes = rng.integers(0, 64 if mode == 2 else 16, (experts, n, k))
        low = (codes[..., 0::2] & 15) | ((codes[..., 1::2] & 15) << 4)
        if mode == 2:
            high = np.zeros((experts, n, k // 4), dtype=np.int64)
            for i in range(4):
                high |= ((codes[..., i::4] >> 4) & 3) << (2 * i)
            raw = np.concatenate((low, high), axis=-1)
        else:
            raw = low
        relative = torch.from_numpy((rng.random((experts, n, k // 16)) + 1.0).astype(np.float32)).to(FP8)
        aux = torch.zeros((experts, n, k // 16 + (8 if mode == 3 else 4)), dtype=torch.uint8)
        aux[..., :k // 16] = relative.view(torch.uint8)
        aux[..., k // 16:k // 16 + 4] = torch.from_numpy(channel).view(torch.uint8)
        if mode == 3:
            table = np.linspace(-12.0, 13.0, 16) + rng.normal(0.0, 0.25, (experts, 16))
            aux[:, :16, k // 16 + 4:] = torch.from_numpy(table.astype(np.float32)).view(torch.uint8).reshape(
                experts, 16, 4)
        bank[f"{name}_weight"] = torch.from_numpy(raw.astype(np.uint8)).view(torch.int8)
        bank[f"{name}_scale_inv"] = aux
    return bank
