// GPTQ W4A16 dequantisation as the reference computes it: each weight is
// bf16((code - zero) * scale) with the scale in bf16 (or fp32 from an f16
// scale), the level code - zero exact in bf16 and the product rounded once
// (QuantizedExpertBackend mode 0, src/drama_low_vram/quantized_kernels.py).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace drama {

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// bf16x2 of two levels already biased by 128 in bf16 (128 + code):
// bf16((code - zp) * scale) for both. zb = bf16x2 (128 + zp) twice; BF16: sc2 =
// bf16x2 scale twice; else scf = the fp32 scale.
template <bool BF16>
__device__ __forceinline__ uint32_t int4_dequant2(uint32_t biased, uint32_t zb, uint32_t sc2, float scf) {
    const uint32_t level = bf2_sub(biased, zb);  // code - zp, exact
    if constexpr (BF16) {
        return bf2_mul(level, sc2);  // exact product rounded once, as in fp32 then .to(bf16)
    } else {
        const float lo = __fmul_rn(__uint_as_float(level << 16), scf);
        const float hi = __fmul_rn(__uint_as_float(level & 0xffff0000u), scf);
        const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t*>(&p);
    }
}

// bf16x2 (w_i, w_{i+4}) of nibbles i and i + 4 of word W.
template <bool BF16>
__device__ __forceinline__ uint32_t int4_pair(uint32_t W, int i, uint32_t zb, uint32_t sc2, float scf) {
    return int4_dequant2<BF16>(((W >> (4 * i)) & 0x000F000Fu) | 0x43004300u, zb, sc2, scf);
}

// bf16x2 (w_0, w_1) and (w_2, w_3) of the four nibbles in the low 16 bits of v.
template <bool BF16>
__device__ __forceinline__ void int4_quad(uint32_t v, uint32_t zb, uint32_t sc2, float scf, uint32_t& lo,
                                          uint32_t& hi) {
    lo = int4_dequant2<BF16>((v & 0xFu) | ((v & 0xF0u) << 12) | 0x43004300u, zb, sc2, scf);
    hi = int4_dequant2<BF16>(((v >> 8) & 0xFu) | ((v & 0xF000u) << 4) | 0x43004300u, zb, sc2, scf);
}

// bf16x2 (128 + zp) in both halves, for int4_dequant2.
__device__ __forceinline__ uint32_t int4_zero_bias(uint32_t zp) { return (0x4300u + zp) * 0x10001u; }

}  // namespace drama
