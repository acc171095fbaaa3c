// Pieces shared by the grouped expert GEMMs (prefill_gemm.cu, expert_rows.cu):
// the bf16 tensor-core MMA, the FP8 expansion, the tile walk over experts and
// the SwiGLU rounding points of TorchExpertBackend (src/drama_low_vram/
// offload.py:237-238: gate and up rounded to bf16, silu(gate) rounded to
// bf16, times up rounded to bf16).
#pragma once

#include "common.cuh"
#include "decode_tiles.cuh"

namespace drama {

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// FP8 E4M3 x4 -> 4 fp32 (exact): bytes 0, 1 -> lo halves; 2, 3 -> hi.
__device__ __forceinline__ void fp8x4_to_f32(uint32_t w, float (&o)[4]) {
    uint32_t lo, hi;
    e4m3x4_to_f16x2x2(w, lo, hi);
    o[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(lo & 0xffffu)));
    o[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(lo >> 16)));
    o[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(hi & 0xffffu)));
    o[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(hi >> 16)));
}

// Four E4M3 bytes times their block scale as two bf16x2 words, the
// reference's dequant rounding bf16(fp8 * scale) (offload.py:44-56).
__device__ __forceinline__ void fp8x4_dequant_bf16(uint32_t w, float scale, uint32_t& lo, uint32_t& hi) {
    float v[4];
    fp8x4_to_f32(w, v);
    const __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0] * scale, v[1] * scale);
    const __nv_bfloat162 p1 = __floats2bfloat162_rn(v[2] * scale, v[3] * scale);
    lo = *reinterpret_cast<const uint32_t*>(&p0);
    hi = *reinterpret_cast<const uint32_t*>(&p1);
}

// h = bf16(bf16(silu(bf16(gate))) * bf16(up)) from fp32 accumulators, as fp32.
__device__ __forceinline__ float swiglu_rounded(float gate_acc, float up_acc) {
    const float gate = __bfloat162float(__float2bfloat16_rn(gate_acc));
    const float up = __bfloat162float(__float2bfloat16_rn(up_acc));
    const float act = __bfloat162float(__float2bfloat16_rn(gate / (1.0f + expf(-gate))));
    return act * up;
}

// Tile t of the flattened list (expert, m block, n block); prefix[e] = tiles
// of experts < e.
__device__ __forceinline__ void decode_tile(int t, const int* prefix, int E, int nblocks, int& e, int& mb, int& nb) {
    int lo = 0, hi = E;  // largest e with prefix[e] <= t
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] <= t) lo = mid;
        else hi = mid;
    }
    e = lo;
    const int local = t - prefix[lo];
    mb = local / nblocks;
    nb = local % nblocks;
}

}  // namespace drama
