// Shared device helpers for the B200 routed-expert kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "drama_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "drama_b200 kernels are written for sm_100a (B200) only"
#endif

namespace drama {

// ---------------------------------------------------------------------------
// Host-side error plumbing: every entry point validates before it launches and
// reports failures as a status code plus a thread-local message.
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(const char* fmt, ...);
int check_launch(const char* what);

// ---------------------------------------------------------------------------
// Scalar conversions with the reference's rounding points.
// ---------------------------------------------------------------------------
template <int DT> struct Scalar;
template <> struct Scalar<DRAMA_B200_F32> {
    using T = float;
    static __device__ __forceinline__ float load(const T* p) { return *p; }
    static __device__ __forceinline__ float round(float v) { return v; }
    static __device__ __forceinline__ T from(float v) { return v; }
};
template <> struct Scalar<DRAMA_B200_BF16> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ float load(const T* p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ float round(float v) {
        return __bfloat162float(__float2bfloat16_rn(v));
    }
    static __device__ __forceinline__ T from(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Scalar<DRAMA_B200_F16> {
    using T = __half;
    static __device__ __forceinline__ float load(const T* p) { return __half2float(*p); }
    static __device__ __forceinline__ float round(float v) {
        return __half2float(__float2half_rn(v));
    }
    static __device__ __forceinline__ T from(float v) { return __float2half_rn(v); }
};

__device__ __forceinline__ float load_any(const void* base, int dtype, int64_t i) {
    switch (dtype) {
        case DRAMA_B200_F32: return static_cast<const float*>(base)[i];
        case DRAMA_B200_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
        default: return __half2float(static_cast<const __half*>(base)[i]);
    }
}

__device__ __forceinline__ int64_t load_index(const void* base, int dtype, int64_t i) {
    return dtype == DRAMA_B200_I64 ? static_cast<const int64_t*>(base)[i]
                                   : static_cast<int64_t>(static_cast<const int32_t*>(base)[i]);
}

__device__ __forceinline__ void store_index(void* base, int dtype, int64_t i, int64_t v) {
    if (dtype == DRAMA_B200_I64) static_cast<int64_t*>(base)[i] = v;
    else static_cast<int32_t*>(base)[i] = static_cast<int32_t>(v);
}

__device__ __forceinline__ void store_any(void* base, int dtype, int64_t i, float v) {
    switch (dtype) {
        case DRAMA_B200_F32: static_cast<float*>(base)[i] = v; break;
        case DRAMA_B200_BF16: static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v); break;
        default: static_cast<__half*>(base)[i] = __float2half_rn(v); break;
    }
}

__device__ __forceinline__ float round_any(float v, int dtype) {
    switch (dtype) {
        case DRAMA_B200_F32: return v;
        case DRAMA_B200_BF16: return __bfloat162float(__float2bfloat16_rn(v));
        default: return __half2float(__float2half_rn(v));
    }
}

// ---------------------------------------------------------------------------
// PTX wrappers.
// ---------------------------------------------------------------------------

// Programmatic dependent launch: wait for the predecessor grid's results, and
// let the successor grid start its prologue.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Atomic add with acquire-release semantics at GPU scope (the pattern of a
// split-K semaphore): after a CTA barrier the release covers every write the
// CTA made before it, and reads that follow the next CTA barrier are ordered
// after the acquire.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Streaming 16-byte load of immutable expert weights: no L1 allocation and
// first-out in L2, so the weight stream does not evict activations or the
// down-projection slabs prefetched into L2.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p, uint64_t policy) {
    uint4 v;
    asm volatile(
        "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p), "l"(policy));
    return v;
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// Bulk prefetch of a contiguous, 16-byte aligned range into L2 (no SM copy).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Two E4M3 bytes (low 16 bits of `pair`) -> f16x2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t pair) {
    uint32_t out;
    asm("{\n\t.reg .b16 lo;\n\tcvt.u16.u32 lo, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, lo;\n\t}"
        : "=r"(out)
        : "r"(pair));
    return out;
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    uint32_t out;
    asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(out) : "f"(lo), "f"(hi));
    return out;
}

// Route-slot combine step on 8 bf16 values: acc += fp32(row) * w, the product
// rounded to fp32 before the add (offload.py:212, 1244: weighted fp32 pair
// rows summed in slot order), so no FMA contraction.
__device__ __forceinline__ void combine_accumulate(float (&acc)[8], uint4 q, float w) {
    const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        acc[2 * u] = __fadd_rn(acc[2 * u], __fmul_rn(__uint_as_float(v[u] << 16), w));
        acc[2 * u + 1] = __fadd_rn(acc[2 * u + 1], __fmul_rn(__uint_as_float(v[u] & 0xffff0000u), w));
    }
}

__device__ __forceinline__ float ld_cg_f32(const float* p) { return __ldcg(p); }

// Power-of-two exponent e such that |amax| * 2^-e lies in [2^14, 2^15): the
// f16 copy of a row scaled by 2^-e keeps every bf16 value of magnitude
// >= amax * 2^-28 exact and never overflows.
__device__ __forceinline__ int f16_exponent_for(float amax) {
    if (!(amax > 0.0f) || !isfinite(amax)) return 0;
    int e;
    frexpf(amax, &e);  // amax = m * 2^e, m in [0.5, 1)
    return e - 15;
}

}  // namespace drama
