// tcgen05 (5th-generation tensor core) helpers for sm_100a kernels.
//
// The shared-memory and instruction descriptors are CuTe's sm100 UMMA
// bitfield unions (cute/arch/mma_sm100_desc.hpp) filled for the one operand
// form used here, and the MMA, TMEM allocation and commit go through CuTe /
// CUTLASS's sm100 wrappers (SM100_MMA_F8F6F4_SS, TMEM::Allocator1Sm,
// umma_arrive), which issue from one elected lane of a converged warp. Only
// the TMEM loads are written here, so that their wait can name the loaded
// registers (no use can be scheduled before the wait).
//
// Operand form: E4M3 A [128 rows][K] and B [N rows][K], both K-major, each
// 128-byte row of K in shared memory written by a SWIZZLE_128B tensor-map
// load (16-byte chunk c of row r at c ^ (r & 7)), 8-row groups 1024 bytes
// apart, tile bases 1024-byte aligned. One MMA covers K = 32 bytes; the k-th
// slice of a 128-byte row starts 32k bytes in.
#pragma once

#include <stdint.h>

#include <cute/arch/mma_sm100_desc.hpp>
#include <cute/arch/mma_sm100_umma.hpp>
#include <cute/arch/tmem_allocator_sm100.hpp>
#include <cute/numeric/numeric_types.hpp>
#include <cutlass/arch/barrier.h>

#if defined(__CUDA_ARCH__) && \
    (!defined(CUTE_ARCH_TCGEN05_MXF8F6F4_MMA_ENABLED) || !defined(CUTE_ARCH_TCGEN05_TMEM_ENABLED))
#error "tcgen05 kernels must be compiled for sm_100a (compute_100a)"
#endif

namespace drama {

// Shared-memory matrix descriptor of a K-major SWIZZLE_128B E4M3 tile that
// starts at shared address `addr` (1024-byte aligned, or a 32-byte K step
// past such an address).
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t addr) {
    cute::UMMA::SmemDescriptor d;
    d.version_ = 1;                                           // sm_100 descriptor
    d.lbo_mode_ = 0;
    d.layout_type_ = static_cast<uint8_t>(cute::UMMA::LayoutType::SWIZZLE_128B);
    d.base_offset_ = 0;
    d.start_address_ = static_cast<uint16_t>((addr & 0x3FFFFu) >> 4);
    d.leading_byte_offset_ = 1;                               // unused by swizzled K-major tiles
    d.stride_byte_offset_ = 1024 >> 4;                        // 8-row groups 1024 bytes apart
    return static_cast<uint64_t>(d);
}

// Instruction descriptor (upper 32 bits of the runtime form) of an
// M = 128 x N E4M3 x E4M3 -> fp32 MMA, both operands K-major.
template <int N>
__host__ __device__ constexpr uint64_t umma_idesc_e4m3_f32() {
    return cute::UMMA::make_runtime_instr_desc<cute::float_e4m3_t, cute::float_e4m3_t, float, 128, N,
                                               cute::UMMA::Major::K, cute::UMMA::Major::K>();
}

// D[tmem] (+)= A * B^T for one K = 32 slice; call from the whole (converged)
// MMA warp: one elected lane issues it.
__device__ __forceinline__ void umma_e4m3(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint64_t idesc,
                                          bool accumulate) {
    cute::SM100_MMA_F8F6F4_SS::fma(desc_a, desc_b, tmem_d, accumulate ? 1u : 0u, idesc);
}

// The mbarrier at shared address `bar` gets one arrival once every tcgen05
// operation this warp issued so far has completed (whole warp; one lane issues).
__device__ __forceinline__ void umma_commit(uint64_t* bar) { cutlass::arch::umma_arrive(bar); }

// Ordering of tcgen05 operations around thread synchronisation (mbarrier
// waits and arrivals between the MMA warp and the TMEM readers).
__device__ __forceinline__ void tcgen05_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tcgen05_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes (lane i of the
// warp gets lane (addr >> 16) + i); complete only after tmem_wait16.
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr));
}
// Waits for this thread's outstanding TMEM loads; the two register sets are
// named so that no use of them moves above the wait.
__device__ __forceinline__ void tmem_wait2x16(uint32_t (&a)[16], uint32_t (&b)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]),
                   "+r"(a[15]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]),
                   "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]),
                   "+r"(b[14]), "+r"(b[15])
                 :
                 : "memory");
}

// acc = fma(x, s, acc) on a pair of fp32 lanes packed in 64 bits.
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t x, uint64_t s, uint64_t acc) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(x), "l"(s), "l"(acc));
    return d;
}

// Tiled 2-D tensor load (no multicast), as tma_load_3d.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* map, int c0, int c1, uint32_t bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar), "l"(policy)
        : "memory");
}

// Arrival on `bar` once every cp.async this thread issued has landed; the
// barrier's expected count includes this arrival.
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

}  // namespace drama
