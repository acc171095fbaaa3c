// K2 prefill on tcgen05: the FP8 W8A8 expert contract as two grouped GEMMs on
// the 5th-generation tensor cores, accumulators in tensor memory.
//
// Contract: the reference's production GPU backend for many rows
// (TritonExpertBackend.forward_pairs, src/drama_low_vram/offload.py:289-341:
// 1x128 activation quantisation, the grouped FP8 GEMM with 128x128 weight
// block scales, SiLU * up requantised 1x128, the down GEMM times the route
// weight in fp32), with the arithmetic of fp8_decode.py:114-147 and its CPU
// statement native/src/runtime.cpp:162-237:
//   x row -> 1x128 blocks: scale = max(amax, 1e-10) * (1/448), q = e4m3(x / scale)
//   gu[n] = sum over K blocks b of dot_b(W13[n], q) * (xs_b * S13[n/128][b])
//   gate, up = bf16(gu); h = (gate / (1 + exp(-gate))) * up  (fp32), requantised 1x128
//   down[n] = sum over I blocks of dot_b(W2[n], hq) * (hs_b * S2[n/128][b])
//   pair_out = down * route weight (fp32); out[t] = bf16(slot-ordered sum)
// dot_b (128 E4M3 products) runs as four K = 32 tcgen05 MMAs; the addition
// order inside the tensor core is the hardware's. The gate/up epilogue takes
// SiLU with the fast exponential and division intrinsics and requantises h
// by multiplying with the IEEE reciprocal of its block scale (a few ulp from
// the reference's fp32 division; the token rows use the exact division).
//
// Launches, one stream, each after the previous by programmatic dependent
// launch: permute (pairs bucketed by expert, stable, over many CTAs;
// router.cu) -> quantise each token row once into its pairs' sorted rows ->
// gate/up GEMM -> down GEMM -> slot combine.
//
// GEMM CTA (one per SM, persistent, tiles taken with a static stride):
//   tile = (expert, 128 sorted pair rows, 256 output columns); the gate/up
//          tile's columns are 128 gate rows and the matching 128 up rows of
//          W13, the down tile's are 256 rows of W2;
//   warp 0 loads each K block of 128 bytes (A 128 rows, B 256 rows) with
//          SWIZZLE_128B tensor-map copies (no multicast) into a 4-stage ring,
//          and stages each tile's activation and weight scales into shared
//          memory with cp.async early in the previous tile;
//   warp 1 owns 512 TMEM columns (two fp32 accumulators of 256 columns) and
//          issues, per K block, four MMAs into one of them;
//   warps 2-17 load that accumulator (warp w reads lanes 32 (w % 4) ..: the
//          tile row is the TMEM lane; the four warps of a lane quarter split
//          the columns), release it, and promote it into register
//          accumulators with the two block scales; after the last K block
//          they run the tile's epilogue (32-byte row stores).
// Every wait is bounded: on a timeout the CTA sets status[1], stops issuing,
// waits (bounded) for its copies and MMAs in flight and frees its TMEM.
#include <utility>

#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"
#include "umma.cuh"

namespace drama {
namespace {

constexpr int kTcThreads = 576;              // warp 0 TMA, warp 1 MMA, warps 2-17 accumulators
constexpr int kTcStages = 4;
constexpr int kTcM = 128;                     // sorted pair rows per tile
constexpr int kTcN = 256;                     // output columns per tile
constexpr uint32_t kTcA = kTcM * 128;         // A bytes per stage
constexpr uint32_t kTcB = kTcN * 128;         // B bytes per stage
constexpr uint32_t kTcStage = kTcA + kTcB;
constexpr int kTcMaxKb = 16;                  // K blocks of 128 (H, I <= 2048)
constexpr int kTcMaxExperts = 512;
constexpr uint32_t kTmemCols = 512;
constexpr int kTcEpiThreads = 512;
constexpr int kTcGroups = 4;                  // column groups of the accumulator warps

// Shared memory (offsets from the 1024-aligned base).
constexpr uint32_t kOffStages = 0;
constexpr uint32_t kScaleSlot = (kTcMaxKb * kTcM + 2 * kTcMaxKb) * 4;      // activation [kb][row] + 2 weight rows
constexpr uint32_t kOffScales = kOffStages + kTcStages * kTcStage;
constexpr uint32_t kOffAmax = kOffScales + 2 * kScaleSlot;                 // [2 tiles][4 groups][128]
constexpr uint32_t kOffTiles = kOffAmax + 2 * kTcGroups * kTcM * 4;        // first M tile of each expert [E + 1]
constexpr uint32_t kOffRows = kOffTiles + (kTcMaxExperts + 1) * 4;         // first sorted row of each expert [E + 1]
constexpr uint32_t kOffBars = (kOffRows + (kTcMaxExperts + 1) * 4 + 15) & ~15u;
constexpr int kBarFull = 0, kBarEmpty = kTcStages, kBarTFull = 2 * kTcStages, kBarTEmpty = kBarTFull + 2,
              kBarSFull = kBarTEmpty + 2, kBarSEmpty = kBarSFull + 2, kBarAmax = kBarSEmpty + 2,
              kBarDone = kBarAmax + 2, kBarCount = kBarDone + 1;
constexpr uint32_t kOffMisc = kOffBars + kBarCount * 8;                    // TMEM base, abort flag
constexpr uint32_t kTcSmem = kOffMisc + 16 + 1024;                         // + alignment slack

struct TcGemmArgs {
    CUtensorMap a_map;          // [rows][K] E4M3 sorted pair rows (x or h)
    CUtensorMap b_map;          // [slots][N rows][K] E4M3 (W13 or W2)
    const float* a_scale;       // [rows][K/128]
    const float* sorted_w;      // down: route weight of each sorted row [P]
    const float* b_scale;       // [slots][N/128][K/128] (bank strides below)
    int64_t b_scale_slot_stride, b_scale_row_stride;
    const int64_t* offsets;     // [E + 1] first sorted row of each expert
    const int64_t* order;       // [P] sorted row -> pair
    int E, K, I, H;
    uint8_t* hq;                // gate/up: [rows][I] E4M3
    float* hs;                  // gate/up: [rows][I/128]
    const void* weights;        // down: route weights [P]
    int weights_dtype;
    float* pair_out;            // down: [P][H]
    int32_t* status;
};

struct TcTile {
    int e, n0, rows;
    int64_t row0;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Tile t of this GEMM: experts' M tiles in expert order, `nt` column tiles
// of `width` output columns each.
__device__ __forceinline__ TcTile tc_tile(int t, int nt, int width, int E, const int* s_tiles, const int* s_rows) {
    const int m = t / nt;
    int lo = 0, hi = E;  // largest e with s_tiles[e] <= m (experts without rows have equal entries)
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_tiles[mid] <= m) lo = mid;
        else hi = mid;
    }
    TcTile x;
    x.e = lo;
    const int local = m - s_tiles[lo];
    x.row0 = s_rows[lo] + static_cast<int64_t>(local) * kTcM;
    const int end = s_rows[lo + 1];
    x.rows = static_cast<int>(end - x.row0 < kTcM ? end - x.row0 : kTcM);
    x.n0 = (t - m * nt) * width;
    return x;
}

// A wait whose outcome is the same in every lane of the warp (the callers
// then take warp-collective steps: MMA issue, TMEM loads, syncs).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int32_t* flag) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, flag));
}
__device__ __forceinline__ bool warp_aborted(volatile uint32_t* misc) { return __any_sync(0xffffffffu, misc[1] != 0); }

__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ uint64_t splat_f32x2(float s) { return pack_f32x2(s, s); }

// a, b rounded to bf16 (round to nearest even) and widened back to fp32, with
// one paired conversion for the two values.
__device__ __forceinline__ void round_bf16_pair(float& a, float& b) {
    uint32_t p;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(b), "f"(a));  // upper half b, lower half a
    a = __uint_as_float(p << 16);
    b = __uint_as_float(p & 0xffff0000u);
}

// acc[j/2] += (cols j, j+1 of r) * s for 16 columns.
__device__ __forceinline__ void promote16(uint64_t* acc, const uint32_t (&r)[16], uint64_t s) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
        acc[j] = fma_f32x2(pack_f32x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), s, acc[j]);
}

// 32 bytes of one row (a whole L2 sector) from one thread; p 32-byte aligned.
__device__ __forceinline__ void st_global_32b(void* p, uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3, uint32_t v4,
                                              uint32_t v5, uint32_t v6, uint32_t v7) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v0), "r"(v1), "r"(v2), "r"(v3),
                 "r"(v4), "r"(v5), "r"(v6), "r"(v7)
                 : "memory");
}

// The same store with an L2 eviction policy (the down GEMM's fp32 pair rows
// go out evict-first, so they do not push weight and activation rows out of L2).
__device__ __forceinline__ void st_global_32b_hint(void* p, uint64_t policy, uint32_t v0, uint32_t v1, uint32_t v2,
                                                   uint32_t v3, uint32_t v4, uint32_t v5, uint32_t v6, uint32_t v7) {
    asm volatile("st.global.L2::cache_hint.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8}, %9;" ::"l"(p), "r"(v0), "r"(v1),
                 "r"(v2), "r"(v3), "r"(v4), "r"(v5), "r"(v6), "r"(v7), "l"(policy)
                 : "memory");
}

template <int MODE>  // 0: gate/up + SwiGLU + requantise; 1: down * route weight
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ TcGemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment of the shared-window address (the swizzle atom)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
    auto bar = [&](int i) { return sbase + kOffBars + 8u * i; };
    volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc);  // [0] TMEM base [1] abort
    int* s_tiles = reinterpret_cast<int*>(smem + kOffTiles);
    int* s_rows = reinterpret_cast<int*>(smem + kOffRows);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int32_t* timeout_flag = a.status ? a.status + 1 : nullptr;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(bar(kBarFull + s), 1);
            mbar_init(bar(kBarEmpty + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar(kBarTFull + b), 1);
            mbar_init(bar(kBarTEmpty + b), kTcEpiThreads / 32);
            mbar_init(bar(kBarSFull + b), 32);
            mbar_init(bar(kBarSEmpty + b), kTcEpiThreads / 32);
            mbar_init(bar(kBarAmax + b), kTcEpiThreads / 32);
        }
        mbar_init(bar(kBarDone), 1);
        misc[1] = 0;
        fence_mbar_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.a_map)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.b_map)) : "memory");
    }
    if (warp == 1) {
        cute::TMEM::Allocator1Sm alloc;
        alloc.allocate(kTmemCols, const_cast<uint32_t*>(misc));
        alloc.release_allocation_lock();
        tcgen05_before_sync();
    }
    __syncthreads();
    tcgen05_after_sync();
    const uint32_t tmem = misc[0];

    // The sorted rows and expert offsets come from the earlier launches.
    grid_dependency_wait();
    grid_launch_dependents();
    const int E = a.E;
    if (warp == 0) {
        // M tiles per expert, exclusive scan over experts in chunks of 32
        int carry = 0;
        for (int base = 0; base <= E; base += 32) {
            const int e = base + lane;
            int64_t r0 = 0, r1 = 0;
            if (e <= E) r0 = a.offsets[e];
            if (e < E) r1 = a.offsets[e + 1];
            const int mt = e < E ? static_cast<int>((r1 - r0 + kTcM - 1) / kTcM) : 0;
            int x = mt;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, off);
                if (lane >= off) x += y;
            }
            if (e <= E) {
                s_tiles[e] = carry + x - mt;
                s_rows[e] = static_cast<int>(r0);
            }
            carry += __shfl_sync(0xffffffffu, x, 31);
        }
    }
    __syncthreads();
    // gate/up tiles: 128 h columns (128 gate + 128 up rows of W13); down: 256 hidden columns
    const int width = MODE == 0 ? 128 : kTcN;
    const int nt = MODE == 0 ? a.I / 128 : a.H / kTcN;
    const int tiles = s_tiles[E] * nt;
    const int KB = a.K / 128;

    if (warp == 0) {
        // ---------------- producer: TMA ring and tile scales ----------------
        const uint64_t pol_a = policy_evict_last();
        // weight rows: read once for an expert with one row tile, by every
        // row tile otherwise (normal priority then, so they stay in L2)
        const uint64_t pol_b_once = policy_evict_first(), pol_b_shared = policy_evict_normal();
        // Scales of tile t (the it-th of this CTA) into slot it & 1: the
        // activation scales as [kb][row] (kb-major copies, so the lanes of one
        // copy write 32 consecutive rows: distinct banks) and the tile's two
        // weight scale rows; completes on the slot's full barrier.
        auto stage_scales = [&](int t, int it) -> bool {
            const TcTile x = tc_tile(t, nt, width, E, s_tiles, s_rows);
            const int slot = it & 1;
            if (!warp_wait(bar(kBarSEmpty + slot), ((it >> 1) & 1) ^ 1, timeout_flag)) return false;
            const uint32_t sc_addr = sbase + kOffScales + slot * kScaleSlot;
            for (int i = lane; i < kTcM * KB; i += 32) {
                const int kb = i / kTcM, r = i - kb * kTcM;
                cp4(sc_addr + 4u * (kb * kTcM + r), a.a_scale + (x.row0 + r) * KB + kb);
            }
            const float* bs = a.b_scale + x.e * a.b_scale_slot_stride;
            const int nb0 = x.n0 / 128;
            const int nb1 = MODE == 0 ? (a.I + x.n0) / 128 : x.n0 / 128 + 1;
            for (int i = lane; i < 2 * KB; i += 32) {
                const int which = i / KB, kb = i - which * KB;
                cp4(sc_addr + 4u * (kTcMaxKb * kTcM + which * kTcMaxKb + kb),
                    bs + (which ? nb1 : nb0) * a.b_scale_row_stride + kb);
            }
            cp_async_arrive_noinc(bar(kBarSFull + slot));
            return true;
        };
        uint32_t c = 0;  // K blocks issued
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
            const TcTile x = tc_tile(t, nt, width, E, s_tiles, s_rows);
            // this tile's scales were staged during the previous tile (all but the first)
            if (it == 0 && !stage_scales(t, 0)) {
                ok = false;
                break;
            }
            for (int kb = 0; kb < KB; ++kb, ++c) {
                const int s = c % kTcStages;
                if (!warp_wait(bar(kBarEmpty + s), ((c / kTcStages) & 1) ^ 1, timeout_flag) || warp_aborted(misc)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint64_t pol_b = s_tiles[x.e + 1] - s_tiles[x.e] > 1 ? pol_b_shared : pol_b_once;
                    const uint32_t st = sbase + kOffStages + s * kTcStage;
                    mbar_arrive_expect_tx(bar(kBarFull + s), kTcStage);
                    tma_load_2d(st, &a.a_map, kb * 128, static_cast<int>(x.row0), bar(kBarFull + s), pol_a);
                    if (MODE == 0) {
                        tma_load_3d(st + kTcA, &a.b_map, kb * 128, x.n0, x.e, bar(kBarFull + s), pol_b);
                        tma_load_3d(st + kTcA + kTcB / 2, &a.b_map, kb * 128, a.I + x.n0, x.e, bar(kBarFull + s),
                                    pol_b);
                    } else {
                        tma_load_3d(st + kTcA, &a.b_map, kb * 128, x.n0, x.e, bar(kBarFull + s), pol_b);
                    }
                }
                __syncwarp();
                // the next tile's scales, halfway through this one (its slot was
                // released when the tile before this one left the K loop)
                if (kb == KB / 2 && t + static_cast<int>(gridDim.x) < tiles &&
                    !stage_scales(t + gridDim.x, it + 1)) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) misc[1] = 1;
        asm volatile("cp.async.wait_all;" ::: "memory");
        // The last loads of each stage have landed before the CTA exits (the
        // MMA warp waits for every load unless it stopped early).
        for (uint32_t k = c > kTcStages ? c - kTcStages : 0; k < c; ++k)
            mbar_wait(bar(kBarFull + k % kTcStages), (k / kTcStages) & 1, timeout_flag);
    } else if (warp == 1) {
        // ---------------- MMA issue ----------------
        const uint64_t idesc = umma_idesc_e4m3_f32<kTcN>();
        uint32_t c = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < KB; ++kb, ++c) {
                const int s = c % kTcStages, buf = c & 1;
                if (warp_aborted(misc) || !warp_wait(bar(kBarFull + s), (c / kTcStages) & 1, timeout_flag) ||
                    !warp_wait(bar(kBarTEmpty + buf), ((c >> 1) & 1) ^ 1, timeout_flag)) {
                    ok = false;
                    break;
                }
                tcgen05_after_sync();
                const uint32_t st = sbase + kOffStages + s * kTcStage;
                const uint64_t da = umma_desc_k_sw128(st), db = umma_desc_k_sw128(st + kTcA);
                const uint32_t d = tmem + buf * kTcN;
#pragma unroll
                for (int k = 0; k < 4; ++k) umma_e4m3(d, da + 2 * k, db + 2 * k, idesc, k > 0);
                umma_commit(&bars[kBarEmpty + s]);
                umma_commit(&bars[kBarTFull + buf]);
                __syncwarp();
            }
        }
        if (!ok) misc[1] = 1;
        // every MMA issued has completed before TMEM is released
        umma_commit(&bars[kBarDone]);
        __syncwarp();
        mbar_wait(bar(kBarDone), 0, timeout_flag);
    } else {
        // ---------------- accumulator warps ----------------
        // lane quarter q, column group g: MODE 0 gate columns [32g, 32g + 32)
        // and the matching up columns 128 + [32g, 32g + 32) (h columns
        // [32g, 32g + 32) of the tile); MODE 1 columns [64g, 64g + 64).
        const int q = warp & 3, g = (warp - 2) >> 2, r = q * 32 + lane;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const uint32_t c0 = MODE == 0 ? 32 * g : 64 * g;
        const uint32_t c1 = MODE == 0 ? 128 + 32 * g : 64 * g + 32;
        float* amax = reinterpret_cast<float*>(smem + kOffAmax);
        uint32_t c = 0;
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
            const TcTile x = tc_tile(t, nt, width, E, s_tiles, s_rows);
            const int slot = it & 1;
            if (warp_aborted(misc) || !warp_wait(bar(kBarSFull + slot), (it >> 1) & 1, timeout_flag)) {
                ok = false;
                break;
            }
            const float* sc = reinterpret_cast<const float*>(smem + kOffScales + slot * kScaleSlot);
            int64_t pair = 0;
            float route_w = 0.0f;
            if (MODE == 1 && r < x.rows) {
                // both independent of each other: neither load holds the K loop
                pair = a.order[x.row0 + r];
                route_w = a.sorted_w[x.row0 + r];
            }
            uint64_t acc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0ull;
            for (int kb = 0; kb < KB; ++kb, ++c) {
                const int buf = c & 1;
                if (!warp_wait(bar(kBarTFull + buf), (c >> 1) & 1, timeout_flag)) {
                    ok = false;
                    break;
                }
                tcgen05_after_sync();
                const uint32_t base = lane_addr + buf * kTcN;
                uint32_t ra[16], rb[16];
                tmem_ld16(base + c0, ra);
                tmem_ld16(base + c0 + 16, rb);
                const float sa = sc[kb * kTcM + r];
                const float* sw = sc + kTcMaxKb * kTcM;
                const uint64_t s0 = splat_f32x2(__fmul_rn(sa, MODE == 0 ? sw[kb] : sw[(g >> 1) * kTcMaxKb + kb]));
                const uint64_t s1 = MODE == 0 ? splat_f32x2(__fmul_rn(sa, sw[kTcMaxKb + kb])) : s0;
                tmem_wait2x16(ra, rb);
                promote16(acc, ra, s0);
                promote16(acc + 8, rb, s0);
                tmem_ld16(base + c1, ra);
                tmem_ld16(base + c1 + 16, rb);
                tmem_wait2x16(ra, rb);
                tcgen05_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarTEmpty + buf));
                promote16(acc + 16, ra, s1);
                promote16(acc + 24, rb, s1);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarSEmpty + slot));
            if (!ok) break;
            if (MODE == 0) {
                // acc[0..15]: gate columns, acc[16..31]: the matching up columns
                float hv[32];
                float m = 0.0f;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    float g0, g1, u0, u1;
                    unpack_f32x2(acc[j], g0, g1);
                    unpack_f32x2(acc[16 + j], u0, u1);
                    round_bf16_pair(g0, g1);  // gate and up as the bf16 rows of the reference
                    round_bf16_pair(u0, u1);
                    hv[2 * j] = __fmul_rn(__fdividef(g0, __fadd_rn(1.0f, __expf(-g0))), u0);
                    hv[2 * j + 1] = __fmul_rn(__fdividef(g1, __fadd_rn(1.0f, __expf(-g1))), u1);
                    m = fmaxf(m, fmaxf(fabsf(hv[2 * j]), fabsf(hv[2 * j + 1])));
                }
                // the row's other 96 h columns of the 1x128 block are in the other groups' threads
                float* am = amax + slot * kTcGroups * kTcM;
                am[g * kTcM + r] = m;
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarAmax + slot));
                if (!warp_wait(bar(kBarAmax + slot), (it >> 1) & 1, timeout_flag)) {
                    ok = false;
                    break;
                }
                const float row_max =
                    fmaxf(fmaxf(fmaxf(am[r], am[kTcM + r]), fmaxf(am[2 * kTcM + r], am[3 * kTcM + r])), 1e-10f);
                const float scale = __fmul_rn(row_max, 1.0f / 448.0f);
                const float inv = __frcp_rn(scale);
                if (r < x.rows) {
                    const int64_t row = x.row0 + r;
                    uint32_t w[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        w[u] = e4m3x2(__fmul_rn(hv[4 * u], inv), __fmul_rn(hv[4 * u + 1], inv)) |
                               (e4m3x2(__fmul_rn(hv[4 * u + 2], inv), __fmul_rn(hv[4 * u + 3], inv)) << 16);
                    st_global_32b(a.hq + row * a.I + x.n0 + 32 * g, w[0], w[1], w[2], w[3], w[4], w[5], w[6], w[7]);
                    if (g == 0) a.hs[row * (a.I / 128) + x.n0 / 128] = scale;
                }
            } else if (r < x.rows) {
                const uint64_t pol_out = policy_evict_first();
                float* dst = a.pair_out + pair * a.H + x.n0 + 64 * g;
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    float f[8];
#pragma unroll
                    for (int u = 0; u < 4; ++u) unpack_f32x2(acc[4 * v + u], f[2 * u], f[2 * u + 1]);
                    st_global_32b_hint(dst + 8 * v, pol_out, __float_as_uint(__fmul_rn(f[0], route_w)),
                                       __float_as_uint(__fmul_rn(f[1], route_w)),
                                       __float_as_uint(__fmul_rn(f[2], route_w)),
                                       __float_as_uint(__fmul_rn(f[3], route_w)),
                                       __float_as_uint(__fmul_rn(f[4], route_w)),
                                       __float_as_uint(__fmul_rn(f[5], route_w)),
                                       __float_as_uint(__fmul_rn(f[6], route_w)),
                                       __float_as_uint(__fmul_rn(f[7], route_w)));
                }
            }
        }
        if (!ok) misc[1] = 1;
    }
    tcgen05_before_sync();
    __syncthreads();
    if (warp == 1) {
        tcgen05_after_sync();
        cute::TMEM::Allocator1Sm().free(tmem, kTmemCols);
    }
}

// One token row per CTA: its 1x128 blocks quantised once (half a warp per
// block, 8 values per lane) and written to the sorted position of each of
// the token's pairs, with each pair's route weight (fp32) at its position.
__global__ void __launch_bounds__(256) tc_quant_tokens_kernel(const __nv_bfloat16* x, int H, int top_k,
                                                              const int64_t* position, const void* weights,
                                                              int weights_dtype, uint8_t* xq, float* xs,
                                                              float* sorted_w) {
    __shared__ int64_t s_pos[32];
    grid_dependency_wait();
    grid_launch_dependents();
    const int64_t token = blockIdx.x;
    if (threadIdx.x < top_k) {
        const int64_t p = token * top_k + threadIdx.x;
        const int64_t r = position[p];
        s_pos[threadIdx.x] = r;
        if (r >= 0) sorted_w[r] = load_any(weights, weights_dtype, p);
    }
    __syncthreads();
    const int hw = threadIdx.x >> 4, l = threadIdx.x & 15, nblk = H / 128;
    for (int base = 0; base < nblk; base += 16) {
        const int blk = base + hw;
        const bool on = blk < nblk;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (on) v = __ldg(reinterpret_cast<const uint4*>(x + token * H + blk * 128 + l * 8));
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = bf16_at(v, j);
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(f[j]));
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        const float scale = __fmul_rn(fmaxf(m, 1e-10f), 1.0f / 448.0f);
        if (!on) continue;
        uint2 q;
        q.x = e4m3x2(__fdiv_rn(f[0], scale), __fdiv_rn(f[1], scale)) |
              (e4m3x2(__fdiv_rn(f[2], scale), __fdiv_rn(f[3], scale)) << 16);
        q.y = e4m3x2(__fdiv_rn(f[4], scale), __fdiv_rn(f[5], scale)) |
              (e4m3x2(__fdiv_rn(f[6], scale), __fdiv_rn(f[7], scale)) << 16);
        for (int s = 0; s < top_k; ++s) {
            const int64_t r = s_pos[s];
            if (r < 0) continue;
            *reinterpret_cast<uint2*>(xq + r * H + blk * 128 + l * 8) = q;
            if (l == 0) xs[r * nblk + blk] = scale;
        }
    }
}

// out[t][c..c+3] = bf16(sum over slots, in slot order, of pair_out); a pair
// whose expert id is out of range contributes zero and, when its row is
// returned to the caller, has that row zeroed.
__global__ void tc_combine_kernel(float* pair_out, const void* ids, int ids_dtype, int experts, int64_t tokens,
                                  int top_k, int H, bool zero_dropped, __nv_bfloat16* out) {
    grid_dependency_wait();
    const int64_t n = tokens * (H / 4);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / (H / 4);
        const int c = static_cast<int>(i - t * (H / 4)) * 4;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int s = 0; s < top_k; ++s) {
            const int64_t p = t * top_k + s;
            const int64_t id = load_index(ids, ids_dtype, p);
            float4* row = reinterpret_cast<float4*>(pair_out + p * H + c);
            if (id < 0 || id >= experts) {
                if (zero_dropped) *row = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                continue;
            }
            const float4 v = *row;
            acc[0] = __fadd_rn(acc[0], v.x);
            acc[1] = __fadd_rn(acc[1], v.y);
            acc[2] = __fadd_rn(acc[2], v.z);
            acc[3] = __fadd_rn(acc[3], v.w);
        }
        if (out) {
            const __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0], acc[1]);
            const __nv_bfloat162 hi = __floats2bfloat162_rn(acc[2], acc[3]);
            uint2 o;
            o.x = *reinterpret_cast<const uint32_t*>(&lo);
            o.y = *reinterpret_cast<const uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(out + t * H + c) = o;
        }
    }
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_smem(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args&&... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

bool encode_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_stride,
               uint32_t box_rows) {
    const TensorMapEncode encode = tensor_map_encoder();
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_stride};
    const cuuint32_t box[2] = {128, box_rows};
    const cuuint32_t unit[2] = {1, 1};
    return encode && encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, unit,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t slots, uint64_t row_stride,
               uint64_t slot_stride, uint32_t box_rows) {
    const TensorMapEncode encode = tensor_map_encoder();
    const cuuint64_t dims[3] = {cols, rows, slots};
    const cuuint64_t strides[2] = {row_stride, slot_stride};
    const cuuint32_t box[3] = {128, box_rows, 1};
    const cuuint32_t unit[3] = {1, 1, 1};
    return encode && encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, unit,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool fp8_prefill_tc_supported(int hidden, int intermediate, int experts) {
    return tensor_map_encoder() != nullptr && hidden % kTcN == 0 && intermediate % 128 == 0 &&
           hidden / 128 <= kTcMaxKb && intermediate / 128 <= kTcMaxKb && experts >= 1 &&
           experts <= kTcMaxExperts;
}

size_t fp8_prefill_tc_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, int experts,
                                       char* base, Fp8PrefillWorkspace* ws) {
    const int64_t P = tokens * top_k;
    const int64_t rows = P + kTcM;  // tiles may read up to 127 rows past the last pair
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += (bytes + 1023) & ~static_cast<size_t>(1023);
        return p;
    };
    Fp8PrefillWorkspace w{};
    w.status = reinterpret_cast<int32_t*>(take(16));
    w.order = reinterpret_cast<int64_t*>(take(P * 8));
    w.counts = reinterpret_cast<int64_t*>(take(static_cast<size_t>(experts) * 8));
    w.offsets = reinterpret_cast<int64_t*>(take(static_cast<size_t>(experts + 1) * 8));
    w.position = reinterpret_cast<int64_t*>(take(P * 8));
    w.sorted_w = reinterpret_cast<float*>(take(P * 4));
    w.chunk_counts = reinterpret_cast<int*>(take(permute_wide_scratch_bytes(P, experts)));
    w.xq = reinterpret_cast<uint8_t*>(take(rows * hidden));
    w.xs = reinterpret_cast<float*>(take(rows * (hidden / 128) * 4));
    w.hq = reinterpret_cast<uint8_t*>(take(rows * intermediate));
    w.hs = reinterpret_cast<float*>(take(rows * (intermediate / 128) * 4));
    w.pair_out = reinterpret_cast<float*>(take(P * hidden * 4));
    if (ws) *ws = w;
    return off;
}

cudaError_t fp8_prefill_tc_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t tokens, int top_k,
                                  const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                                  float* pair_out, const Fp8PrefillWorkspace& ws, int sm_count, cudaStream_t s) {
    static bool configured = false;  // benign race: identical values
    if (!configured) {
        cudaError_t err = cudaFuncSetAttribute(tc_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kTcSmem));
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(tc_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kTcSmem));
        if (err != cudaSuccess) return err;
        configured = true;
    }
    const int H = bank.hidden, I = bank.intermediate, E = bank.slots;
    const int64_t P = tokens * top_k;
    const int64_t rows = P + kTcM;
    float* pairs = pair_out ? pair_out : ws.pair_out;
    cudaError_t err = cudaMemsetAsync(ws.status, 0, 16, s);
    if (err != cudaSuccess) return err;
    PermuteArgs pa{ids, ids_dtype, P, E, ws.order, ws.counts, ws.offsets, ws.status};
    if ((err = permute_routes_wide(pa, ws.chunk_counts, ws.position, s)) != cudaSuccess) return err;
    if ((err = launch_pdl_smem(tc_quant_tokens_kernel, dim3(static_cast<unsigned>(tokens)), dim3(256), 0, s,
                               static_cast<const __nv_bfloat16*>(x), H, top_k,
                               static_cast<const int64_t*>(ws.position), weights, weights_dtype, ws.xq, ws.xs,
                               ws.sorted_w)) != cudaSuccess)
        return err;
    TcGemmArgs g{};
    g.offsets = ws.offsets;
    g.order = ws.order;
    g.sorted_w = ws.sorted_w;
    g.E = E;
    g.I = I;
    g.H = H;
    g.hq = ws.hq;
    g.hs = ws.hs;
    g.weights = weights;
    g.weights_dtype = weights_dtype;
    g.pair_out = pairs;
    g.status = ws.status;
    // gate/up: A = sorted x rows [rows][H], B = W13 [slots][2I][H]
    g.K = H;
    g.a_scale = ws.xs;
    g.b_scale = bank.w13_scale;
    g.b_scale_slot_stride = bank.w13_scale_slot_stride;
    g.b_scale_row_stride = bank.w13_scale_row_stride;
    if (!encode_2d(&g.a_map, ws.xq, H, rows, H, kTcM) ||
        !encode_3d(&g.b_map, bank.w13, H, 2 * static_cast<uint64_t>(I), E, bank.w13_row_stride,
                   bank.w13_slot_stride, kTcM))
        return cudaErrorInvalidValue;
    if ((err = launch_pdl_smem(tc_gemm_kernel<0>, dim3(sm_count), dim3(kTcThreads), kTcSmem, s, g)) != cudaSuccess)
        return err;
    // down: A = sorted h rows [rows][I], B = W2 [slots][H][I]
    g.K = I;
    g.a_scale = ws.hs;
    g.b_scale = bank.w2_scale;
    g.b_scale_slot_stride = bank.w2_scale_slot_stride;
    g.b_scale_row_stride = bank.w2_scale_row_stride;
    if (!encode_2d(&g.a_map, ws.hq, I, rows, I, kTcM) ||
        !encode_3d(&g.b_map, bank.w2, I, H, E, bank.w2_row_stride, bank.w2_slot_stride, kTcN))
        return cudaErrorInvalidValue;
    if ((err = launch_pdl_smem(tc_gemm_kernel<1>, dim3(sm_count), dim3(kTcThreads), kTcSmem, s, g)) != cudaSuccess)
        return err;
    const int64_t chunks = tokens * (H / 4);
    const int blocks = static_cast<int>(chunks / 256 + 1 < sm_count * 8 ? chunks / 256 + 1 : sm_count * 8);
    return launch_pdl_smem(tc_combine_kernel, dim3(blocks), dim3(256), 0, s, pairs, ids, ids_dtype, E, tokens, top_k,
                           H, pair_out != nullptr, static_cast<__nv_bfloat16*>(out));
}

}  // namespace drama
