// Device building blocks of the K1 expert GEMVs (shared by the per-layer
// kernels in expert_decode.cu and the persistent stack kernel).
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace drama {

namespace {


__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ uint32_t sub_f16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Two nibbles (m, m+4) of an 8-nibble word -> f16x2 {1024+n_m, 1024+n_{m+4}}.
__device__ __forceinline__ uint32_t nibbles_to_f16x2_biased(uint32_t w) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w), "r"(0x000F000Fu), "r"(0x64006400u));
    return d;
}

// Four E4M3 bytes -> two f16x2 (bytes 0,1 -> lo; bytes 2,3 -> hi), exact.
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}

__device__ __forceinline__ uint32_t comp(const uint4& q, int i) {
    return i == 0 ? q.x : i == 1 ? q.y : i == 2 ? q.z : q.w;
}

__device__ __forceinline__ float load_scale16(const void* p, int dtype, int64_t i) {
    return dtype == DRAMA_B200_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i])
                                    : __half2float(static_cast<const __half*>(p)[i]);
}

struct GroupRec {
    int id, slot, start, count;
    uint32_t tok[4];
};

__device__ __forceinline__ void load_group(GroupRec& r, int id, const DecodeWorkspace& ws) {
    if (r.id == id) return;
    const int4 a = __ldcg(ws.g_rec + 2 * id);
    const int4 b = __ldcg(ws.g_rec + 2 * id + 1);
    r.id = id;
    r.slot = a.x;
    r.start = a.y;
    r.count = a.z;
    r.tok[0] = static_cast<uint32_t>(b.x);
    r.tok[1] = static_cast<uint32_t>(b.y);
    r.tok[2] = static_cast<uint32_t>(b.z);
    r.tok[3] = static_cast<uint32_t>(b.w);
}

__device__ __forceinline__ int rec_pair(const GroupRec& r, int col) {
    const int i = col >> 1;  // select, not an indexed load: keeps tok[] in registers
    const uint32_t w = i == 0 ? r.tok[0] : i == 1 ? r.tok[1] : i == 2 ? r.tok[2] : r.tok[3];
    return static_cast<int>((w >> (16 * (col & 1))) & 0xffffu);
}

// Even partition: worker w owns cells [w*q, min(cells, (w+1)*q)).
struct Partition {
    int cells, q, workers;
};
__device__ __forceinline__ Partition make_partition(int cells, int max_workers, int unit) {
    Partition p;
    p.cells = cells;
    const int q = cells > 0 ? (cells + max_workers - 1) / max_workers : 1;
    p.q = (q + unit - 1) / unit * unit;
    p.workers = cells > 0 ? (cells + p.q - 1) / p.q : 0;
    return p;
}

// Eight consecutive elements starting at a multiple of 8.
__device__ __forceinline__ void load8(const void* base, int dtype, int64_t i, float (&v)[8]) {
    if (dtype == DRAMA_B200_F32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
        const float4 a = __ldg(p), b = __ldg(p + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + i));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (dtype == DRAMA_B200_BF16) {
                v[2 * j] = __uint_as_float(w[j] << 16);
                v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
            } else {
                v[2 * j] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[j] & 0xffffu)));
                v[2 * j + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(w[j] >> 16)));
            }
        }
    }
}

// Pack 8 floats (scaled) as 4 f16x2 words in the format's B-fragment order:
// natural for FP8; nibble-pair order [0,4,1,5,2,6,3,7] for INT4.
template <int FMT>
__device__ __forceinline__ uint4 pack8(const float (&v)[8], float sc) {
    uint4 o;
    if (FMT == 1) {
        o.x = pack_f16x2(v[0] * sc, v[4] * sc);
        o.y = pack_f16x2(v[1] * sc, v[5] * sc);
        o.z = pack_f16x2(v[2] * sc, v[6] * sc);
        o.w = pack_f16x2(v[3] * sc, v[7] * sc);
    } else {
        o.x = pack_f16x2(v[0] * sc, v[1] * sc);
        o.y = pack_f16x2(v[2] * sc, v[3] * sc);
        o.z = pack_f16x2(v[4] * sc, v[5] * sc);
        o.w = pack_f16x2(v[6] * sc, v[7] * sc);
    }
    return o;
}

// ---------------------------------------------------------------------------
// Split-K bookkeeping: a tile's K-cells are spread over consecutive workers;
// every contributor but a sole one writes its fragment partial, and the last
// to arrive sums them in worker (= K) order. Returns true when this warp
// must finalise `tile` with `acc` (now the full sum).
// ---------------------------------------------------------------------------
template <int NV>
__device__ __forceinline__ bool tile_flush(float (&acc)[NV], int tile, int kb_per_tile, const Partition& pt,
                                           int w, float* part, int32_t* cnt, int lane) {
    const int first = tile * kb_per_tile;
    const int wf = first / pt.q;
    const int wl = (first + kb_per_tile - 1) / pt.q;
    if (wf == wl) return true;
    const int which = (tile == (w * pt.q) / kb_per_tile) ? 0 : 1;
    float* dst = part + ((static_cast<int64_t>(w) * 2 + which) * 32 + lane) * NV;
#pragma unroll
    for (int i = 0; i < NV; i += 4)
        __stcg(reinterpret_cast<float4*>(dst + i), make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]));
    __syncwarp();
    int old = 0;
    if (lane == 0) {
        fence_acq_rel_gpu();
        old = atomicAdd(cnt + tile, 1);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != wl - wf) return false;
    fence_acq_rel_gpu();
#pragma unroll
    for (int i = 0; i < NV; ++i) acc[i] = 0.0f;
    for (int v0 = wf; v0 <= wl; v0 += 4) {
        float4 q[4][NV / 4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int v = v0 + j;
            if (v <= wl) {
                const int wh = (tile == (v * pt.q) / kb_per_tile) ? 0 : 1;
                const float4* src = reinterpret_cast<const float4*>(
                    part + ((static_cast<int64_t>(v) * 2 + wh) * 32 + lane) * NV);
#pragma unroll
                for (int i = 0; i < NV / 4; ++i) q[j][i] = __ldcg(src + i);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (v0 + j <= wl) {
#pragma unroll
                for (int i = 0; i < NV / 4; ++i) {
                    acc[4 * i] += q[j][i].x;
                    acc[4 * i + 1] += q[j][i].y;
                    acc[4 * i + 2] += q[j][i].z;
                    acc[4 * i + 3] += q[j][i].w;
                }
            }
        }
    }
    return true;
}

// ---------------------------------------------------------------------------
// Asynchronous global -> shared copies (16 bytes per lane, no registers held).
// Each warp owns a private ring of DEPTH stages; stage data is laid out
// [chunk][lane] so that every 16-byte shared access of a warp is conflict-free.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, uint64_t pol) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
                 : "memory");
}
// Zero-fills 16 bytes; no global byte is read.
__device__ __forceinline__ void cp16_zero(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, 0;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kRingBudget = 192 * 1024;  // shared memory for one CTA's warp rings
constexpr int kXReserve = 32 * 1024;     // up kernel: staged activation rows (T * H * 2 bytes)

// Per-kernel geometry: chunks of 16 bytes per lane per cell (NCH), warps per
// CTA, ring depth, and the partition unit (a warp's cell range is a multiple
// of UNIT cells; UNIT = cells per tile means no tile is split between warps).
template <int FMT>
struct UpShape {
    static constexpr int NCH = FMT == 0 ? 8 : 4;
    static constexpr int WARPS = FMT == 0 ? 6 : 6;
    static constexpr int DEPTH = kRingBudget / (WARPS * NCH * 512);  // 8 (FP8) / 16 (INT4)
    static constexpr int UNIT_DIV = FMT == 0 ? 2 : 1;                // FP8: half tiles
};
template <int FMT, int XDT>
struct DnShape {
    static constexpr int NW = FMT == 0 ? 4 : 2;               // weight chunks
    static constexpr int NH = XDT == DRAMA_B200_F32 ? 8 : 4;  // activation chunks
    static constexpr int NCH = NW + NH;
    static constexpr int WARPS = kRingBudget / (6 * NCH * 512) > 16 ? 16 : kRingBudget / (6 * NCH * 512);
    static constexpr int DEPTH = 6;  // one 768-wide tile per warp at I = 768
    static constexpr int UNIT_DIV = 1;
};

struct CellIt {
    int grp, jt, kb;
};
__device__ __forceinline__ CellIt cell_at(int c, int KB, int TILES) {
    const int tile = c / KB;
    return {tile / TILES, tile % TILES, c % KB};
}
__device__ __forceinline__ void advance(CellIt& it, int KB, int TILES) {
    if (++it.kb == KB) {
        it.kb = 0;
        if (++it.jt == TILES) {
            it.jt = 0;
            ++it.grp;
        }
    }
}

// Static partition for single-token calls (the group count is at most top_k
// and need not be read before the first loads), dynamic otherwise.
struct Work {
    Partition pt;
    int c0, c1, groups;
};
__device__ __forceinline__ Work plan_work(const DecodeArgs& a, int tiles, int kb, int max_workers, int unit, int w,
                                          GroupRec& first) {
    Work r;
    const bool single = a.tokens == 1;
    if (single) {
        r.pt = make_partition(a.top_k * tiles * kb, max_workers, unit);
        r.c0 = w < r.pt.workers ? w * r.pt.q : 0;
        r.c1 = w < r.pt.workers ? min(r.pt.cells, r.c0 + r.pt.q) : 0;
        if (r.c0 < r.c1) load_group(first, r.c0 / (tiles * kb), a.ws);  // in flight with num_groups
        r.groups = __ldcg(a.ws.num_groups);
        r.c1 = min(r.c1, r.groups * tiles * kb);
    } else {
        r.groups = __ldcg(a.ws.num_groups);
        r.pt = make_partition(r.groups * tiles * kb, max_workers, unit);
        r.c0 = w < r.pt.workers ? w * r.pt.q : 0;
        r.c1 = w < r.pt.workers ? min(r.pt.cells, r.c0 + r.pt.q) : 0;
    }
    if (r.c0 >= r.c1) r.c0 = r.c1 = 0;
    return r;
}

// ---------------------------------------------------------------------------
// up: gate/up GEMV + SiLU*mul
// ---------------------------------------------------------------------------
template <int FMT>
__device__ __forceinline__ void up_issue(uint32_t dst, const DecodeArgs& a, int slot, const CellIt& it, int g, int t,
                                         uint64_t pol) {
    const int I = a.intermediate;
    if (FMT == 0) {
        const DramaB200Fp8Bank& b = a.fp8;
        // Lane t copies bytes [16t, 16t+16) and [64+16t, 64+16t+16) of a
        // row's 128-byte block: the four lanes of a row cover whole sectors.
        const uint8_t* base = static_cast<const uint8_t*>(b.w13) + slot * b.w13_slot_stride +
                              static_cast<int64_t>(it.jt * 16 + g) * b.w13_row_stride + it.kb * 128 + 16 * t;
        const int64_t r8 = 8 * b.w13_row_stride, ru = static_cast<int64_t>(I) * b.w13_row_stride;
        cp16(dst + 0 * 512, base, pol);
        cp16(dst + 1 * 512, base + 64, pol);
        cp16(dst + 2 * 512, base + r8, pol);
        cp16(dst + 3 * 512, base + r8 + 64, pol);
        cp16(dst + 4 * 512, base + ru, pol);
        cp16(dst + 5 * 512, base + ru + 64, pol);
        cp16(dst + 6 * 512, base + ru + r8, pol);
        cp16(dst + 7 * 512, base + ru + r8 + 64, pol);
    } else {
        const DramaB200Int4Bank& b = a.int4;
        const int32_t* base = b.w13 + slot * b.w13_slot_stride +
                              static_cast<int64_t>(it.jt * 16 + g) * b.w13_row_stride + it.kb * 16 + 4 * t;
        const int64_t r8 = 8 * b.w13_row_stride, ru = static_cast<int64_t>(I) * b.w13_row_stride;
        cp16(dst + 0 * 512, base, pol);
        cp16(dst + 1 * 512, base + r8, pol);
        cp16(dst + 2 * 512, base + ru, pol);
        cp16(dst + 3 * 512, base + ru + r8, pol);
    }
}

// FP8 gate/up cell with its two 128x128 block scales already in hand (gate
// rows' scale sg, up rows' scale su): 16 rows x 128 K of each projection
// against the B fragments xb, block sums scaled and added to tot in fp32.
__device__ __forceinline__ void up_mma_fp8_scaled(const uint4 (&q)[8], float sg, float su, const uint32_t (&xb)[16],
                                                  float (&tot)[8]) {
    float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int qi = s >> 2, ci = s & 3;
        uint32_t A[4], B[4];
        e4m3x4_to_f16x2x2(comp(q[qi], ci), A[0], A[2]);
        e4m3x4_to_f16x2x2(comp(q[2 + qi], ci), A[1], A[3]);
        mma_f16_16816(ag, A, xb[2 * s], xb[2 * s + 1]);
        e4m3x4_to_f16x2x2(comp(q[4 + qi], ci), B[0], B[2]);
        e4m3x4_to_f16x2x2(comp(q[6 + qi], ci), B[1], B[3]);
        mma_f16_16816(au, B, xb[2 * s], xb[2 * s + 1]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        tot[i] = fmaf(ag[i], sg, tot[i]);
        tot[4 + i] = fmaf(au[i], su, tot[4 + i]);
    }
}

template <int FMT>
__device__ __forceinline__ void up_mma(const uint4 (&q)[UpShape<FMT>::NCH], const DecodeArgs& a, int slot,
                                       const CellIt& it, int g, const uint32_t (&xb)[16], float (&tot)[8]) {
    float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
    const int I = a.intermediate;
    if constexpr (FMT == 0) {
        const DramaB200Fp8Bank& b = a.fp8;
        const float* sp = b.w13_scale + slot * b.w13_scale_slot_stride + it.kb;
        const float sg = __ldg(sp + ((it.jt * 16) >> 7) * b.w13_scale_row_stride);
        const float su = __ldg(sp + ((I + it.jt * 16) >> 7) * b.w13_scale_row_stride);
        up_mma_fp8_scaled(q, sg, su, xb, tot);
    } else {
        const DramaB200Int4Bank& b = a.int4;
        const int rows[4] = {it.jt * 16 + g, it.jt * 16 + g + 8, I + it.jt * 16 + g, I + it.jt * 16 + g + 8};
        float sc[4];
        uint32_t zc[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            sc[r] = load_scale16(b.w13_scale, b.scale_dtype,
                                 slot * b.w13_scale_slot_stride + rows[r] * b.w13_scale_row_stride + it.kb);
            uint32_t z = 8;
            if (b.w13_zeros) {
                const uint32_t word = static_cast<uint32_t>(__ldg(
                    b.w13_zeros + slot * b.w13_zeros_slot_stride + (rows[r] >> 3) * b.w13_zeros_row_stride + it.kb));
                z = (word >> (4 * (rows[r] & 7))) & 15u;
            }
            zc[r] = (0x6400u + z) * 0x10001u;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wg = comp(q[0], i), wg8 = comp(q[1], i);
            const uint32_t wu = comp(q[2], i), wu8 = comp(q[3], i);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int s = 2 * i + h;
                const uint32_t A[4] = {sub_f16x2(nibbles_to_f16x2_biased(wg >> (8 * h)), zc[0]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wg8 >> (8 * h)), zc[1]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wg >> (8 * h + 4)), zc[0]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wg8 >> (8 * h + 4)), zc[1])};
                mma_f16_16816(ag, A, xb[2 * s], xb[2 * s + 1]);
                const uint32_t B[4] = {sub_f16x2(nibbles_to_f16x2_biased(wu >> (8 * h)), zc[2]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wu8 >> (8 * h)), zc[3]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wu >> (8 * h + 4)), zc[2]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wu8 >> (8 * h + 4)), zc[3])};
                mma_f16_16816(au, B, xb[2 * s], xb[2 * s + 1]);
            }
        }
        tot[0] = fmaf(ag[0], sc[0], tot[0]);
        tot[1] = fmaf(ag[1], sc[0], tot[1]);
        tot[2] = fmaf(ag[2], sc[1], tot[2]);
        tot[3] = fmaf(ag[3], sc[1], tot[3]);
        tot[4] = fmaf(au[0], sc[2], tot[4]);
        tot[5] = fmaf(au[1], sc[2], tot[5]);
        tot[6] = fmaf(au[2], sc[3], tot[6]);
        tot[7] = fmaf(au[3], sc[3], tot[7]);
    }
}

template <int XDT>
__device__ __forceinline__ void up_finalize(const DecodeArgs& a, const GroupRec& gi, int jt, const float (&acc)[8],
                                            int g, int t) {
    using T = typename Scalar<XDT>::T;
    const int I = a.intermediate;
    T* h = static_cast<T*>(a.ws.h);
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int col = 2 * t + cc;
        if (col >= gi.count) continue;
        const int pair = rec_pair(gi, col);
        const float xs = __ldcg(a.ws.xscale + pair / a.top_k);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float gate = Scalar<XDT>::round(acc[r * 2 + cc] * xs);
            const float up = Scalar<XDT>::round(acc[4 + r * 2 + cc] * xs);
            const float act = Scalar<XDT>::round(gate / (1.0f + expf(-gate)));
            h[static_cast<int64_t>(pair) * I + jt * 16 + g + 8 * r] = Scalar<XDT>::from(act * up);
        }
    }
}

// Every CTA issues its share (item i goes to CTA i % grid): a kernel does not
// complete before its bulk prefetches land, and each SM's copy engine serves
// only its own CTAs' requests, so the prefetch must be spread over all SMs.
__device__ __forceinline__ void prefetch_down_slabs(const DecodeArgs& a, int groups) {
    const int tiles = a.hidden / 16;
    const int items = groups * tiles;
    GroupRec r{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
    for (int it = blockIdx.x + gridDim.x * threadIdx.x; it < items; it += gridDim.x * blockDim.x) {
        load_group(r, it / tiles, a.ws);
        const int nt = it % tiles;
        const char* base;
        int64_t row_bytes, stride_bytes;
        if (a.format == 0) {
            base = static_cast<const char*>(a.fp8.w2) + r.slot * a.fp8.w2_slot_stride +
                   static_cast<int64_t>(nt) * 16 * a.fp8.w2_row_stride;
            row_bytes = a.intermediate;
            stride_bytes = a.fp8.w2_row_stride;
        } else {
            base = reinterpret_cast<const char*>(a.int4.w2 + r.slot * a.int4.w2_slot_stride +
                                                 static_cast<int64_t>(nt) * 16 * a.int4.w2_row_stride);
            row_bytes = a.intermediate / 2;
            stride_bytes = a.int4.w2_row_stride * 4;
        }
        if (stride_bytes == row_bytes) {
            prefetch_l2_bulk(base, static_cast<uint32_t>(16 * row_bytes));
        } else {
            for (int rr = 0; rr < 16; ++rr)
                prefetch_l2_bulk(base + rr * stride_bytes, static_cast<uint32_t>(row_bytes));
        }
    }
}

// ---------------------------------------------------------------------------
// down: W2 GEMV + route weight + slot combine. The activations h arrive with
// the weights; each 128-wide block of a column is scaled to f16 by the power
// of two of its own maximum (exact for bf16/f16 h), undone in fp32.
// ---------------------------------------------------------------------------
template <int FMT, int XDT>
__device__ __forceinline__ void dn_issue(uint32_t dst, const DecodeArgs& a, const GroupRec& rec, const CellIt& it,
                                         int g, int t, uint64_t pol) {
    using S = DnShape<FMT, XDT>;
    using T = typename Scalar<XDT>::T;
    if (FMT == 0) {
        const DramaB200Fp8Bank& b = a.fp8;
        const uint8_t* base = static_cast<const uint8_t*>(b.w2) + rec.slot * b.w2_slot_stride +
                              static_cast<int64_t>(it.jt * 16 + g) * b.w2_row_stride + it.kb * 128 + 16 * t;
        const int64_t r8 = 8 * b.w2_row_stride;
        cp16(dst + 0 * 512, base, pol);
        cp16(dst + 1 * 512, base + 64, pol);
        cp16(dst + 2 * 512, base + r8, pol);
        cp16(dst + 3 * 512, base + r8 + 64, pol);
    } else {
        const DramaB200Int4Bank& b = a.int4;
        const int32_t* base = b.w2 + rec.slot * b.w2_slot_stride +
                              static_cast<int64_t>(it.jt * 16 + g) * b.w2_row_stride + it.kb * 16 + 4 * t;
        cp16(dst + 0 * 512, base, pol);
        cp16(dst + 1 * 512, base + 8 * b.w2_row_stride, pol);
    }
    const T* hrow = static_cast<const T*>(a.ws.h);
    if (g < rec.count) {
        // Same k set as the weights: FP8 lanes own k = 16t.. and 64+16t..,
        // INT4 lanes own k = 32t.. (each 16-byte chunk = 16/sizeof(T) values).
        const char* src = reinterpret_cast<const char*>(
            hrow + static_cast<int64_t>(rec_pair(rec, g)) * a.intermediate + it.kb * 128);
        constexpr int kPer = 16 / static_cast<int>(sizeof(T));  // values per chunk
#pragma unroll
        for (int v = 0; v < S::NH; ++v) {
            const int k0 = FMT == 0 ? (v < S::NH / 2 ? 16 * t + v * kPer : 64 + 16 * t + (v - S::NH / 2) * kPer)
                                    : 32 * t + v * kPer;
            cp16(dst + (S::NW + v) * 512, src + k0 * static_cast<int>(sizeof(T)), pol);
        }
    } else {
#pragma unroll
        for (int v = 0; v < S::NH; ++v) cp16_zero(dst + (S::NW + v) * 512, a.ws.h);
    }
}

// Lane (g, t) holds 32 activations of column g; returns f16 B fragments
// scaled by 2^-e with e from the block's max over the four lanes of g.
template <int FMT, int XDT>
__device__ __forceinline__ int dn_fragment(const uint4* hq, uint32_t (&hb)[16]) {
    float v[32];
    if (XDT == DRAMA_B200_F32) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            v[4 * c] = __uint_as_float(hq[c].x);
            v[4 * c + 1] = __uint_as_float(hq[c].y);
            v[4 * c + 2] = __uint_as_float(hq[c].z);
            v[4 * c + 3] = __uint_as_float(hq[c].w);
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t wv[4] = {hq[c].x, hq[c].y, hq[c].z, hq[c].w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (XDT == DRAMA_B200_BF16) {
                    v[8 * c + 2 * u] = __uint_as_float(wv[u] << 16);
                    v[8 * c + 2 * u + 1] = __uint_as_float(wv[u] & 0xffff0000u);
                } else {
                    v[8 * c + 2 * u] = __half2float(__ushort_as_half(static_cast<unsigned short>(wv[u] & 0xffffu)));
                    v[8 * c + 2 * u + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(wv[u] >> 16)));
                }
            }
        }
    }
    // max |v| as a tree (max is exact in any order)
    float mx[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) mx[j] = fmaxf(fmaxf(fabsf(v[j]), fabsf(v[j + 8])), fmaxf(fabsf(v[j + 16]), fabsf(v[j + 24])));
#pragma unroll
    for (int j = 0; j < 4; ++j) mx[j] = fmaxf(mx[j], mx[j + 4]);
    float m = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const int e = f16_exponent_for(m);
    const float inv = ldexpf(1.0f, -e);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float (&vv)[8] = *reinterpret_cast<const float(*)[8]>(v + 8 * c);
        const uint4 o = pack8<FMT>(vv, inv);
        hb[4 * c] = o.x;
        hb[4 * c + 1] = o.y;
        hb[4 * c + 2] = o.z;
        hb[4 * c + 3] = o.w;
    }
    return e;
}

// FP8 down-projection block: 16 rows x 128 K against the activation
// fragments hb, scaled by the weight block scale sb and the activation
// columns' powers of two s0 / s1, added to tot in fp32. `ad` is zero scratch.
__device__ __forceinline__ void dn_mma_fp8_block(const uint4* wq, float sb, float s0, float s1,
                                                 const uint32_t (&hb)[16], float (&ad)[4], float (&tot)[4]) {
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int qi = s >> 2, ci = s & 3;
        uint32_t A[4];
        e4m3x4_to_f16x2x2(comp(wq[qi], ci), A[0], A[2]);
        e4m3x4_to_f16x2x2(comp(wq[2 + qi], ci), A[1], A[3]);
        mma_f16_16816(ad, A, hb[2 * s], hb[2 * s + 1]);
    }
    tot[0] = fmaf(ad[0], sb * s0, tot[0]);
    tot[1] = fmaf(ad[1], sb * s1, tot[1]);
    tot[2] = fmaf(ad[2], sb * s0, tot[2]);
    tot[3] = fmaf(ad[3], sb * s1, tot[3]);
}

// The same block with the 8 MMAs in two independent chains (k steps 0-3 and
// 4-7, summed before scaling): shorter latency when one warp owns a whole
// K range.
__device__ __forceinline__ void dn_mma_fp8_block2(const uint4* wq, float sb, float s0, float s1,
                                                  const uint32_t (&hb)[16], float (&tot)[4]) {
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        uint32_t A[4], B[4];
        e4m3x4_to_f16x2x2(comp(wq[0], s), A[0], A[2]);
        e4m3x4_to_f16x2x2(comp(wq[2], s), A[1], A[3]);
        mma_f16_16816(a0, A, hb[2 * s], hb[2 * s + 1]);
        e4m3x4_to_f16x2x2(comp(wq[1], s), B[0], B[2]);
        e4m3x4_to_f16x2x2(comp(wq[3], s), B[1], B[3]);
        mma_f16_16816(a1, B, hb[2 * (s + 4)], hb[2 * (s + 4) + 1]);
    }
    tot[0] = fmaf(a0[0] + a1[0], sb * s0, tot[0]);
    tot[1] = fmaf(a0[1] + a1[1], sb * s1, tot[1]);
    tot[2] = fmaf(a0[2] + a1[2], sb * s0, tot[2]);
    tot[3] = fmaf(a0[3] + a1[3], sb * s1, tot[3]);
}

// Power-of-two scales of the activation columns 2t and 2t + 1 (their
// exponents e are held by lanes 8t and 8t + 4).
__device__ __forceinline__ void column_scales(int e, int t, float& s0, float& s1) {
    s0 = ldexpf(1.0f, __shfl_sync(0xffffffffu, e, 8 * t));
    s1 = ldexpf(1.0f, __shfl_sync(0xffffffffu, e, 8 * t + 4));
}

template <int FMT>
__device__ __forceinline__ void dn_mma(const uint4* wq, const DecodeArgs& a, int slot, const CellIt& it, int g, int t,
                                       const uint32_t (&hb)[16], int e, float (&tot)[4]) {
    float ad[4] = {0.f, 0.f, 0.f, 0.f};
    // exponent of the activation columns 2t and 2t+1 (held by lanes 8t and 8t+4)
    const float s0 = ldexpf(1.0f, __shfl_sync(0xffffffffu, e, 8 * t));
    const float s1 = ldexpf(1.0f, __shfl_sync(0xffffffffu, e, 8 * t + 4));
    if constexpr (FMT == 0) {
        const DramaB200Fp8Bank& b = a.fp8;
        const float sb =
            __ldg(b.w2_scale + slot * b.w2_scale_slot_stride + ((it.jt * 16) >> 7) * b.w2_scale_row_stride + it.kb);
        dn_mma_fp8_block(wq, sb, s0, s1, hb, ad, tot);
    } else {
        const DramaB200Int4Bank& b = a.int4;
        const int rows[2] = {it.jt * 16 + g, it.jt * 16 + g + 8};
        float sc[2];
        uint32_t zc[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            sc[r] = load_scale16(b.w2_scale, b.scale_dtype,
                                 slot * b.w2_scale_slot_stride + rows[r] * b.w2_scale_row_stride + it.kb);
            uint32_t z = 8;
            if (b.w2_zeros) {
                const uint32_t word = static_cast<uint32_t>(__ldg(
                    b.w2_zeros + slot * b.w2_zeros_slot_stride + (rows[r] >> 3) * b.w2_zeros_row_stride + it.kb));
                z = (word >> (4 * (rows[r] & 7))) & 15u;
            }
            zc[r] = (0x6400u + z) * 0x10001u;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w0 = comp(wq[0], i), w8 = comp(wq[1], i);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int s = 2 * i + h;
                const uint32_t A[4] = {sub_f16x2(nibbles_to_f16x2_biased(w0 >> (8 * h)), zc[0]),
                                       sub_f16x2(nibbles_to_f16x2_biased(w8 >> (8 * h)), zc[1]),
                                       sub_f16x2(nibbles_to_f16x2_biased(w0 >> (8 * h + 4)), zc[0]),
                                       sub_f16x2(nibbles_to_f16x2_biased(w8 >> (8 * h + 4)), zc[1])};
                mma_f16_16816(ad, A, hb[2 * s], hb[2 * s + 1]);
            }
        }
        tot[0] = fmaf(ad[0], sc[0] * s0, tot[0]);
        tot[1] = fmaf(ad[1], sc[0] * s1, tot[1]);
        tot[2] = fmaf(ad[2], sc[1] * s0, tot[2]);
        tot[3] = fmaf(ad[3], sc[1] * s1, tot[3]);
    }
}

template <int XDT>
__device__ __forceinline__ void dn_finalize(const DecodeArgs& a, const GroupRec& gi, int nt, const float (&acc)[4],
                                            int g, int t, int lane, int groups, float* pair_out) {
    const DecodeWorkspace& ws = a.ws;
    const int H = a.hidden;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int col = 2 * t + cc;
        if (col >= gi.count) continue;
        const int pair = rec_pair(gi, col);
        const float wt = __ldcg(ws.wts + pair);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float down = Scalar<XDT>::round(acc[r * 2 + cc]);
            __stcg(pair_out + static_cast<int64_t>(pair) * H + nt * 16 + g + 8 * r, down * wt);
        }
    }
    if (a.out == nullptr) return;
    __syncwarp();
    int old = 0;
    if (lane == 0) {
        fence_acq_rel_gpu();
        old = atomicAdd(ws.cmb_cnt + nt, 1);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != groups - 1) return;
    fence_acq_rel_gpu();
    const int k = a.top_k;
    using T = typename Scalar<XDT>::T;
    for (int64_t idx = lane; idx < a.tokens * 16; idx += 32) {
        const int64_t tok = idx >> 4;
        const int n = nt * 16 + static_cast<int>(idx & 15);
        const float* src = pair_out + tok * k * H + n;
        float acc2 = 0.0f;
        for (int s0 = 0; s0 < k; s0 += 8) {
            float part[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) part[j] = s0 + j < k ? __ldcg(src + static_cast<int64_t>(s0 + j) * H) : 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (s0 + j < k) acc2 += part[j];
        }
        float v = Scalar<XDT>::round(acc2);
        if (a.moe_out) static_cast<T*>(a.moe_out)[tok * H + n] = Scalar<XDT>::from(v);
        if (a.residual) v = Scalar<XDT>::round(Scalar<XDT>::load(static_cast<const T*>(a.residual) + tok * H + n) + v);
        static_cast<T*>(a.out)[tok * H + n] = Scalar<XDT>::from(v);
    }
}

}  // namespace

}  // namespace drama
