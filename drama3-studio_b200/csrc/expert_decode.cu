// K1: decode-regime dequantising SwiGLU expert FFN (FP8 block-scaled / INT4).
//
// Semantics follow the reference's PyTorch dequant path, TorchExpertBackend
// (src/drama_low_vram/offload.py:199-244), and QuantizedExpertBackend(0)
// (src/drama_low_vram/quantized_kernels.py:217-248): gate/up projections are
// rounded to x's dtype, silu(gate) and silu(gate)*up are rounded to x's dtype,
// the down projection is rounded to x's dtype, multiplied by the route weight
// in fp32, and route slots are summed in slot order in fp32.
//
// Structure (three launches chained with programmatic dependent launch):
//   prep : stable bucket of route slots into expert groups of <= 8 tokens,
//          f16 copy of x scaled by a power of two per token (exact for bf16).
//   up   : weight-streaming GEMV over (group, 16-row gate/up tile, 128-K block)
//          cells, balanced evenly over all warps of a persistent grid. Weights
//          are streamed with 16-byte no-L1 loads, converted in registers
//          (E4M3x2 -> f16x2 in one instruction; INT4 nibbles with a magic-number
//          LOP3) and fed to m16n8k16 tensor-core MMAs whose N dimension holds
//          the group's tokens, so weight bytes are read once per group. Block
//          scales are applied per 128-K block in fp32. Tiles split between
//          warps are reduced deterministically by the last arriving warp,
//          which applies SiLU*mul. The up kernel also bulk-prefetches the
//          selected experts' down-projection slabs into L2.
//   down : same scheme over (group, 16-row tile of H, 128-K block); the last
//          arriving warp of a tile rounds, applies the route weight and, when
//          all groups of a row tile are done, sums the route slots.
#include "common.cuh"
#include "kernels.h"
#include "bucket.cuh"

namespace drama {

namespace {

constexpr int kUpDepth = 2;

__device__ __forceinline__ int64_t range_start(int64_t w, int64_t cells, int64_t workers) {
    return w * cells / workers;
}
__device__ __forceinline__ int64_t worker_of(int64_t c, int64_t cells, int64_t workers) {
    return ((c + 1) * workers - 1) / cells;
}

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

__device__ __forceinline__ uint32_t word_of(const uint4& a, const uint4& b, int s) {
    const uint4& q = s < 4 ? a : b;
    switch (s & 3) {
        case 0: return q.x;
        case 1: return q.y;
        case 2: return q.z;
        default: return q.w;
    }
}
__device__ __forceinline__ uint32_t comp(const uint4& q, int i) {
    switch (i) {
        case 0: return q.x;
        case 1: return q.y;
        case 2: return q.z;
        default: return q.w;
    }
}

__device__ __forceinline__ float load_scale16(const void* p, int dtype, int64_t i) {
    return dtype == DRAMA_B200_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i])
                                    : __half2float(static_cast<const __half*>(p)[i]);
}

struct GroupInfo {
    int id;
    int slot, start, count;
};

__device__ __forceinline__ void fetch_group(GroupInfo& g, int id, const DecodeWorkspace& ws) {
    if (g.id != id) {
        g.id = id;
        g.slot = __ldcg(ws.g_slot + id);
        g.start = __ldcg(ws.g_start + id);
        g.count = __ldcg(ws.g_count + id);
    }
}

// Eight consecutive elements starting at a multiple of 8 (16-byte aligned for
// 2-byte types, two 16-byte loads for fp32).
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

// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------
template <int FMT>
__global__ void __launch_bounds__(1024) decode_prep_kernel(DecodeArgs a) {
    extern __shared__ int smem[];
    __shared__ int dropped;
    __shared__ int warp_tot[32];
    grid_dependency_wait();
    grid_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t P = a.tokens * a.top_k;
    const int S = a.slots;
    const DecodeWorkspace& ws = a.ws;
    if (tid == 0) dropped = 0;
    __syncthreads();
    stable_bucket(a.ids, a.ids_dtype, P, S, smem, nullptr, ws.order, &dropped);
    // groups of <= 8 pairs per slot, in slot order.
    const int* counts = smem;
    const int* ends = smem + S;
    int ng = 0;
    if (tid < S) ng = (counts[tid] + kGroupTokens - 1) / kGroupTokens;
    // block exclusive scan of ng (S <= 1024)
    int x = ng;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int t = warp_tot[lane];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, off);
            if (lane >= off) t += y;
        }
        warp_tot[lane] = t;
    }
    __syncthreads();
    const int gbase = x - ng + (warp ? warp_tot[warp - 1] : 0);
    if (tid < S && ng) {
        const int c = counts[tid];
        const int start = ends[tid] - c;
        for (int j = 0; j < ng; ++j) {
            ws.g_slot[gbase + j] = tid;
            ws.g_start[gbase + j] = start + j * kGroupTokens;
            ws.g_count[gbase + j] = min(kGroupTokens, c - j * kGroupTokens);
        }
    }
    const int groups = warp_tot[31];
    if (tid == 0) {
        ws.num_groups[0] = groups;
        ws.status[0] = dropped;
    }
    zero_split_counters(ws, groups, a.hidden, a.intermediate, tid, blockDim.x);
    for (int64_t p = tid; p < P; p += blockDim.x) {
        ws.wts[p] = load_any(a.weights, a.weights_dtype, p);
        ws.hmax[p] = 0u;
    }
    if (dropped) {
        // Pairs with an out-of-range slot contribute zero (and are counted).
        float* po = a.pair_out ? a.pair_out : ws.pair_out;
        for (int64_t p = 0; p < P; ++p) {
            const int64_t id = load_index(a.ids, a.ids_dtype, p);
            if (id < 0 || id >= S)
                for (int n = tid; n < a.hidden; n += blockDim.x) po[p * a.hidden + n] = 0.0f;
        }
    }
    // f16 copy of every token row, scaled by 2^-e: all threads work on
    // 8-element chunks of all rows; per-row amax via an order-free atomicMax.
    const int H = a.hidden;
    unsigned* s_amax = reinterpret_cast<unsigned*>(smem + 34 * S);
    for (int64_t t = tid; t < a.tokens; t += blockDim.x) s_amax[t] = 0u;
    __syncthreads();
    const int64_t chunks = a.tokens * (H / 8);
    for (int64_t c = tid; c < chunks; c += blockDim.x) {
        float v[8];
        load8(a.x, a.x_dtype, c * 8, v);
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
        atomicMax(s_amax + c / (H / 8), __float_as_uint(m));
    }
    __syncthreads();
    for (int64_t t = tid; t < a.tokens; t += blockDim.x)
        ws.xscale[t] = ldexpf(1.0f, f16_exponent_for(__uint_as_float(s_amax[t])));
    for (int64_t c = tid; c < chunks; c += blockDim.x) {
        float v[8];
        load8(a.x, a.x_dtype, c * 8, v);
        const float inv = ldexpf(1.0f, -f16_exponent_for(__uint_as_float(s_amax[c / (H / 8)])));
        uint4 o;
        if (FMT == 1) {  // nibble-pair order inside each 8: [0,4,1,5,2,6,3,7]
            o.x = pack_f16x2(v[0] * inv, v[4] * inv);
            o.y = pack_f16x2(v[1] * inv, v[5] * inv);
            o.z = pack_f16x2(v[2] * inv, v[6] * inv);
            o.w = pack_f16x2(v[3] * inv, v[7] * inv);
        } else {
            o.x = pack_f16x2(v[0] * inv, v[1] * inv);
            o.y = pack_f16x2(v[2] * inv, v[3] * inv);
            o.z = pack_f16x2(v[4] * inv, v[5] * inv);
            o.w = pack_f16x2(v[6] * inv, v[7] * inv);
        }
        reinterpret_cast<uint4*>(ws.x16)[c] = o;
    }
}

// ---------------------------------------------------------------------------
// Shared split-K bookkeeping: a tile's 16 (or 6) K-cells are spread over
// consecutive workers; every contributor but a sole one writes its fragment
// partial, and the last to arrive sums them in worker (= K) order.
// ---------------------------------------------------------------------------
template <int NV>
struct TileFlush {
    // returns true when this warp must finalise `tile` with `acc` (summed).
    __device__ __forceinline__ static bool run(float (&acc)[NV], int64_t tile, int kb_per_tile,
                                               int64_t cells, int64_t workers, int64_t w,
                                               float* part, int32_t* cnt, int lane) {
        const int64_t first_cell = tile * kb_per_tile;
        const int64_t wf = worker_of(first_cell, cells, workers);
        const int64_t wl = worker_of(first_cell + kb_per_tile - 1, cells, workers);
        if (wf == wl) return true;
        const int64_t my_first_tile = range_start(w, cells, workers) / kb_per_tile;
        const int which = (tile == my_first_tile) ? 0 : 1;
        float* dst = part + ((w * 2 + which) * 32 + lane) * NV;
#pragma unroll
        for (int i = 0; i < NV; i += 4)
            __stcg(reinterpret_cast<float4*>(dst + i), make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]));
        __threadfence();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(cnt + tile, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != static_cast<int>(wl - wf)) return false;
        __threadfence();
#pragma unroll
        for (int i = 0; i < NV; ++i) acc[i] = 0.0f;
        for (int64_t v = wf; v <= wl; ++v) {
            const int64_t vt = range_start(v, cells, workers) / kb_per_tile;
            const int wh = (tile == vt) ? 0 : 1;
            const float* src = part + ((v * 2 + wh) * 32 + lane) * NV;
#pragma unroll
            for (int i = 0; i < NV; i += 4) {
                const float4 q = __ldcg(reinterpret_cast<const float4*>(src + i));
                acc[i] += q.x;
                acc[i + 1] += q.y;
                acc[i + 2] += q.z;
                acc[i + 3] += q.w;
            }
        }
        if (lane == 0) cnt[tile] = 0;
        return true;
    }
};

// ---------------------------------------------------------------------------
// up: gate/up GEMV + SiLU*mul
// ---------------------------------------------------------------------------
struct UpCell {
    uint4 q[8];   // FP8: rows g,g+8 of gate (q0..3) and up (q4..7), 32 B each
                  // INT4: q0 gate g, q1 gate g+8, q2 up g, q3 up g+8 (16 B each)
    float sc[4];  // FP8: sc0 = gate block scale, sc1 = up; INT4: per-row scales
    uint32_t zc[4];
};

template <int FMT>
__device__ __forceinline__ void up_load(UpCell& c, const DecodeArgs& a, int slot, int jt, int kb,
                                        int g, int t, uint64_t pol) {
    const int I = a.intermediate;
    if (FMT == 0) {
        const DramaB200Fp8Bank& b = a.fp8;
        const uint8_t* base = static_cast<const uint8_t*>(b.w13) + slot * b.w13_slot_stride +
                              static_cast<int64_t>(jt * 16 + g) * b.w13_row_stride + kb * 128 + 32 * t;
        const int64_t r8 = 8 * b.w13_row_stride, ru = static_cast<int64_t>(I) * b.w13_row_stride;
        c.q[0] = ld_stream_v4(base, pol);
        c.q[1] = ld_stream_v4(base + 16, pol);
        c.q[2] = ld_stream_v4(base + r8, pol);
        c.q[3] = ld_stream_v4(base + r8 + 16, pol);
        c.q[4] = ld_stream_v4(base + ru, pol);
        c.q[5] = ld_stream_v4(base + ru + 16, pol);
        c.q[6] = ld_stream_v4(base + ru + r8, pol);
        c.q[7] = ld_stream_v4(base + ru + r8 + 16, pol);
        const float* s = b.w13_scale + slot * b.w13_scale_slot_stride + kb;
        c.sc[0] = __ldg(s + ((jt * 16) >> 7) * b.w13_scale_row_stride);
        c.sc[1] = __ldg(s + ((I + jt * 16) >> 7) * b.w13_scale_row_stride);
    } else {
        const DramaB200Int4Bank& b = a.int4;
        const int32_t* base = b.w13 + slot * b.w13_slot_stride +
                              static_cast<int64_t>(jt * 16 + g) * b.w13_row_stride + kb * 16 + 4 * t;
        const int64_t r8 = 8 * b.w13_row_stride, ru = static_cast<int64_t>(I) * b.w13_row_stride;
        c.q[0] = ld_stream_v4(base, pol);
        c.q[1] = ld_stream_v4(base + r8, pol);
        c.q[2] = ld_stream_v4(base + ru, pol);
        c.q[3] = ld_stream_v4(base + ru + r8, pol);
        const int rows[4] = {jt * 16 + g, jt * 16 + g + 8, I + jt * 16 + g, I + jt * 16 + g + 8};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            c.sc[r] = load_scale16(b.w13_scale, b.scale_dtype,
                                   slot * b.w13_scale_slot_stride + rows[r] * b.w13_scale_row_stride + kb);
            uint32_t z = 8;
            if (b.w13_zeros) {
                const uint32_t word = static_cast<uint32_t>(__ldg(
                    b.w13_zeros + slot * b.w13_zeros_slot_stride + (rows[r] >> 3) * b.w13_zeros_row_stride + kb));
                z = (word >> (4 * (rows[r] & 7))) & 15u;
            }
            c.zc[r] = (0x6400u + z) * 0x10001u;
        }
    }
}

template <int FMT>
__device__ __forceinline__ void up_mma(const UpCell& c, const uint32_t (&xb)[16], float (&tot)[8]) {
    float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
    if (FMT == 0) {
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const uint32_t wg = word_of(c.q[0], c.q[1], s), wg8 = word_of(c.q[2], c.q[3], s);
            const uint32_t wu = word_of(c.q[4], c.q[5], s), wu8 = word_of(c.q[6], c.q[7], s);
            const uint32_t A[4] = {e4m3x2_to_f16x2(wg), e4m3x2_to_f16x2(wg8), e4m3x2_to_f16x2(wg >> 16),
                                   e4m3x2_to_f16x2(wg8 >> 16)};
            mma_f16_16816(ag, A, xb[2 * s], xb[2 * s + 1]);
            const uint32_t B[4] = {e4m3x2_to_f16x2(wu), e4m3x2_to_f16x2(wu8), e4m3x2_to_f16x2(wu >> 16),
                                   e4m3x2_to_f16x2(wu8 >> 16)};
            mma_f16_16816(au, B, xb[2 * s], xb[2 * s + 1]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            tot[i] = fmaf(ag[i], c.sc[0], tot[i]);
            tot[4 + i] = fmaf(au[i], c.sc[1], tot[4 + i]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wg = comp(c.q[0], i), wg8 = comp(c.q[1], i);
            const uint32_t wu = comp(c.q[2], i), wu8 = comp(c.q[3], i);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int s = 2 * i + h;
                const uint32_t A[4] = {sub_f16x2(nibbles_to_f16x2_biased(wg >> (8 * h)), c.zc[0]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wg8 >> (8 * h)), c.zc[1]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wg >> (8 * h + 4)), c.zc[0]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wg8 >> (8 * h + 4)), c.zc[1])};
                mma_f16_16816(ag, A, xb[2 * s], xb[2 * s + 1]);
                const uint32_t B[4] = {sub_f16x2(nibbles_to_f16x2_biased(wu >> (8 * h)), c.zc[2]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wu8 >> (8 * h)), c.zc[3]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wu >> (8 * h + 4)), c.zc[2]),
                                       sub_f16x2(nibbles_to_f16x2_biased(wu8 >> (8 * h + 4)), c.zc[3])};
                mma_f16_16816(au, B, xb[2 * s], xb[2 * s + 1]);
            }
        }
        tot[0] = fmaf(ag[0], c.sc[0], tot[0]);
        tot[1] = fmaf(ag[1], c.sc[0], tot[1]);
        tot[2] = fmaf(ag[2], c.sc[1], tot[2]);
        tot[3] = fmaf(ag[3], c.sc[1], tot[3]);
        tot[4] = fmaf(au[0], c.sc[2], tot[4]);
        tot[5] = fmaf(au[1], c.sc[2], tot[5]);
        tot[6] = fmaf(au[2], c.sc[3], tot[6]);
        tot[7] = fmaf(au[3], c.sc[3], tot[7]);
    }
}

template <int XDT>
__device__ __forceinline__ void up_finalize(const DecodeArgs& a, const GroupInfo& gi, int jt,
                                            const float (&acc)[8], int g, int t) {
    const DecodeWorkspace& ws = a.ws;
    const int I = a.intermediate;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int col = 2 * t + cc;
        if (col >= gi.count) continue;
        const int pair = __ldcg(ws.order + gi.start + col);
        const float xs = __ldcg(ws.xscale + pair / a.top_k);
        float hmax = 0.0f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float gate = Scalar<XDT>::round(acc[r * 2 + cc] * xs);
            const float up = Scalar<XDT>::round(acc[4 + r * 2 + cc] * xs);
            const float act = Scalar<XDT>::round(gate / (1.0f + expf(-gate)));
            const float hv = Scalar<XDT>::round(act * up);
            ws.h[static_cast<int64_t>(pair) * I + jt * 16 + g + 8 * r] = hv;
            hmax = fmaxf(hmax, fabsf(hv));
        }
        atomicMax(ws.hmax + pair, __float_as_uint(hmax));
    }
}

__device__ __forceinline__ void prefetch_down_slabs(const DecodeArgs& a, int groups) {
    const int H = a.hidden;
    const int tiles = H / 16;
    const int64_t items = static_cast<int64_t>(groups) * tiles;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < items; it += stride) {
        const int group = static_cast<int>(it / tiles), nt = static_cast<int>(it % tiles);
        const int slot = __ldcg(a.ws.g_slot + group);
        const char* base;
        int64_t row_bytes, stride_bytes;
        if (a.format == 0) {
            base = static_cast<const char*>(a.fp8.w2) + slot * a.fp8.w2_slot_stride +
                   static_cast<int64_t>(nt) * 16 * a.fp8.w2_row_stride;
            row_bytes = a.intermediate;
            stride_bytes = a.fp8.w2_row_stride;
        } else {
            base = reinterpret_cast<const char*>(a.int4.w2 + slot * a.int4.w2_slot_stride +
                                                 static_cast<int64_t>(nt) * 16 * a.int4.w2_row_stride);
            row_bytes = a.intermediate / 2;
            stride_bytes = a.int4.w2_row_stride * 4;
        }
        if (stride_bytes == row_bytes) {
            prefetch_l2_bulk(base, static_cast<uint32_t>(16 * row_bytes));
        } else {
            for (int r = 0; r < 16; ++r) prefetch_l2_bulk(base + r * stride_bytes, static_cast<uint32_t>(row_bytes));
        }
    }
}

template <int FMT, int XDT>
__global__ void __launch_bounds__(kDecodeWarps * 32, kDecodeCtasPerSm) decode_up_kernel(DecodeArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int groups = __ldcg(a.ws.num_groups);
    const int KB = a.hidden / 128, TILES = a.intermediate / 16;
    const int64_t cells = static_cast<int64_t>(groups) * TILES * KB;
    const int64_t workers = min(static_cast<int64_t>(a.workers_up), cells);
    const int64_t w = static_cast<int64_t>(blockIdx.x) * kDecodeWarps + warp;
    const bool active = w < workers;
    const int64_t c0 = active ? range_start(w, cells, workers) : 0;
    const int64_t c1 = active ? range_start(w + 1, cells, workers) : 0;
    const uint64_t pol = policy_evict_first();
    const __half* x16 = reinterpret_cast<const __half*>(a.ws.x16);

    UpCell ring[kUpDepth];
    GroupInfo lg{-1, 0, 0, 0}, cg{-1, 0, 0, 0};
    auto issue = [&](UpCell& dst, int64_t c) {
        const int64_t tile = c / KB;
        fetch_group(lg, static_cast<int>(tile / TILES), a.ws);
        up_load<FMT>(dst, a, lg.slot, static_cast<int>(tile % TILES), static_cast<int>(c % KB), g, t, pol);
    };
#pragma unroll
    for (int i = 0; i < kUpDepth - 1; ++i)
        if (c0 + i < c1) issue(ring[i], c0 + i);
    // With the first weight loads in flight, pull the down-projection slabs
    // of this call's experts into L2 for the down kernel.
    prefetch_down_slabs(a, groups);
    if (!active) return;

    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int64_t cur_tile = c0 / KB;
    const __half* xrow = nullptr;
    auto flush = [&](int64_t tile) {
        if (TileFlush<8>::run(acc, tile, KB, cells, workers, w, a.ws.up_part, a.ws.up_cnt, lane)) {
            GroupInfo fg{-1, 0, 0, 0};
            fetch_group(fg, static_cast<int>(tile / TILES), a.ws);
            up_finalize<XDT>(a, fg, static_cast<int>(tile % TILES), acc, g, t);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    };

    for (int64_t cb = c0; cb < c1; cb += kUpDepth) {
#pragma unroll
        for (int i = 0; i < kUpDepth; ++i) {
            const int64_t c = cb + i;
            if (c < c1) {
                const int64_t nxt = c + kUpDepth - 1;
                if (nxt < c1) issue(ring[(i + kUpDepth - 1) % kUpDepth], nxt);
                const int64_t tile = c / KB;
                if (tile != cur_tile) {
                    flush(cur_tile);
                    cur_tile = tile;
                }
                const int group = static_cast<int>(tile / TILES);
                if (cg.id != group) {
                    fetch_group(cg, group, a.ws);
                    xrow = nullptr;
                    if (g < cg.count) {
                        const int pair = __ldcg(a.ws.order + cg.start + g);
                        xrow = x16 + static_cast<int64_t>(pair / a.top_k) * a.hidden;
                    }
                }
                uint32_t xb[16];
                const int kb = static_cast<int>(c % KB);
                if (xrow) {
                    const uint4* src = reinterpret_cast<const uint4*>(xrow + kb * 128 + 32 * t);
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        const uint4 q = __ldg(src + v);
                        xb[4 * v] = q.x;
                        xb[4 * v + 1] = q.y;
                        xb[4 * v + 2] = q.z;
                        xb[4 * v + 3] = q.w;
                    }
                } else {
#pragma unroll
                    for (int v = 0; v < 16; ++v) xb[v] = 0u;
                }
                up_mma<FMT>(ring[i], xb, acc);
            }
        }
    }
    flush(cur_tile);
}

// ---------------------------------------------------------------------------
// down: W2 GEMV + route weight + slot combine
// ---------------------------------------------------------------------------
struct DnCell {
    uint4 q[4];   // FP8: rows g (q0,q1), g+8 (q2,q3); INT4: q0 row g, q1 row g+8
    float sc[2];  // FP8: sc0 block scale; INT4: per-row scales
    uint32_t zc[2];
};

template <int FMT>
__device__ __forceinline__ void dn_load(DnCell& c, const DecodeArgs& a, int slot, int nt, int kb, int g,
                                        int t, uint64_t pol) {
    if (FMT == 0) {
        const DramaB200Fp8Bank& b = a.fp8;
        const uint8_t* base = static_cast<const uint8_t*>(b.w2) + slot * b.w2_slot_stride +
                              static_cast<int64_t>(nt * 16 + g) * b.w2_row_stride + kb * 128 + 32 * t;
        const int64_t r8 = 8 * b.w2_row_stride;
        c.q[0] = ld_stream_v4(base, pol);
        c.q[1] = ld_stream_v4(base + 16, pol);
        c.q[2] = ld_stream_v4(base + r8, pol);
        c.q[3] = ld_stream_v4(base + r8 + 16, pol);
        c.sc[0] = __ldg(b.w2_scale + slot * b.w2_scale_slot_stride + ((nt * 16) >> 7) * b.w2_scale_row_stride + kb);
    } else {
        const DramaB200Int4Bank& b = a.int4;
        const int32_t* base = b.w2 + slot * b.w2_slot_stride + static_cast<int64_t>(nt * 16 + g) * b.w2_row_stride +
                              kb * 16 + 4 * t;
        c.q[0] = ld_stream_v4(base, pol);
        c.q[1] = ld_stream_v4(base + 8 * b.w2_row_stride, pol);
        const int rows[2] = {nt * 16 + g, nt * 16 + g + 8};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            c.sc[r] = load_scale16(b.w2_scale, b.scale_dtype,
                                   slot * b.w2_scale_slot_stride + rows[r] * b.w2_scale_row_stride + kb);
            uint32_t z = 8;
            if (b.w2_zeros) {
                const uint32_t word = static_cast<uint32_t>(__ldg(
                    b.w2_zeros + slot * b.w2_zeros_slot_stride + (rows[r] >> 3) * b.w2_zeros_row_stride + kb));
                z = (word >> (4 * (rows[r] & 7))) & 15u;
            }
            c.zc[r] = (0x6400u + z) * 0x10001u;
        }
    }
}

template <int FMT>
__device__ __forceinline__ void dn_mma(const DnCell& c, const uint32_t (&hb)[16], float (&tot)[4]) {
    float ad[4] = {0.f, 0.f, 0.f, 0.f};
    if (FMT == 0) {
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const uint32_t w0 = word_of(c.q[0], c.q[1], s), w8 = word_of(c.q[2], c.q[3], s);
            const uint32_t A[4] = {e4m3x2_to_f16x2(w0), e4m3x2_to_f16x2(w8), e4m3x2_to_f16x2(w0 >> 16),
                                   e4m3x2_to_f16x2(w8 >> 16)};
            mma_f16_16816(ad, A, hb[2 * s], hb[2 * s + 1]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) tot[i] = fmaf(ad[i], c.sc[0], tot[i]);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w0 = comp(c.q[0], i), w8 = comp(c.q[1], i);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int s = 2 * i + h;
                const uint32_t A[4] = {sub_f16x2(nibbles_to_f16x2_biased(w0 >> (8 * h)), c.zc[0]),
                                       sub_f16x2(nibbles_to_f16x2_biased(w8 >> (8 * h)), c.zc[1]),
                                       sub_f16x2(nibbles_to_f16x2_biased(w0 >> (8 * h + 4)), c.zc[0]),
                                       sub_f16x2(nibbles_to_f16x2_biased(w8 >> (8 * h + 4)), c.zc[1])};
                mma_f16_16816(ad, A, hb[2 * s], hb[2 * s + 1]);
            }
        }
        tot[0] = fmaf(ad[0], c.sc[0], tot[0]);
        tot[1] = fmaf(ad[1], c.sc[0], tot[1]);
        tot[2] = fmaf(ad[2], c.sc[1], tot[2]);
        tot[3] = fmaf(ad[3], c.sc[1], tot[3]);
    }
}

template <int XDT>
__device__ __forceinline__ void dn_finalize(const DecodeArgs& a, const GroupInfo& gi, int nt,
                                            const float (&acc)[4], int g, int t, int lane,
                                            int groups, float* pair_out) {
    const DecodeWorkspace& ws = a.ws;
    const int H = a.hidden;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int col = 2 * t + cc;
        if (col >= gi.count) continue;
        const int pair = __ldcg(ws.order + gi.start + col);
        const float hscale = ldexpf(1.0f, f16_exponent_for(__uint_as_float(__ldcg(ws.hmax + pair))));
        const float wt = __ldcg(ws.wts + pair);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float down = Scalar<XDT>::round(acc[r * 2 + cc] * hscale);
            __stcg(pair_out + static_cast<int64_t>(pair) * H + nt * 16 + g + 8 * r, down * wt);
        }
    }
    if (a.out == nullptr) return;
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(ws.cmb_cnt + nt, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != groups - 1) return;
    __threadfence();
    const int k = a.top_k;
    for (int64_t idx = lane; idx < a.tokens * 16; idx += 32) {
        const int64_t tok = idx >> 4;
        const int n = nt * 16 + static_cast<int>(idx & 15);
        float acc2 = 0.0f;
        for (int s = 0; s < k; ++s) acc2 += __ldcg(pair_out + (tok * k + s) * H + n);
        float v = Scalar<XDT>::round(acc2);
        if (a.residual) v = Scalar<XDT>::round(Scalar<XDT>::load(static_cast<const typename Scalar<XDT>::T*>(a.residual) + tok * H + n) + v);
        static_cast<typename Scalar<XDT>::T*>(a.out)[tok * H + n] = Scalar<XDT>::from(v);
    }
    if (lane == 0) ws.cmb_cnt[nt] = 0;
}

template <int FMT, int XDT>
__global__ void __launch_bounds__(kDecodeWarps * 32, kDecodeCtasPerSm) decode_down_kernel(DecodeArgs a) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int groups = __ldcg(a.ws.num_groups);
    const int KB = a.intermediate / 128, TILES = a.hidden / 16;
    const int64_t cells = static_cast<int64_t>(groups) * TILES * KB;
    if (cells == 0) {
        // Every pair was dropped: the combined output is zero (plus residual).
        if (a.out && blockIdx.x == 0) {
            for (int64_t i = threadIdx.x; i < a.tokens * a.hidden; i += blockDim.x) {
                float v = 0.0f;
                if (a.residual)
                    v = Scalar<XDT>::round(Scalar<XDT>::load(static_cast<const typename Scalar<XDT>::T*>(a.residual) + i));
                static_cast<typename Scalar<XDT>::T*>(a.out)[i] = Scalar<XDT>::from(v);
            }
        }
        return;
    }
    const int64_t workers = min(static_cast<int64_t>(a.workers_dn), cells);
    const int64_t w = static_cast<int64_t>(blockIdx.x) * kDecodeWarps + warp;
    if (w >= workers) return;
    const int64_t c0 = range_start(w, cells, workers), c1 = range_start(w + 1, cells, workers);
    const uint64_t pol = policy_evict_first();
    float* pair_out = a.pair_out ? a.pair_out : a.ws.pair_out;
    const int I = a.intermediate;

    DnCell ring[kUpDepth];
    GroupInfo lg{-1, 0, 0, 0}, cg{-1, 0, 0, 0};
    auto issue = [&](DnCell& dst, int64_t c) {
        const int64_t tile = c / KB;
        fetch_group(lg, static_cast<int>(tile / TILES), a.ws);
        dn_load<FMT>(dst, a, lg.slot, static_cast<int>(tile % TILES), static_cast<int>(c % KB), g, t, pol);
    };
#pragma unroll
    for (int i = 0; i < kUpDepth - 1; ++i)
        if (c0 + i < c1) issue(ring[i], c0 + i);

    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int64_t cur_tile = c0 / KB;
    const float* hrow = nullptr;
    float hinv = 1.0f;
    auto flush = [&](int64_t tile) {
        if (TileFlush<4>::run(acc, tile, KB, cells, workers, w, a.ws.dn_part, a.ws.dn_cnt, lane)) {
            GroupInfo fg{-1, 0, 0, 0};
            fetch_group(fg, static_cast<int>(tile / TILES), a.ws);
            dn_finalize<XDT>(a, fg, static_cast<int>(tile % TILES), acc, g, t, lane, groups, pair_out);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = 0.0f;
    };

    for (int64_t cb = c0; cb < c1; cb += kUpDepth) {
#pragma unroll
        for (int i = 0; i < kUpDepth; ++i) {
            const int64_t c = cb + i;
            if (c < c1) {
                const int64_t nxt = c + kUpDepth - 1;
                if (nxt < c1) issue(ring[(i + kUpDepth - 1) % kUpDepth], nxt);
                const int64_t tile = c / KB;
                if (tile != cur_tile) {
                    flush(cur_tile);
                    cur_tile = tile;
                }
                const int group = static_cast<int>(tile / TILES);
                if (cg.id != group) {
                    fetch_group(cg, group, a.ws);
                    hrow = nullptr;
                    if (g < cg.count) {
                        const int pair = __ldcg(a.ws.order + cg.start + g);
                        hrow = a.ws.h + static_cast<int64_t>(pair) * I;
                        hinv = ldexpf(1.0f, -f16_exponent_for(__uint_as_float(__ldcg(a.ws.hmax + pair))));
                    }
                }
                uint32_t hb[16];
                const int kb = static_cast<int>(c % KB);
                if (hrow) {
                    const float4* src = reinterpret_cast<const float4*>(hrow + kb * 128 + 32 * t);
                    float v[32];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 f = __ldcg(src + q);
                        v[4 * q] = f.x * hinv;
                        v[4 * q + 1] = f.y * hinv;
                        v[4 * q + 2] = f.z * hinv;
                        v[4 * q + 3] = f.w * hinv;
                    }
                    if (FMT == 0) {
#pragma unroll
                        for (int r = 0; r < 16; ++r) hb[r] = pack_f16x2(v[2 * r], v[2 * r + 1]);
                    } else {
#pragma unroll
                        for (int i8 = 0; i8 < 4; ++i8)
#pragma unroll
                            for (int m = 0; m < 4; ++m) hb[4 * i8 + m] = pack_f16x2(v[8 * i8 + m], v[8 * i8 + m + 4]);
                    }
                } else {
#pragma unroll
                    for (int r = 0; r < 16; ++r) hb[r] = 0u;
                }
                dn_mma<FMT>(ring[i], hb, acc);
            }
        }
    }
    flush(cur_tile);
}

template <int FMT, int XDT>
cudaError_t launch_experts(const DecodeArgs& a, cudaStream_t s) {
    cudaError_t err = launch_pdl(decode_up_kernel<FMT, XDT>, dim3(a.ctas), dim3(kDecodeWarps * 32), 0, s, a);
    if (err != cudaSuccess) return err;
    return launch_pdl(decode_down_kernel<FMT, XDT>, dim3(a.ctas), dim3(kDecodeWarps * 32), 0, s, a);
}

template <int FMT, int XDT>
cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t s) {
    const size_t smem = bucket_smem_bytes(a.slots);
    static int configured_smem = -1;  // per template instance; benign race
    cudaError_t err = cudaSuccess;
    if (static_cast<int>(smem) > configured_smem) {
        err = cudaFuncSetAttribute(decode_prep_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(bucket_smem_bytes(kMaxSlots) + kMaxDecodePairs * sizeof(unsigned)));
        if (err != cudaSuccess) return err;
        configured_smem = static_cast<int>(bucket_smem_bytes(kMaxSlots));
    }
    err = launch_pdl(decode_prep_kernel<FMT>, dim3(1), dim3(1024), smem + a.tokens * sizeof(unsigned), s, a);
    if (err != cudaSuccess) return err;
    return launch_experts<FMT, XDT>(a, s);
}

}  // namespace

size_t decode_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, int sm_count,
                               int experts, char* base, DecodeWorkspace* ws) {
    const int64_t P = tokens * top_k;
    const int64_t W = static_cast<int64_t>(sm_count) * kDecodeCtasPerSm * kDecodeWarps;
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return p;
    };
    DecodeWorkspace w{};
    w.status = reinterpret_cast<int32_t*>(take(16));
    w.num_groups = reinterpret_cast<int32_t*>(take(4));
    w.order = reinterpret_cast<int32_t*>(take(P * 4));
    w.g_slot = reinterpret_cast<int32_t*>(take(P * 4));
    w.g_start = reinterpret_cast<int32_t*>(take(P * 4));
    w.g_count = reinterpret_cast<int32_t*>(take(P * 4));
    w.xscale = reinterpret_cast<float*>(take(tokens * 4));
    w.x16 = reinterpret_cast<uint16_t*>(take(tokens * hidden * 2));
    w.wts = reinterpret_cast<float*>(take(P * 4));
    w.h = reinterpret_cast<float*>(take(P * intermediate * 4));
    w.hmax = reinterpret_cast<uint32_t*>(take(P * 4));
    w.pair_out = reinterpret_cast<float*>(take(P * hidden * 4));
    w.up_part = reinterpret_cast<float*>(take(W * 2 * 32 * 8 * 4));
    w.up_cnt = reinterpret_cast<int32_t*>(take(P * (intermediate / 16) * 4));
    w.dn_part = reinterpret_cast<float*>(take(W * 2 * 32 * 4 * 4));
    w.dn_cnt = reinterpret_cast<int32_t*>(take(P * (hidden / 16) * 4));
    w.cmb_cnt = reinterpret_cast<int32_t*>(take((hidden / 16) * 4));
    if (experts > 0) {
        w.logits = reinterpret_cast<float*>(take(tokens * experts * 4));
        w.router_cnt = reinterpret_cast<int32_t*>(take(4));
    }
    if (ws) *ws = w;
    return off;
}

cudaError_t decode_experts_launch(const DecodeArgs& a, cudaStream_t s) {
    const int key = a.format * 8 + a.x_dtype;
    switch (key) {
        case 0 * 8 + DRAMA_B200_BF16: return launch_experts<0, DRAMA_B200_BF16>(a, s);
        case 0 * 8 + DRAMA_B200_F16: return launch_experts<0, DRAMA_B200_F16>(a, s);
        case 0 * 8 + DRAMA_B200_F32: return launch_experts<0, DRAMA_B200_F32>(a, s);
        case 1 * 8 + DRAMA_B200_BF16: return launch_experts<1, DRAMA_B200_BF16>(a, s);
        case 1 * 8 + DRAMA_B200_F16: return launch_experts<1, DRAMA_B200_F16>(a, s);
        default: return launch_experts<1, DRAMA_B200_F32>(a, s);
    }
}

cudaError_t decode_launch(const DecodeArgs& a, cudaStream_t s) {
    const int key = a.format * 8 + a.x_dtype;
    switch (key) {
        case 0 * 8 + DRAMA_B200_BF16: return launch_decode<0, DRAMA_B200_BF16>(a, s);
        case 0 * 8 + DRAMA_B200_F16: return launch_decode<0, DRAMA_B200_F16>(a, s);
        case 0 * 8 + DRAMA_B200_F32: return launch_decode<0, DRAMA_B200_F32>(a, s);
        case 1 * 8 + DRAMA_B200_BF16: return launch_decode<1, DRAMA_B200_BF16>(a, s);
        case 1 * 8 + DRAMA_B200_F16: return launch_decode<1, DRAMA_B200_F16>(a, s);
        default: return launch_decode<1, DRAMA_B200_F32>(a, s);
    }
}

}  // namespace drama
