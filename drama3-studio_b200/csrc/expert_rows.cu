// Grouped expert GEMMs for few rows per expert (decode batches, expert
// parallelism, staged offload): the weight rows are the MMA's M dimension and
// an expert's token rows its N dimension ("swap AB").
//
// Arithmetic: the decode kernels' form of TorchExpertBackend (src/
// drama_low_vram/offload.py:199-244). E4M3 weights expand exactly to f16 (one
// cvt per pair); activations travel as f16 scaled by a power of two per
// 64-wide block of each row (exact for every bf16 value above 2^-24 of the
// block's largest); f16 x f16 products are exact in the fp32 MMA accumulator,
// and each 64-wide K span's partial sum is multiplied by its weight block
// scale and activation scale in fp32. gu, silu(g), silu(g) * up and down are
// rounded to bf16 as the reference rounds them. Every output element is one
// warp's accumulator over the whole K in a fixed order, so a row's result does
// not depend on the other rows of the call.
//
// Work items are (expert, chunk of <= 32 rows, block of weight rows): 64 gate
// + 64 up rows for the first GEMM (so SiLU * up is formed in the CTA), 128
// rows of H for the second. A CTA of 8 warps (16 weight rows each) streams the
// FP8 rows and the chunk's f16 activation rows through a 4-stage cp.async
// ring of 128-wide K blocks and issues m16n8k16 MMAs for the n8 blocks of the
// chunk that hold rows. Inside each 64-wide K span a thread takes 16
// consecutive weight bytes of its two rows; the activation fragments use the
// same K permutation, which leaves every dot product unchanged. Weight bytes
// are read once per (expert, chunk): the whole bank once when no expert has
// more than 32 rows.
#include "common.cuh"
#include "decode_tiles.cuh"
#include "grouped.cuh"
#include "kernels.h"
#include "peer.cuh"

namespace drama {

namespace {

constexpr int kSwThreads = 256;                   // 8 warps x 16 weight rows
constexpr int kSwRows = 128;                      // weight rows per item
constexpr int kSwTok = 32;                        // token rows per item (4 n8 blocks)
constexpr int kSwBK = 128;                        // K per stage = one weight scale block
constexpr int kSwStages = 4;
constexpr int kSwW = kSwRows * kSwBK;             // 16 KB of FP8 per stage
constexpr int kSwX = kSwTok * kSwBK * 2;          // 8 KB of f16 per stage
constexpr int kSwS = kSwTok * 2 * 4;              // activation scales: 32 rows x 2 spans
constexpr int kSwStage = kSwW + kSwX + kSwS;
constexpr int kSwSmem = kSwStages * kSwStage;     // ~97 KB: two CTAs per SM

struct SwapArgs {
    DramaB200Fp8Bank bank;
    const __half* x;             // GEMM 0: f16 rows [*, H] (row = order[s] / top_k); GEMM 1: h [P, I] sorted
    const float* xs;             // their scales: [*, H / 64] or [P, I / 64]
    const int64_t* order;        // [P] rows sorted by expert
    const int64_t* offsets;      // [E + 1]
    __half* h;                   // GEMM 0 out: f16 h [P, I] sorted, scaled per 64 columns
    float* hs;                   // GEMM 0 out: [P, I / 64] scales of h
    __nv_bfloat16* out;          // GEMM 1 out: down [*, H] by order[s]
    RowsScatter scatter;         // GEMM 1 out to peers instead (ranks > 0)
    int top_k, E, H, I;
};

__device__ __forceinline__ void cp16_plain(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp8(uint32_t dst, const void* src, bool ok) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(ok ? 8 : 0) : "memory");
}

// 8 values -> f16 x 8 times `inv` (a power of two).
__device__ __forceinline__ uint4 pack_f16x8(const float (&v)[8], float inv) {
    uint32_t o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const __half2 p = __floats2half2_rn(v[2 * u] * inv, v[2 * u + 1] * inv);
        o[u] = *reinterpret_cast<const uint32_t*>(&p);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// bf16 rows (row r at x + r * x_stride) -> f16 rows [rows, H] scaled by 2^-e
// per 64-wide block, and 2^e. Eight threads per block (16 bytes each); the
// block maximum by shuffles. With `ids` set, the int32 at element H of each
// row (a tagged row) is copied to ids[r].
__global__ void rows_to_f16_kernel(const __nv_bfloat16* x, int64_t x_stride, int64_t rows, int H, __half* xh,
                                   float* xs, int32_t* ids, RowsReceive recv) {
    // Rows written by other ranks: wait for their flags, then treat the rows of
    // block s past count[s] as unused (id recv.unused, nothing converted).
    __shared__ int s_count[8];
    PeerWait pw;
    pw.flags = recv.signals;
    pw.epoch = recv.epoch;
    pw.ranks = recv.ranks;
    pw.bit = 1;
    pw.status = recv.status;
    pw.limit_ns = peer_wait_limit(recv.wait_ns);
    peer_wait_cta(pw);
    if (recv.signals) {
        if (static_cast<int>(threadIdx.x) < recv.ranks)
            s_count[threadIdx.x] = ld_acquire_sys(recv.signals + recv.ranks + threadIdx.x);
        __syncthreads();
    }
    const int64_t n = rows * (H / 8);
    const int64_t n_pad = (n + 31) & ~int64_t(31);   // whole warps iterate together (the shuffles)
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_pad;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / (H / 8), c = i - r * (H / 8);
        bool ok = i < n;
        if (ok && recv.signals) {
            const int64_t src = r / recv.cap;
            if (r - src * recv.cap >= s_count[src]) {
                ok = false;
                if (c == 0) ids[r] = recv.unused;
            }
        }
        // peer-written rows are read through L2 (never from a stale L1 line)
        const uint4 q = ok ? (recv.signals ? __ldcg(reinterpret_cast<const uint4*>(x + r * x_stride) + c)
                                           : __ldg(reinterpret_cast<const uint4*>(x + r * x_stride) + c))
                           : make_uint4(0u, 0u, 0u, 0u);
        if (ok && ids && c == 0)
            ids[r] = recv.signals ? __ldcg(reinterpret_cast<const int32_t*>(x + r * x_stride + H))
                                  : *reinterpret_cast<const int32_t*>(x + r * x_stride + H);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        float v[8];
        float m = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            v[2 * u] = __uint_as_float(w[u] << 16);
            v[2 * u + 1] = __uint_as_float(w[u] & 0xffff0000u);
            m = fmaxf(m, fmaxf(fabsf(v[2 * u]), fabsf(v[2 * u + 1])));
        }
        // the 8 chunks of a 64-wide block sit on 8 consecutive lanes (H / 8 is a multiple of 8)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        const int e = f16_exponent_for(m);
        if (ok) {
            reinterpret_cast<uint4*>(xh)[i] = pack_f16x8(v, ldexpf(1.0f, -e));
            if ((i & 7) == 0) xs[i >> 3] = ldexpf(1.0f, e);
        }
    }
}

template <int MODE>
__global__ void __launch_bounds__(kSwThreads, 2) swap_gemm_kernel(SwapArgs a) {
    extern __shared__ __align__(16) uint8_t smem_sw[];
    __shared__ int s_prefix[1025];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int E = a.E, H = a.H, I = a.I;
    const int K = MODE == 0 ? H : I;
    const int KT = K / kSwBK;
    const int nblocks = MODE == 0 ? I / 64 : H / kSwRows;
    const DramaB200Fp8Bank& b = a.bank;
    const uint32_t sbase = smem_u32(smem_sw);
    const uint64_t pol_x = policy_evict_last();

    if (tid == 0) {
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            s_prefix[e] = acc;
            const int64_t cnt = a.offsets[e + 1] - a.offsets[e];
            acc += static_cast<int>((cnt + kSwTok - 1) / kSwTok) * nblocks;
        }
        s_prefix[E] = acc;
    }
    __syncthreads();
    const int total = s_prefix[E];

    // This thread's copy jobs. Weight tile: 128 rows x 8 chunks of 16 bytes,
    // chunks (tid + 256 i), i < 4; activation tile: 32 rows x 16 chunks,
    // chunks (tid + 256 i), i < 2; scales: 32 rows x 8 bytes (threads < 32).
    const int wr0 = tid >> 3, wc = tid & 7;           // weight rows wr0 + 32 i
    const int xr0 = tid >> 4, xc = tid & 15;          // activation rows xr0 + 16 i
    const int xsK = K / 64;                           // scales per activation row

    for (int item = blockIdx.x; item < total; item += gridDim.x) {
        int e, ch, rb;
        decode_tile(item, s_prefix, E, nblocks, e, ch, rb);
        const int64_t off = a.offsets[e];
        const int cnt = static_cast<int>(a.offsets[e + 1] - off);
        const int tok0 = ch * kSwTok;
        const int live = min(kSwTok, cnt - tok0);     // rows of this chunk (>= 1)
        const int nb8 = (live + 7) >> 3;              // n8 blocks holding rows (warp-uniform)

        const uint8_t* wbase = static_cast<const uint8_t*>(MODE == 0 ? b.w13 : b.w2) +
                               e * (MODE == 0 ? b.w13_slot_stride : b.w2_slot_stride);
        const int64_t wstride = MODE == 0 ? b.w13_row_stride : b.w2_row_stride;
        const uint8_t* wsrc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = wr0 + 32 * i;
            const int64_t row = MODE == 0 ? (r < 64 ? 64 * rb + r : I + 64 * rb + (r - 64)) : kSwRows * rb + r;
            wsrc[i] = wbase + row * wstride + wc * 16;
        }
        const __half* xsrc[2];
        bool xok[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int n = xr0 + 16 * i;
            xok[i] = n < live;
            const int64_t s = off + tok0 + (xok[i] ? n : 0);
            const int64_t row = MODE == 0 ? a.order[s] / a.top_k : s;
            xsrc[i] = a.x + row * K + xc * 8;
        }
        const float* ssrc = nullptr;                  // this thread's scale row (threads < 32)
        const bool sok = tid < kSwTok && tid < live;
        if (tid < kSwTok) {
            const int64_t s = off + tok0 + (sok ? tid : 0);
            const int64_t row = MODE == 0 ? a.order[s] / a.top_k : s;
            ssrc = a.xs + row * xsK;
        }
        // this warp's weight block scale row: gate rows (warps 0-3) / up rows (4-7), or H rows
        const int srow = MODE == 0 ? (warp < 4 ? (64 * rb) >> 7 : (I + 64 * rb) >> 7) : rb;
        const float* sptr = (MODE == 0 ? b.w13_scale : b.w2_scale) +
                            e * (MODE == 0 ? b.w13_scale_slot_stride : b.w2_scale_slot_stride) +
                            srow * (MODE == 0 ? b.w13_scale_row_stride : b.w2_scale_row_stride);

        auto issue = [&](int kb) {
            const uint32_t st = sbase + (kb % kSwStages) * kSwStage;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = wr0 + 32 * i;
                cp16_plain(st + r * kSwBK + ((wc ^ ((r & 1) << 2)) << 4), wsrc[i] + kb * kSwBK);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int n = xr0 + 16 * i;
                const uint32_t d = st + kSwW + n * (kSwBK * 2) + ((xc ^ (n & 1)) << 4);
                if (xok[i]) cp16(d, xsrc[i] + kb * kSwBK, pol_x);
                else cp16_zero(d, a.x);
            }
            if (tid < kSwTok) cp8(st + kSwW + kSwX + tid * 8, ssrc + 2 * kb, sok);
        };

        float tot[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) tot[j][q] = 0.0f;

#pragma unroll
        for (int kb = 0; kb < kSwStages - 1; ++kb) {
            if (kb < KT) issue(kb);
            cp_commit();
        }
        const int ra = 16 * warp + g, rbw = ra + 8;   // this thread's two weight rows in the tile
        for (int kb = 0; kb < KT; ++kb) {
            cp_wait<kSwStages - 2>();
            __syncthreads();   // stage kb landed for all; stage kb - 1 is no longer read
            if (kb + kSwStages - 1 < KT) issue(kb + kSwStages - 1);
            cp_commit();
            const float wscale = __ldg(sptr + kb);
            const uint8_t* st = smem_sw + (kb % kSwStages) * kSwStage;
            const float* sx = reinterpret_cast<const float*>(st + kSwW + kSwX);   // [32 rows][2 spans]
#pragma unroll
            for (int span = 0; span < 2; ++span) {
                const int c = 4 * span + t;
                const uint4 qa = *reinterpret_cast<const uint4*>(st + ra * kSwBK + ((c ^ ((ra & 1) << 2)) << 4));
                const uint4 qb = *reinterpret_cast<const uint4*>(st + rbw * kSwBK + ((c ^ ((rbw & 1) << 2)) << 4));
                uint4 xq[4][2];
                float part[4][4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) part[j][q] = 0.0f;
                    if (j < nb8) {
                        const int n = 8 * j + g;
                        const uint8_t* xr = st + kSwW + n * (kSwBK * 2);
                        xq[j][0] = *reinterpret_cast<const uint4*>(xr + (((8 * span + 2 * t) ^ (n & 1)) << 4));
                        xq[j][1] = *reinterpret_cast<const uint4*>(xr + (((8 * span + 2 * t + 1) ^ (n & 1)) << 4));
                    }
                }
#pragma unroll
                for (int ci = 0; ci < 4; ++ci) {
                    uint32_t A[4];
                    e4m3x4_to_f16x2x2(comp(qa, ci), A[0], A[2]);
                    e4m3x4_to_f16x2x2(comp(qb, ci), A[1], A[3]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (j < nb8) {
                            const uint4& u = xq[j][ci >> 1];
                            mma_f16_16816(part[j], A, comp(u, 2 * (ci & 1)), comp(u, 2 * (ci & 1) + 1));
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (j < nb8) {
                        const float s0 = wscale * sx[(8 * j + 2 * t) * 2 + span];
                        const float s1 = wscale * sx[(8 * j + 2 * t + 1) * 2 + span];
                        tot[j][0] = fmaf(part[j][0], s0, tot[j][0]);
                        tot[j][1] = fmaf(part[j][1], s1, tot[j][1]);
                        tot[j][2] = fmaf(part[j][2], s0, tot[j][2]);
                        tot[j][3] = fmaf(part[j][3], s1, tot[j][3]);
                    }
                }
            }
        }
        cp_wait<0>();
        __syncthreads();   // every stage consumed: the ring is reused for the epilogue

        // tot[j][q]: weight row ra (q < 2) or rbw (q >= 2), token 8j + 2t + (q & 1).
        if (MODE == 0) {
            // up warps publish their sums; gate warps form h = bf16(bf16(silu(g)) * up).
            float* s_up = reinterpret_cast<float*>(smem_sw);                        // [64 rows][32 tokens]
            float* s_h = reinterpret_cast<float*>(smem_sw + 64 * kSwTok * 4);       // [32 tokens][64 cols]
            if (warp >= 4) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int row = ra - 64 + ((q >> 1) << 3), tok = 8 * j + 2 * t + (q & 1);
                        s_up[row * kSwTok + tok] = tot[j][q];
                    }
            }
            __syncthreads();
            if (warp < 4) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int row = ra + ((q >> 1) << 3), tok = 8 * j + 2 * t + (q & 1);
                        s_h[tok * 64 + row] = __bfloat162float(
                            __float2bfloat16_rn(swiglu_rounded(tot[j][q], s_up[row * kSwTok + tok])));
                    }
            }
            __syncthreads();
            // 32 tokens x 64 columns: eight threads per token, 8 values each;
            // the token's 64-column block scale by shuffles over those 8 lanes.
            const int tok = tid >> 3, c8 = tid & 7;
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = s_h[tok * 64 + 8 * c8 + u];
            float m = 0.0f;
#pragma unroll
            for (int u = 0; u < 8; ++u) m = fmaxf(m, fabsf(v[u]));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
            const int ex = f16_exponent_for(m);
            if (tok < live) {
                const int64_t row = off + tok0 + tok;
                *reinterpret_cast<uint4*>(a.h + row * I + 64 * rb + 8 * c8) = pack_f16x8(v, ldexpf(1.0f, -ex));
                if (c8 == 0) a.hs[row * (I / 64) + rb] = ldexpf(1.0f, ex);
            }
        } else {
            __nv_bfloat16* s_d = reinterpret_cast<__nv_bfloat16*>(smem_sw);  // [32 tokens][128 rows]
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int row = ra + ((q >> 1) << 3), tok = 8 * j + 2 * t + (q & 1);
                    s_d[tok * kSwRows + row] = __float2bfloat16_rn(tot[j][q]);
                }
            __syncthreads();
            // 32 tokens x 128 columns x 2 bytes: two 16-byte chunks per thread
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int q = tid + 256 * i, tok = q >> 4, c8 = q & 15;
                if (tok < live) {
                    const int64_t row = a.order[off + tok0 + tok];
                    __nv_bfloat16* dst;
                    if (a.scatter.ranks > 0) {
                        // received row r came from rank r / cap as its row r % cap: straight back into
                        // that rank's return buffer, block of this rank
                        const int64_t src = row / a.scatter.cap, j = row - src * a.scatter.cap;
                        dst = a.scatter.dst[src] + (a.scatter.rank * a.scatter.cap + j) * H;
                    } else {
                        dst = a.out + row * H;
                    }
                    *reinterpret_cast<uint4*>(dst + kSwRows * rb + 8 * c8) =
                        *reinterpret_cast<const uint4*>(s_d + tok * kSwRows + 8 * c8);
                }
            }
        }
        __syncthreads();   // the next item's loads reuse the ring
    }
    if (MODE == 1 && a.scatter.ranks > 0) {
        // every CTA's peer stores fenced; the last CTA to finish publishes the return flags
        __threadfence_system();
        __syncthreads();
        if (tid == 0 && atomicAdd(a.scatter.done, 1) == static_cast<int>(gridDim.x) - 1) {
            __threadfence_system();
            const int e = *a.scatter.epoch;
            for (int d = 0; d < a.scatter.ranks; ++d)
                st_release_sys(a.scatter.signals[d] + 2 * a.scatter.ranks + a.scatter.rank, e);
            *a.scatter.done = 0;
        }
    }
}

int grid_for(int64_t work, int sm_count) {
    const int64_t blocks = (work + 255) / 256;
    return static_cast<int>(blocks < 1 ? 1 : (blocks > sm_count * 8 ? sm_count * 8 : blocks));
}

}  // namespace

size_t expert_rows_workspace_layout(int64_t rows, int hidden, int intermediate, int experts, char* base,
                                    RowsWorkspace* ws) {
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return p;
    };
    RowsWorkspace w{};
    w.status = reinterpret_cast<int32_t*>(take(16));
    w.order = reinterpret_cast<int64_t*>(take(rows * 8));
    w.counts = reinterpret_cast<int64_t*>(take(static_cast<size_t>(experts) * 8));
    w.offsets = reinterpret_cast<int64_t*>(take(static_cast<size_t>(experts + 1) * 8));
    w.xh = reinterpret_cast<__half*>(take(static_cast<size_t>(rows) * hidden * 2));
    w.xs = reinterpret_cast<float*>(take(static_cast<size_t>(rows) * (hidden / 64) * 4));
    w.h = reinterpret_cast<__half*>(take(static_cast<size_t>(rows) * intermediate * 2));
    w.hs = reinterpret_cast<float*>(take(static_cast<size_t>(rows) * (intermediate / 64) * 4));
    w.ids = reinterpret_cast<int32_t*>(take(static_cast<size_t>(rows) * 4));
    if (ws) *ws = w;
    return off;
}

cudaError_t expert_rows_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t x_stride, int64_t rows,
                               const void* ids, int ids_dtype, void* out, const RowsWorkspace& ws, int sm_count,
                               cudaStream_t s, const RowsScatter* scatter, const RowsReceive* receive) {
    static bool configured = false;  // benign race: identical values
    if (!configured) {
        cudaError_t err = cudaFuncSetAttribute(swap_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kSwSmem);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(swap_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSwSmem);
        if (err != cudaSuccess) return err;
        configured = true;
    }
    rows_to_f16_kernel<<<grid_for(rows * (bank.hidden / 8), sm_count), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), x_stride, rows, bank.hidden, ws.xh, ws.xs, ids ? nullptr : ws.ids,
        receive ? *receive : RowsReceive{});
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    PermuteArgs pa{ids ? ids : ws.ids, ids ? ids_dtype : DRAMA_B200_I32, rows, bank.slots, ws.order, ws.counts,
                   ws.offsets, ws.status};
    err = permute_routes(pa, s);
    if (err != cudaSuccess) return err;
    SwapArgs a{};
    a.bank = bank;
    a.order = ws.order;
    a.offsets = ws.offsets;
    a.top_k = 1;
    a.E = bank.slots;
    a.H = bank.hidden;
    a.I = bank.intermediate;
    a.x = ws.xh;
    a.xs = ws.xs;
    a.h = ws.h;
    a.hs = ws.hs;
    swap_gemm_kernel<0><<<2 * sm_count, kSwThreads, kSwSmem, s>>>(a);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    a.x = ws.h;
    a.xs = ws.hs;
    a.out = static_cast<__nv_bfloat16*>(out);
    if (scatter) a.scatter = *scatter;
    swap_gemm_kernel<1><<<2 * sm_count, kSwThreads, kSwSmem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace drama
