// Grouped expert GEMMs for few rows per expert (decode batches, expert
// parallelism, staged offload): the weight rows are the MMA's M dimension and
// an expert's token rows its N dimension ("swap AB").
//
// Same arithmetic as the prefill GEMMs and TorchExpertBackend (src/
// drama_low_vram/offload.py:199-244, dequant at 44-56): W = bf16(fp8 * block
// scale); gu = bf16(x @ W13^T); h = bf16(bf16(silu(gate)) * up);
// down = bf16(h @ W2^T). Every output element is one warp's fp32 accumulator
// over the whole K in a fixed order, so a row's result does not depend on the
// other rows of the call.
//
// Work items are (expert, chunk of <= 32 rows, block of weight rows): 64 gate
// + 64 up rows for the first GEMM (so SiLU * up is formed in the CTA), 128
// rows of H for the second. A CTA of 8 warps (16 weight rows each) streams its
// FP8 weight rows and the chunk's activation rows through a 4-stage cp.async
// ring of 128-wide K blocks (one scale block each), expands the FP8 bytes in
// registers to bf16 times the block scale, and issues m16n8k16 MMAs for the
// n8 blocks of the chunk that hold rows. Inside each 64-wide K span a thread
// takes 16 consecutive weight bytes of its two rows; the activation fragments
// use the same K permutation, which leaves every dot product unchanged.
// Weight bytes are read once per (expert, chunk): the whole bank once when an
// expert has at most 32 rows.
#include "common.cuh"
#include "decode_tiles.cuh"
#include "grouped.cuh"
#include "kernels.h"

namespace drama {

namespace {

constexpr int kSwThreads = 256;                   // 8 warps x 16 weight rows
constexpr int kSwRows = 128;                      // weight rows per item
constexpr int kSwTok = 32;                        // token rows per item (4 n8 blocks)
constexpr int kSwBK = 128;                        // K per stage = one scale block
constexpr int kSwStages = 4;
constexpr int kSwW = kSwRows * kSwBK;             // 16 KB of FP8 per stage
constexpr int kSwX = kSwTok * kSwBK * 2;          // 8 KB of bf16 per stage
constexpr int kSwStage = kSwW + kSwX;
constexpr int kSwSmem = kSwStages * kSwStage;     // 96 KB: two CTAs per SM

struct SwapArgs {
    DramaB200Fp8Bank bank;
    const __nv_bfloat16* x;      // GEMM 0: hidden rows [*, H] (row = order[s] / top_k); GEMM 1: h [P, I] sorted
    const int64_t* order;        // [P] rows sorted by expert
    const int64_t* offsets;      // [E + 1]
    __nv_bfloat16* out;          // GEMM 0: h [P, I] sorted; GEMM 1: down [P, H] by order[s]
    int top_k, E, H, I;
};

__device__ __forceinline__ void cp16_plain(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
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
    // chunks (tid + 256 i), i < 2.
    const int wr0 = tid >> 3, wc = tid & 7;           // weight rows wr0 + 32 i
    const int xr0 = tid >> 4, xc = tid & 15;          // activation rows xr0 + 16 i

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
        const __nv_bfloat16* xsrc[2];
        bool xok[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int n = xr0 + 16 * i;
            xok[i] = n < live;
            const int64_t s = off + tok0 + (xok[i] ? n : 0);
            xsrc[i] = MODE == 0 ? a.x + (a.order[s] / a.top_k) * H + xc * 8 : a.x + s * static_cast<int64_t>(I) + xc * 8;
        }
        // this warp's block scale row: gate rows (warps 0-3) / up rows (4-7), or H rows
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
        };

        float acc[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[j][q] = 0.0f;

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
            const float scale = __ldg(sptr + kb);
            const uint8_t* st = smem_sw + (kb % kSwStages) * kSwStage;
#pragma unroll
            for (int span = 0; span < 2; ++span) {
                const int c = 4 * span + t;
                const uint4 qa = *reinterpret_cast<const uint4*>(st + ra * kSwBK + ((c ^ ((ra & 1) << 2)) << 4));
                const uint4 qb = *reinterpret_cast<const uint4*>(st + rbw * kSwBK + ((c ^ ((rbw & 1) << 2)) << 4));
                uint4 xq[4][2];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
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
                    fp8x4_dequant_bf16(comp(qa, ci), scale, A[0], A[2]);
                    fp8x4_dequant_bf16(comp(qb, ci), scale, A[1], A[3]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (j < nb8) {
                            const uint4& u = xq[j][ci >> 1];
                            mma_bf16_16816(acc[j], A, comp(u, 2 * (ci & 1)), comp(u, 2 * (ci & 1) + 1));
                        }
                    }
                }
            }
        }
        cp_wait<0>();
        __syncthreads();   // every stage consumed: the ring is reused for the epilogue

        // acc[j][q]: weight row ra (q < 2) or rbw (q >= 2), token 8j + 2t + (q & 1).
        if (MODE == 0) {
            // up warps publish bf16-rounded up values; gate warps form h.
            float* s_up = reinterpret_cast<float*>(smem_sw);                 // [64 rows][32 tokens]
            __nv_bfloat16* s_h = reinterpret_cast<__nv_bfloat16*>(smem_sw + 64 * kSwTok * 4);  // [32][64]
            if (warp >= 4) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int row = ra - 64 + ((q >> 1) << 3), tok = 8 * j + 2 * t + (q & 1);
                        s_up[row * kSwTok + tok] = acc[j][q];
                    }
            }
            __syncthreads();
            if (warp < 4) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int row = ra + ((q >> 1) << 3), tok = 8 * j + 2 * t + (q & 1);
                        s_h[tok * 64 + row] = __float2bfloat16_rn(swiglu_rounded(acc[j][q], s_up[row * kSwTok + tok]));
                    }
            }
            __syncthreads();
            // 32 tokens x 64 columns x 2 bytes: one 16-byte chunk per thread
            const int tok = tid >> 3, c8 = tid & 7;
            if (tok < live)
                *reinterpret_cast<uint4*>(a.out + (off + tok0 + tok) * static_cast<int64_t>(I) + 64 * rb + 8 * c8) =
                    *reinterpret_cast<const uint4*>(s_h + tok * 64 + 8 * c8);
        } else {
            __nv_bfloat16* s_d = reinterpret_cast<__nv_bfloat16*>(smem_sw);  // [32 tokens][128 rows]
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int row = ra + ((q >> 1) << 3), tok = 8 * j + 2 * t + (q & 1);
                    s_d[tok * kSwRows + row] = __float2bfloat16_rn(acc[j][q]);
                }
            __syncthreads();
            // 32 tokens x 128 columns x 2 bytes: two 16-byte chunks per thread
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int q = tid + 256 * i, tok = q >> 4, c8 = q & 15;
                if (tok < live) {
                    const int64_t row = a.order[off + tok0 + tok];
                    *reinterpret_cast<uint4*>(a.out + row * H + kSwRows * rb + 8 * c8) =
                        *reinterpret_cast<const uint4*>(s_d + tok * kSwRows + 8 * c8);
                }
            }
        }
        __syncthreads();   // the next item's loads reuse the ring
    }
}

}  // namespace

cudaError_t expert_rows_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t rows, const void* ids,
                               int ids_dtype, void* out, const PrefillWorkspace& ws, int sm_count, cudaStream_t s) {
    static bool configured = false;  // benign race: identical values
    if (!configured) {
        cudaError_t err = cudaFuncSetAttribute(swap_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kSwSmem);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(swap_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSwSmem);
        if (err != cudaSuccess) return err;
        configured = true;
    }
    PermuteArgs pa{ids, ids_dtype, rows, bank.slots, ws.order, ws.counts, ws.offsets, ws.status};
    cudaError_t err = permute_routes(pa, s);
    if (err != cudaSuccess) return err;
    SwapArgs a{};
    a.bank = bank;
    a.order = ws.order;
    a.offsets = ws.offsets;
    a.top_k = 1;
    a.E = bank.slots;
    a.H = bank.hidden;
    a.I = bank.intermediate;
    a.x = static_cast<const __nv_bfloat16*>(x);
    a.out = ws.h;
    swap_gemm_kernel<0><<<2 * sm_count, kSwThreads, kSwSmem, s>>>(a);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    a.x = ws.h;
    a.out = static_cast<__nv_bfloat16*>(out);
    swap_gemm_kernel<1><<<2 * sm_count, kSwThreads, kSwSmem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace drama
