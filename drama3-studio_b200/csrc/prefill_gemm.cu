// K2: prefill grouped GEMMs for many tokens per expert.
//
// Semantics are TorchExpertBackend's dequant path (src/drama_low_vram/
// offload.py:199-244, block dequant at offload.py:44-56):
//   W = bf16(fp8 * scale[128x128 block]);  gu = bf16(x @ W13^T)
//   h = bf16(bf16(silu(gate)) * up);       down = bf16(h @ W2^T)
//   out[t] = bf16(sum over route slots, in slot order, of down * weight)
//
// Pairs (token, route slot) are bucketed by expert with the stable permute
// kernel. Each GEMM is a persistent grid over tiles (expert, 128-pair block,
// 64-column block); per 64-wide K stage a CTA gathers its activation rows and
// the expert's FP8 rows with cp.async (double buffered), converts the FP8 rows
// once per CTA to bf16 times the block scale in shared memory, and 8 warps
// (4 along M x 2 along N, 32 x 32 outputs each; gate and up columns side by
// side for the first GEMM) run bf16 m16n8k16 tensor-core MMAs on ldmatrix
// fragments with fp32 accumulators. The epilogues apply the rounding points
// above: SiLU(gate) * up into the sorted activation rows, and the rounded down
// projections into per-pair rows that the combine kernel weights and sums.
//
// (A tcgen05 / TMEM version of this GEMM is not used: it raised an illegal
// instruction on the GPU before its first MMA commit, cause not found.)
#include "common.cuh"
#include "decode_tiles.cuh"
#include "grouped.cuh"
#include "kernels.h"

namespace drama {

namespace {

constexpr int kPfThreads = 256;   // 8 warps
constexpr int kBM = 128;          // pairs per tile
constexpr int kBN = 64;           // output columns per tile (intermediate for GEMM 0, hidden for GEMM 1)
constexpr int kBK = 64;           // K per stage
constexpr int kAStride = kBK + 8;              // bf16 per padded A / B row (144 bytes)
constexpr int kFStride = kBK + 16;             // bytes per padded FP8 row
constexpr int kARows = kBM;
constexpr int kBRowsMax = 2 * kBN;             // gate + up rows
constexpr int kAStage = kARows * kAStride * 2;          // 18432
constexpr int kBStage = kBRowsMax * kAStride * 2;       // 18432
constexpr int kFStage = kBRowsMax * kFStride;           // 10240
constexpr int kStage = kAStage + kBStage + kFStage;     // 47104
constexpr int kPfSmem = 2 * kStage;

struct PrefillArgs {
    DramaB200Fp8Bank bank;
    const __nv_bfloat16* x;      // [T, H] (GEMM 0) or h [P, I] in sorted order (GEMM 1)
    const int64_t* order;        // [P] pairs sorted by expert
    const int64_t* offsets;      // [E + 1]
    __nv_bfloat16* out;          // h [P, I] sorted (GEMM 0) or down [P, H] by pair (GEMM 1)
    int top_k, E, H, I;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// The down GEMM (MODE 1) fits two CTAs per SM (registers and shared memory), so
// it runs twice as many warps to hide the ldmatrix / cp.async latency.
template <int MODE>
__global__ void __launch_bounds__(kPfThreads, MODE == 1 ? 2 : 1) prefill_gemm_kernel(PrefillArgs a) {
    extern __shared__ __align__(16) uint8_t smem_pf[];
    __shared__ int s_prefix[1025];
    constexpr int NT = MODE == 0 ? 8 : 4;        // n8 tiles per warp (gate 4 + up 4, or 4)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int wm = warp & 3, wn = warp >> 2;
    const int E = a.E, H = a.H, I = a.I;
    const int K = MODE == 0 ? H : I;
    const int KT = K / kBK;
    const int nblocks = MODE == 0 ? I / kBN : H / kBN;
    const DramaB200Fp8Bank& b = a.bank;
    const uint32_t sbase = smem_u32(smem_pf);
    const uint64_t pol = policy_evict_last();

    if (tid == 0) {
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            s_prefix[e] = acc;
            const int64_t cnt = a.offsets[e + 1] - a.offsets[e];
            acc += static_cast<int>((cnt + kBM - 1) / kBM) * nblocks;
        }
        s_prefix[E] = acc;
    }
    __syncthreads();
    const int total = s_prefix[E];

    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
        int e, mb, nb;
        decode_tile(tile, s_prefix, E, nblocks, e, mb, nb);
        const int64_t off = a.offsets[e];
        const int cnt = static_cast<int>(a.offsets[e + 1] - off);
        const int n0 = nb * kBN;
        // this thread's copy jobs: A row ar (4 chunks from ac0), FP8 rows
        const int ar = tid >> 1, ac0 = (tid & 1) * 4;
        const int am = mb * kBM + ar;
        const bool a_ok = am < cnt;
        const __nv_bfloat16* arow;
        if (MODE == 0) {
            const int64_t pair = a_ok ? a.order[off + am] : 0;
            arow = a.x + (pair / a.top_k) * H;
        } else {
            arow = a.x + (a_ok ? off + am : 0) * static_cast<int64_t>(I);
        }
        const int fr = MODE == 0 ? tid >> 1 : tid >> 2;              // FP8 row of the tile
        const int fc0 = MODE == 0 ? (tid & 1) * 2 : (tid & 3);       // first 16-byte chunk
        const int nfc = MODE == 0 ? 2 : 1;
        int64_t wrow;
        if (MODE == 0) wrow = fr < kBN ? n0 + fr : I + n0 + (fr - kBN);
        else wrow = n0 + fr;
        const uint8_t* w = static_cast<const uint8_t*>(MODE == 0 ? b.w13 : b.w2) +
                           e * (MODE == 0 ? b.w13_slot_stride : b.w2_slot_stride) +
                           wrow * (MODE == 0 ? b.w13_row_stride : b.w2_row_stride);
        const float* srow = (MODE == 0 ? b.w13_scale : b.w2_scale) +
                            e * (MODE == 0 ? b.w13_scale_slot_stride : b.w2_scale_slot_stride) +
                            (wrow >> 7) * (MODE == 0 ? b.w13_scale_row_stride : b.w2_scale_row_stride);

        auto issue_loads = [&](int kb, int s) {
            const uint32_t sa = sbase + s * kStage, sf = sa + kAStage + kBStage;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t d = sa + ar * (kAStride * 2) + (ac0 + c) * 16;
                if (a_ok) cp16(d, arow + kb * kBK + (ac0 + c) * 8, pol);
                else cp16_zero(d, a.x);
            }
            for (int c = 0; c < nfc; ++c)
                cp16(sf + fr * kFStride + (fc0 + c) * 16, w + kb * kBK + (fc0 + c) * 16, pol);
            cp_commit();
        };
        auto dequant = [&](int kb, int s) {
            const uint8_t* f = smem_pf + s * kStage + kAStage + kBStage;
            __nv_bfloat16* bb = reinterpret_cast<__nv_bfloat16*>(smem_pf + s * kStage + kAStage);
            const float scale = __ldg(srow + ((kb * kBK) >> 7));
            for (int c = 0; c < nfc; ++c) {
                const uint4 q = *reinterpret_cast<const uint4*>(f + fr * kFStride + (fc0 + c) * 16);
                const uint32_t wq[4] = {q.x, q.y, q.z, q.w};
                uint32_t o[8];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float v[4];
                    fp8x4_to_f32(wq[j], v);
                    const __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0] * scale, v[1] * scale);
                    const __nv_bfloat162 p1 = __floats2bfloat162_rn(v[2] * scale, v[3] * scale);
                    o[2 * j] = *reinterpret_cast<const uint32_t*>(&p0);
                    o[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&p1);
                }
                uint4* dst = reinterpret_cast<uint4*>(bb + fr * kAStride + (fc0 + c) * 16);
                dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
            }
        };

        float acc[2][NT][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[mt][j][q] = 0.0f;

        issue_loads(0, 0);
        for (int kb = 0; kb < KT; ++kb) {
            const int s = kb & 1;
            cp_wait<0>();
            __syncthreads();  // stage s landed for every thread; stage s ^ 1 no longer read
            if (kb + 1 < KT) issue_loads(kb + 1, s ^ 1);
            dequant(kb, s);
            __syncthreads();  // B of stage s is bf16
            const uint32_t sa = sbase + s * kStage, sb = sa + kAStage;
            __syncwarp();
#pragma unroll
            for (int k16 = 0; k16 < kBK / 16; ++k16) {
                uint32_t af[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    const int row = 32 * wm + 16 * mt + (lane & 15);
                    ldsm_x4(sa + row * (kAStride * 2) + (k16 * 16 + (lane >> 4) * 8) * 2, af[mt][0], af[mt][1],
                            af[mt][2], af[mt][3]);
                }
#pragma unroll
                for (int jp = 0; jp < NT; jp += 2) {
                    // two n8 tiles (jp, jp + 1): matrices (tile jp, k lo), (jp, k hi), (jp+1, k lo), (jp+1, k hi)
                    const int j = jp + (lane >> 4);
                    int brow;
                    if (MODE == 0) brow = (j < 4 ? 32 * wn + 8 * j : kBN + 32 * wn + 8 * (j - 4)) + (lane & 7);
                    else brow = 32 * wn + 8 * j + (lane & 7);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(sb + brow * (kAStride * 2) + (k16 * 16 + ((lane >> 3) & 1) * 8) * 2, b0, b1, b2, b3);
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        mma_bf16_16816(acc[mt][jp], af[mt], b0, b1);
                        mma_bf16_16816(acc[mt][jp + 1], af[mt], b2, b3);
                    }
                }
            }
        }
        // Epilogue: thread holds rows 32wm + 16mt + g (+8), columns 32wn + 8j + 2t (+1).
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int m = mb * kBM + 32 * wm + 16 * mt + g + 8 * r;
                if (m >= cnt) continue;
                if (MODE == 0) {
                    __nv_bfloat16* hrow = a.out + (off + m) * static_cast<int64_t>(I) + n0 + 32 * wn + 2 * t;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float hv[2];
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            hv[q] = swiglu_rounded(acc[mt][j][2 * r + q], acc[mt][j + 4][2 * r + q]);
                        }
                        *reinterpret_cast<__nv_bfloat162*>(hrow + 8 * j) = __floats2bfloat162_rn(hv[0], hv[1]);
                    }
                } else {
                    const int64_t pair = a.order[off + m];
                    __nv_bfloat16* drow = a.out + pair * H + n0 + 32 * wn + 2 * t;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<__nv_bfloat162*>(drow + 8 * j) =
                            __floats2bfloat162_rn(acc[mt][j][2 * r], acc[mt][j][2 * r + 1]);
                }
            }
        }
        __syncthreads();  // the next tile's first loads reuse stage 0
    }
}

// out[t] = bf16(sum over slots s, in order, of float(down[t*k+s]) * w[t*k+s]);
// pairs whose id is out of range contribute zero.
__global__ void prefill_combine_kernel(const __nv_bfloat16* down, const void* ids, int ids_dtype, int experts,
                                       const void* weights, int weights_dtype, int64_t tokens, int top_k, int H,
                                       __nv_bfloat16* out) {
    const int64_t n = tokens * (H / 8);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / (H / 8);
        const int c = static_cast<int>(i % (H / 8)) * 8;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < top_k; ++s) {
            const int64_t p = t * top_k + s;
            const int64_t id = load_index(ids, ids_dtype, p);
            if (id < 0 || id >= experts) continue;  // dropped pair: contributes zero
            combine_accumulate(acc, __ldg(reinterpret_cast<const uint4*>(down + p * H + c)),
                               load_any(weights, weights_dtype, p));
        }
        uint32_t o[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const __nv_bfloat162 p = __floats2bfloat162_rn(acc[2 * u], acc[2 * u + 1]);
            o[u] = *reinterpret_cast<const uint32_t*>(&p);
        }
        *reinterpret_cast<uint4*>(out + t * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

}  // namespace

size_t prefill_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, int experts, char* base,
                                PrefillWorkspace* ws) {
    const int64_t P = tokens * top_k;
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return p;
    };
    PrefillWorkspace w{};
    w.status = reinterpret_cast<int32_t*>(take(16));
    w.order = reinterpret_cast<int64_t*>(take(P * 8));
    w.counts = reinterpret_cast<int64_t*>(take(static_cast<size_t>(experts) * 8));
    w.offsets = reinterpret_cast<int64_t*>(take(static_cast<size_t>(experts + 1) * 8));
    w.h = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(P) * intermediate * 2));
    w.down = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(P) * hidden * 2));
    if (ws) *ws = w;
    return off;
}

cudaError_t prefill_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t tokens, int top_k, const void* ids,
                           int ids_dtype, const void* weights, int weights_dtype, void* out,
                           const PrefillWorkspace& ws, int sm_count, cudaStream_t s) {
    static bool configured = false;  // benign race: identical values
    if (!configured) {
        cudaError_t err = cudaFuncSetAttribute(prefill_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kPfSmem);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(prefill_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
        if (err != cudaSuccess) return err;
        configured = true;
    }
    const int64_t P = tokens * top_k;
    PermuteArgs pa{ids, ids_dtype, P, bank.slots, ws.order, ws.counts, ws.offsets, ws.status};
    cudaError_t err = permute_routes(pa, s);
    if (err != cudaSuccess) return err;
    PrefillArgs a{};
    a.bank = bank;
    a.order = ws.order;
    a.offsets = ws.offsets;
    a.top_k = top_k;
    a.E = bank.slots;
    a.H = bank.hidden;
    a.I = bank.intermediate;
    a.x = static_cast<const __nv_bfloat16*>(x);
    a.out = ws.h;
    prefill_gemm_kernel<0><<<sm_count, kPfThreads, kPfSmem, s>>>(a);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    a.x = ws.h;
    a.out = ws.down;
    prefill_gemm_kernel<1><<<2 * sm_count, kPfThreads, kPfSmem, s>>>(a);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    const int64_t chunks = tokens * (bank.hidden / 8);
    const int blocks = static_cast<int>(chunks / 256 + 1 < sm_count * 8 ? chunks / 256 + 1 : sm_count * 8);
    prefill_combine_kernel<<<blocks, 256, 0, s>>>(ws.down, ids, ids_dtype, bank.slots, weights, weights_dtype,
                                                  tokens, top_k, bank.hidden, static_cast<__nv_bfloat16*>(out));
    return cudaGetLastError();
}

}  // namespace drama
