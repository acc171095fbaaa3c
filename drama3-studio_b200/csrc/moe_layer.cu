// One decode MoE layer on device: RMSNorm -> router GEMV -> softmax/top-k ->
// expert groups -> FP8 expert GEMVs -> slot combine + residual.
//
// Mirrors BackboneDecodeGraph's per-layer sequence (src/drama_low_vram/
// backbone_graph.py:306-337) without the mixer and the shared expert:
//   normed = rms_norm(hidden); logits = gate(normed) (bf16);
//   probs = softmax(logits.float()); w, ids = probs.topk(k); w /= sum; w -> bf16
//   hidden' = hidden + experts(normed, ids, w)
// Everything stays on the device (no host routing), so a whole decode step can
// be captured in one CUDA graph. The router kernel replaces the decode prep
// kernel; the expert kernels are the same K1 up/down kernels.
//
// Fixed fp32 reduction orders (shared with oracle/restate.py):
//   rms_norm: 256 threads add the squares of H/256 consecutive elements in
//     order, xor butterflies within warps, then the 8 warp totals in order;
//     y = bf16((x * (1/sqrt(sum/H + eps))) * gamma).
//   gate: lane l of a warp owns elements 256*i + 8*l + j and adds products in
//     (i, j) order with separate multiply and add; lanes combine by xor
//     butterfly; logits rounded to bf16.
#include "common.cuh"
#include "kernels.h"
#include "route.cuh"

namespace drama {

namespace {

constexpr int kRouterThreads = 256;
constexpr unsigned kFullMask = 0xffffffffu;
constexpr int kMaxPer = 16;     // H <= 4096: elements of a row per router thread
constexpr int kMaxChunks = 16;  // H <= 4096: 256-element chunks per gate row

__global__ void __launch_bounds__(kRouterThreads) moe_router_kernel(MoeLayerArgs a) {
    extern __shared__ float s_norm[];  // [T][H]
    __shared__ float s_red[8];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = a.hidden, E = a.experts, T = static_cast<int>(a.tokens), k = a.top_k;
    const DecodeWorkspace& ws = a.ws;

    // The next layer's router weights are static: start pulling them into L2,
    // 4 KB per request, spread over all CTAs (chunk i goes to CTA i % grid).
    if (a.next_gate) {
        const int64_t bytes = static_cast<int64_t>(E) * H * 2;
        const int64_t chunk = 4096;
        for (int64_t i = blockIdx.x + static_cast<int64_t>(gridDim.x) * tid; i * chunk < bytes;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x)
            prefetch_l2_bulk(reinterpret_cast<const char*>(a.next_gate) + i * chunk,
                             static_cast<uint32_t>(min(chunk, bytes - i * chunk)));
    }
    grid_dependency_wait();
    grid_launch_dependents();

    // RMSNorm of every token row (each CTA keeps its own copy in smem). Thread
    // `tid` owns the H/256 consecutive elements starting at tid*H/256.
    const int per = H / kRouterThreads;  // multiple of 8 (H % 2048 == 0) or H/256 in {1,2,4}
    for (int t = 0; t < T; ++t) {
        const __nv_bfloat16* xrow = a.hidden_in + static_cast<int64_t>(t) * H + tid * per;
        float v[kMaxPer];
        if ((per & 7) == 0) {
#pragma unroll
            for (int j = 0; j < kMaxPer; j += 8) {
                if (j < per) {
                    const uint4 q = *reinterpret_cast<const uint4*>(xrow + j);
                    const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        v[j + 2 * u] = __uint_as_float(wv[u] << 16);
                        v[j + 2 * u + 1] = __uint_as_float(wv[u] & 0xffff0000u);
                    }
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < kMaxPer; ++j)
                if (j < per) v[j] = __bfloat162float(xrow[j]);
        }
        float sq = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxPer; ++j)
            if (j < per) sq = __fadd_rn(sq, __fmul_rn(v[j], v[j]));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(kFullMask, sq, off));
        if (lane == 0) s_red[warp] = sq;
        __syncthreads();
        float total = 0.0f;
#pragma unroll
        for (int w = 0; w < kRouterThreads / 32; ++w) total = __fadd_rn(total, s_red[w]);
        const float mean = __fmul_rn(total, 1.0f / static_cast<float>(H));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
#pragma unroll
        for (int j = 0; j < kMaxPer; ++j) {
            if (j < per) {
                const int i = tid * per + j;
                const float y = __fmul_rn(__fmul_rn(v[j], inv), a.gamma[i]);
                s_norm[t * H + i] = __bfloat162float(__float2bfloat16_rn(y));
            }
        }
        __syncthreads();
    }

    // CTA 0 publishes the normalised rows: f16 copy scaled by 2^-e for the
    // expert GEMVs, and (optionally) the bf16 rows for inspection.
    if (blockIdx.x == 0) {
        for (int t = warp; t < T; t += kRouterThreads / 32) {
            float amax = 0.0f;
            for (int i = lane; i < H; i += 32) amax = fmaxf(amax, fabsf(s_norm[t * H + i]));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFullMask, amax, off));
            const int e = f16_exponent_for(amax);
            const float sc = ldexpf(1.0f, -e);
            if (lane == 0) ws.xscale[t] = ldexpf(1.0f, e);
            __half* dst = reinterpret_cast<__half*>(ws.x16) + static_cast<int64_t>(t) * H;
            for (int i = lane; i < H; i += 32) {
                dst[i] = __float2half_rn(s_norm[t * H + i] * sc);
                if (a.normed_out) a.normed_out[static_cast<int64_t>(t) * H + i] = __float2bfloat16_rn(s_norm[t * H + i]);
            }
        }
    }

    // Router GEMV: this CTA's experts, one warp per expert; all of a row's
    // 16-byte loads are issued before the first product.
    const int per_cta = (E + gridDim.x - 1) / gridDim.x;
    const int e_begin = blockIdx.x * per_cta, e_end = min(E, e_begin + per_cta);
    const int chunks = H / 256;
    for (int e = e_begin + warp; e < e_end; e += kRouterThreads / 32) {
        const __nv_bfloat16* grow = a.gate + static_cast<int64_t>(e) * H;
        uint4 gq[kMaxChunks];
#pragma unroll
        for (int i = 0; i < kMaxChunks; ++i)
            if (i < chunks) gq[i] = __ldg(reinterpret_cast<const uint4*>(grow + 256 * i + 8 * lane));
        for (int t = 0; t < T; ++t) {
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < kMaxChunks; ++i) {
                if (i < chunks) {
                    const __nv_bfloat16* gv = reinterpret_cast<const __nv_bfloat16*>(&gq[i]);
                    const float* xv = s_norm + t * H + 256 * i + 8 * lane;
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn(xv[j], __bfloat162float(gv[j])));
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(kFullMask, acc, off));
            if (lane == 0) __stcg(ws.logits + static_cast<int64_t>(t) * E + e, __bfloat162float(__float2bfloat16_rn(acc)));
        }
    }

    // The last CTA to finish routes every token and builds the expert groups.
    __syncthreads();
    if (tid == 0) {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        s_last = (atomicAdd(ws.router_cnt, 1) == static_cast<int>(gridDim.x) - 1);
    }
    __syncthreads();
    if (!s_last) return;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (tid == 0) *ws.router_cnt = 0;

    int* s_ids = reinterpret_cast<int*>(s_norm);           // [T*k]
    float* s_w = s_norm + kMaxLayerPairs;                   // [T*k]
    for (int t = warp; t < T; t += kRouterThreads / 32) {
        // softmax / top-k / renormalise in torch's CUDA order (route.cuh).
        const float* lrow = ws.logits + static_cast<int64_t>(t) * E;
        float* s_key = s_w + kMaxLayerPairs + warp * 64;
        int* s_idx = reinterpret_cast<int*>(s_key + 32);
        int idx = 0;
        float wr = 0.0f;
        dispatch_experts(E, [&]<int LANES, int ITERS>() {
            route_row<LANES, ITERS>([&](int i) { return __ldcg(lrow + i); }, E, k, true, lane, s_key, s_idx, idx, wr);
        });
        const float w = __bfloat162float(__float2bfloat16_rn(wr));
        if (lane < k) {
            s_ids[t * k + lane] = idx;
            s_w[t * k + lane] = w;
            if (a.ids_out) a.ids_out[static_cast<int64_t>(t) * k + lane] = idx;
            if (a.weights_out) a.weights_out[static_cast<int64_t>(t) * k + lane] = __float2bfloat16_rn(w);
        }
    }
    __syncthreads();

    // Stable order of the T*k pairs by expert and groups of <= 8 (slot order).
    const int P = T * k;
    int* s_order = reinterpret_cast<int*>(s_w + kMaxLayerPairs + 8 * 64);
    __shared__ int s_groups;
    for (int p = tid; p < P; p += blockDim.x) {
        const int id = s_ids[p];
        int rank = 0;
        for (int q = 0; q < P; ++q) {
            const int o = s_ids[q];
            rank += (o < id) || (o == id && q < p);
        }
        s_order[rank] = p;
        ws.order[rank] = p;
        ws.wts[p] = s_w[p];
    }
    __syncthreads();
    if (tid == 0) {
        int groups = 0, run_start = 0, gstart = 0, gcount = 0, gslot = -1;
        int toks[kGroupTokens];
        for (int pos = 0; pos < P; ++pos) {
            const int p = s_order[pos];
            const int id = s_ids[p];
            const bool new_id = pos == 0 || s_ids[s_order[pos - 1]] != id;
            if (new_id) run_start = pos;
            if (new_id || (pos - run_start) % kGroupTokens == 0) {
                if (gcount) write_group(ws, groups++, gslot, gstart, gcount, toks);
                gslot = id;
                gstart = pos;
                gcount = 0;
            }
            toks[gcount++] = p;
        }
        if (gcount) write_group(ws, groups++, gslot, gstart, gcount, toks);
        ws.num_groups[0] = groups;
        ws.status[0] = 0;
        s_groups = groups;
    }
    __syncthreads();
    zero_split_counters(ws, s_groups, H, a.intermediate, tid, blockDim.x);
}

}  // namespace

cudaError_t moe_router_launch(const MoeLayerArgs& m, cudaStream_t s) {
    const size_t smem = static_cast<size_t>(m.tokens) * m.hidden * sizeof(float) +
                        (3 * kMaxLayerPairs + 8 * 64) * sizeof(float);
    static bool configured = false;
    if (!configured) {
        const cudaError_t err = cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     200 * 1024);
        if (err != cudaSuccess) return err;
        configured = true;
    }
    return launch_pdl(moe_router_kernel, dim3(m.router_ctas), dim3(kRouterThreads), smem, s, m);
}

}  // namespace drama
