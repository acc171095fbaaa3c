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

namespace drama {

namespace {

constexpr int kRouterThreads = 256;
constexpr unsigned kFullMask = 0xffffffffu;

__global__ void __launch_bounds__(kRouterThreads) moe_router_kernel(MoeLayerArgs a) {
    extern __shared__ float s_norm[];  // [T][H]
    __shared__ float s_red[8];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = a.hidden, E = a.experts, T = static_cast<int>(a.tokens), k = a.top_k;
    const DecodeWorkspace& ws = a.ws;

    // The next layer's router weights are static: start pulling them into L2.
    if (a.next_gate) {
        const int64_t bytes = static_cast<int64_t>(E) * H * 2;
        const int64_t chunk = 32768;
        for (int64_t off = (static_cast<int64_t>(blockIdx.x) * blockDim.x + tid) * chunk; off < bytes;
             off += static_cast<int64_t>(gridDim.x) * blockDim.x * chunk)
            prefetch_l2_bulk(reinterpret_cast<const char*>(a.next_gate) + off,
                             static_cast<uint32_t>(min(chunk, bytes - off)));
    }
    grid_dependency_wait();
    grid_launch_dependents();

    // RMSNorm of every token row (each CTA keeps its own copy in smem).
    const int per = H / kRouterThreads;
    for (int t = 0; t < T; ++t) {
        const __nv_bfloat16* xrow = a.hidden_in + static_cast<int64_t>(t) * H;
        float sq = 0.0f;
        for (int j = 0; j < per; ++j) {
            const float v = __bfloat162float(xrow[tid * per + j]);
            sq = __fadd_rn(sq, __fmul_rn(v, v));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(kFullMask, sq, off));
        if (lane == 0) s_red[warp] = sq;
        __syncthreads();
        float total = 0.0f;
#pragma unroll
        for (int w = 0; w < kRouterThreads / 32; ++w) total = __fadd_rn(total, s_red[w]);
        const float mean = __fmul_rn(total, 1.0f / static_cast<float>(H));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        for (int j = 0; j < per; ++j) {
            const int i = tid * per + j;
            const float v = __bfloat162float(xrow[i]);
            const float y = __fmul_rn(__fmul_rn(v, inv), a.gamma[i]);
            s_norm[t * H + i] = __bfloat162float(__float2bfloat16_rn(y));
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

    // Router GEMV: this CTA's experts, one warp per expert.
    const int per_cta = (E + gridDim.x - 1) / gridDim.x;
    const int e_begin = blockIdx.x * per_cta, e_end = min(E, e_begin + per_cta);
    for (int e = e_begin + warp; e < e_end; e += kRouterThreads / 32) {
        const __nv_bfloat16* grow = a.gate + static_cast<int64_t>(e) * H;
        for (int t = 0; t < T; ++t) {
            float acc = 0.0f;
            for (int i = 0; i < H / 256; ++i) {
                const uint4 q = __ldg(reinterpret_cast<const uint4*>(grow + 256 * i + 8 * lane));
                const __nv_bfloat16* gv = reinterpret_cast<const __nv_bfloat16*>(&q);
                const float* xv = s_norm + t * H + 256 * i + 8 * lane;
#pragma unroll
                for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn(xv[j], __bfloat162float(gv[j])));
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(kFullMask, acc, off));
            if (lane == 0) __stcg(ws.logits + static_cast<int64_t>(t) * E + e, __bfloat162float(__float2bfloat16_rn(acc)));
        }
    }

    // The last CTA to finish routes every token and builds the expert groups.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(ws.router_cnt, 1) == static_cast<int>(gridDim.x) - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid == 0) *ws.router_cnt = 0;

    int* s_ids = reinterpret_cast<int*>(s_norm);           // [T*k]
    float* s_w = s_norm + kMaxLayerPairs;                   // [T*k]
    for (int t = warp; t < T; t += kRouterThreads / 32) {
        // softmax in torch's persistent-warp order (E <= 1024).
        const float* lrow = ws.logits + static_cast<int64_t>(t) * E;
        constexpr int kIt = 32;
        float v[kIt];
        int p2 = 1;
        while (p2 < E) p2 <<= 1;
        const int lanes = p2 < 32 ? p2 : 32;
        const int iters = p2 / lanes;
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
            const int idx = lane + i * lanes;
            v[i] = (i < iters && lane < lanes && idx < E) ? __ldcg(lrow + idx) : -INFINITY;
        }
        float m = v[0];
#pragma unroll
        for (int i = 1; i < kIt; ++i) m = fmaxf(m, v[i]);
        for (int off = lanes / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, off));
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
            if (i < iters) {
                v[i] = expf(v[i] - m);
                sum += v[i];
            }
        }
        for (int off = lanes / 2; off > 0; off >>= 1) sum = sum + __shfl_xor_sync(kFullMask, sum, off);
        bool avail[kIt];
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
            const int idx = lane + i * lanes;
            avail[i] = i < iters && lane < lanes && idx < E;
            v[i] = avail[i] ? v[i] / sum : -INFINITY;
        }
        // k-th largest, gather order, bitonic network: as route_topk.
        int need = k;
        float kth = 0.0f;
        bool rem[kIt];
#pragma unroll
        for (int i = 0; i < kIt; ++i) rem[i] = avail[i];
        for (int round = 0; round < k; ++round) {
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < kIt; ++i)
                if (rem[i]) mx = fmaxf(mx, v[i]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, off));
            int cnt = 0;
#pragma unroll
            for (int i = 0; i < kIt; ++i) {
                const bool eq = rem[i] && v[i] == mx;
                cnt += __popc(__ballot_sync(kFullMask, eq));
                if (eq) rem[i] = false;
            }
            kth = mx;
            if (cnt >= need) break;
            need -= cnt;
        }
        float* s_key = s_w + kMaxLayerPairs + warp * 64;
        int* s_idx = reinterpret_cast<int*>(s_key + 32);
        const unsigned lt = (1u << lane) - 1u;
        int base = 0;
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
            const bool pick = avail[i] && v[i] > kth;
            const unsigned b = __ballot_sync(kFullMask, pick);
            if (pick) {
                s_key[base + __popc(b & lt)] = v[i];
                s_idx[base + __popc(b & lt)] = lane + i * lanes;
            }
            base += __popc(b);
        }
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
            const bool eq = avail[i] && v[i] == kth;
            const unsigned b = __ballot_sync(kFullMask, eq);
            const int pos = base + __popc(b & lt);
            if (eq && pos < k) {
                s_key[pos] = v[i];
                s_idx[pos] = lane + i * lanes;
            }
            base += __popc(b);
        }
        __syncwarp();
        float key = lane < k ? s_key[lane] : 0.0f;
        int idx = lane < k ? s_idx[lane] : 0;
        bool valid = lane < k;
        auto stage = [&](int stride, bool flag) {
            const float pk = __shfl_xor_sync(kFullMask, key, stride);
            const int pi = __shfl_xor_sync(kFullMask, idx, stride);
            const bool pv = __shfl_xor_sync(kFullMask, valid, stride);
            const bool is_a = (lane & stride) == 0;
            const float ka = is_a ? key : pk, kb = is_a ? pk : key;
            const bool va = is_a ? valid : pv, vb = is_a ? pv : valid;
            const bool swap = ((ka > kb) && va) || !vb;
            if (swap == flag) {
                key = pk;
                idx = pi;
                valid = pv;
            }
        };
        for (int size = 2; size < 32; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1)
                stage(stride, (((lane / (2 * stride)) * stride + (lane % stride)) & (size >> 1)) != 0);
        for (int stride = 16; stride > 0; stride >>= 1) stage(stride, false);
        int pk2 = 1;
        while (pk2 < k) pk2 <<= 1;
        float tsum = lane < k ? key : 0.0f;
        for (int off = 1; off < pk2; off <<= 1) tsum = tsum + __shfl_down_sync(kFullMask, tsum, off);
        const float total = __shfl_sync(kFullMask, tsum, 0);
        const float w = __bfloat162float(__float2bfloat16_rn(key / total));
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
        ws.hmax[p] = 0u;
    }
    __syncthreads();
    if (tid == 0) {
        int groups = 0, run_start = 0;
        for (int pos = 0; pos < P; ++pos) {
            const int id = s_ids[s_order[pos]];
            const bool new_id = pos == 0 || s_ids[s_order[pos - 1]] != id;
            if (new_id) run_start = pos;
            if (new_id || (pos - run_start) % kGroupTokens == 0) {
                ws.g_slot[groups] = id;
                ws.g_start[groups] = pos;
                ws.g_count[groups] = 1;
                ++groups;
            } else {
                ws.g_count[groups - 1] += 1;
            }
        }
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
