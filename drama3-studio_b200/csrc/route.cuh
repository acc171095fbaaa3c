// Softmax -> top-k -> renormalise for one row per warp, in the arithmetic
// order of torch's CUDA kernels (see router.cu for the restated steps).
#pragma once

#include "common.cuh"

namespace drama {

// Weight of the route in this lane once lanes 0..k-1 hold the k routes in
// their final order (`key` = probability, `valid` = a real route): the
// probability, divided when renormalising by the tree sum of the k keys.
__device__ __forceinline__ float route_weight(int k, bool renormalize, int lane, float key, bool valid) {
    constexpr unsigned kFull = 0xffffffffu;
    float w = valid ? key : 0.0f;
    if (renormalize) {
        int p2 = 1;
        while (p2 < k) p2 <<= 1;
        float tsum = lane < k ? key : 0.0f;
        for (int off = 1; off < p2; off <<= 1) tsum = tsum + __shfl_down_sync(kFull, tsum, off);
        w = w / __shfl_sync(kFull, tsum, 0);
    }
    return w;
}

// Sort + renormalise the k candidates that the selection left in s_key /
// s_idx (gatherTopK order) exactly as torch's CUDA topk(sorted=True) and the
// renormalisation do. Called by a whole warp; lanes 0..k-1 get the result.
__device__ __forceinline__ void route_finish(int k, bool renormalize, int lane, const float* s_key, const int* s_idx,
                                             int& out_idx, float& out_w) {
    constexpr unsigned kFull = 0xffffffffu;
    float key = lane < k ? s_key[lane] : 0.0f;
    // index and validity travel together: (index << 1) | valid
    int iv = lane < k ? (s_idx[lane] << 1) | 1 : 0;
    // 32-slot bitonic network (lane = slot); pair (l, l ^ stride).
    auto stage = [&](int stride, bool flag) {
        const float pk = __shfl_xor_sync(kFull, key, stride);
        const int piv = __shfl_xor_sync(kFull, iv, stride);
        const bool is_a = (lane & stride) == 0;
        const float ka = is_a ? key : pk, kb = is_a ? pk : key;
        const bool va = (is_a ? iv : piv) & 1, vb = (is_a ? piv : iv) & 1;
        const bool swap = ((ka > kb) && va) || !vb;
        if (swap == flag) {
            key = pk;
            iv = piv;
        }
    };
#pragma unroll
    for (int size = 2; size < 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1)
            stage(stride, (((lane / (2 * stride)) * stride + (lane % stride)) & (size >> 1)) != 0);
    }
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) stage(stride, false);
    out_idx = iv >> 1;
    out_w = route_weight(k, renormalize, lane, key, iv & 1);
}

// LANES lanes x ITERS values cover next_pow2(E). `load(idx)` returns the fp32
// logit idx (< E). On return lanes 0..k-1 hold (index, weight) of the k routes
// in torch's topk order; `s_key`/`s_idx` are 32-entry per-warp scratch.
template <int LANES, int ITERS, typename Load>
__device__ __forceinline__ void route_row(Load load, int E, int k, bool renormalize, int lane, float* s_key,
                                          int* s_idx, int& out_idx, float& out_w) {
    constexpr unsigned kFull = 0xffffffffu;
    float v[ITERS];
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        const int idx = lane + i * LANES;
        v[i] = (lane < LANES && idx < E) ? load(idx) : -INFINITY;
    }
    float m = v[0];
#pragma unroll
    for (int i = 1; i < ITERS; ++i) m = fmaxf(m, v[i]);
#pragma unroll
    for (int off = LANES / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, off));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        v[i] = expf(v[i] - m);
        sum += v[i];
    }
#pragma unroll
    for (int off = LANES / 2; off > 0; off >>= 1) sum = sum + __shfl_xor_sync(kFull, sum, off);
    bool live[ITERS];
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        const int idx = lane + i * LANES;
        live[i] = lane < LANES && idx < E;
        v[i] = live[i] ? v[i] / sum : 0.0f;
    }
    // k-th largest probability (with multiplicity).
    bool avail[ITERS];
#pragma unroll
    for (int i = 0; i < ITERS; ++i) avail[i] = live[i];
    int need = k;
    float kth = 0.0f;
    for (int round = 0; round < k; ++round) {
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < ITERS; ++i)
            if (avail[i]) mx = fmaxf(mx, v[i]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
        int cnt = 0;
#pragma unroll
        for (int i = 0; i < ITERS; ++i) {
            const bool eq = avail[i] && v[i] == mx;
            cnt += __popc(__ballot_sync(kFull, eq));
            if (eq) avail[i] = false;
        }
        kth = mx;
        if (cnt >= need) break;
        need -= cnt;
    }
    // gatherTopK order: strictly greater in index order, then equal ones.
    // The k slots hold valid ids first: with NaN probabilities nothing is
    // picked, and the routes then stay inside the expert range.
    s_key[lane] = 0.0f;
    s_idx[lane] = lane < E ? lane : 0;
    __syncwarp();
    const unsigned lt = (1u << lane) - 1u;
    int base = 0;
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        const bool pick = live[i] && v[i] > kth;
        const unsigned b = __ballot_sync(kFull, pick);
        if (pick) {
            s_key[base + __popc(b & lt)] = v[i];
            s_idx[base + __popc(b & lt)] = lane + i * LANES;
        }
        base += __popc(b);
    }
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        const bool eq = live[i] && v[i] == kth;
        const unsigned b = __ballot_sync(kFull, eq);
        const int pos = base + __popc(b & lt);
        if (eq && pos < k) {
            s_key[pos] = v[i];
            s_idx[pos] = lane + i * LANES;
        }
        base += __popc(b);
    }
    __syncwarp();
    route_finish(k, renormalize, lane, s_key, s_idx, out_idx, out_w);
}

// Softmax of one row, by one warp, in route_row's arithmetic order; writes
// p[e] for e < E to `probs` (shared memory).
template <int LANES, int ITERS, typename Load>
__device__ __forceinline__ void route_softmax(Load load, int E, int lane, float* probs) {
    constexpr unsigned kFull = 0xffffffffu;
    float v[ITERS];
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        const int idx = lane + i * LANES;
        v[i] = (lane < LANES && idx < E) ? load(idx) : -INFINITY;
    }
    float m = v[0];
#pragma unroll
    for (int i = 1; i < ITERS; ++i) m = fmaxf(m, v[i]);
#pragma unroll
    for (int off = LANES / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, off));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        v[i] = expf(v[i] - m);
        sum += v[i];
    }
#pragma unroll
    for (int off = LANES / 2; off > 0; off >>= 1) sum = sum + __shfl_xor_sync(kFull, sum, off);
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        const int idx = lane + i * LANES;
        if (lane < LANES && idx < E) probs[idx] = v[i] / sum;
    }
}

// Top-k of the probabilities by rank, over all threads of the CTA: element e
// is chosen when fewer than k elements rank before it (greater, or equal with
// a smaller index), and the chosen ones are placed in gatherTopK order
// (greater than the k-th value in index order, then equal ones in index
// order) in s_key / s_idx[0..k) - the same candidates and slots as
// route_row's selection rounds. `probs` holds E values >= 0 and has room for
// E rounded up to 4 (the padding is set to -1 here); s_cnt is scratch for
// one int per warp plus one float. Contains __syncthreads(): call from every
// thread of the CTA (blockDim.x a multiple of 32, at most 1024).
__device__ __forceinline__ void route_select_cta(float* probs, int E, int k, float* s_key, int* s_idx, int* s_cnt) {
    const int E4 = (E + 3) & ~3;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
    float* s_kth = reinterpret_cast<float*>(s_cnt + 32);
    if (tid < E4 - E) probs[E + tid] = -1.0f;
    __syncthreads();
    const float4* p4 = reinterpret_cast<const float4*>(probs);
    // rank of element e: threads 2e' and 2e' + 1 scan the two halves of the
    // index range and add their counts
    const int n4 = E4 / 4, h4 = (n4 + 1) / 2;
    for (int base = 0; base < E; base += static_cast<int>(blockDim.x) / 2) {
        const int e = base + (tid >> 1), half = tid & 1;
        const float pe = e < E ? probs[e] : 0.0f;
        int r = 0;
        if (e < E) {
            const int j4_end = half ? n4 : h4;
#pragma unroll 4
            for (int j4 = half ? h4 : 0; j4 < j4_end; ++j4) {
                const float4 q = p4[j4];
                const int j = 4 * j4;
                r += (q.x > pe) || (q.x == pe && j < e);
                r += (q.y > pe) || (q.y == pe && j + 1 < e);
                r += (q.z > pe) || (q.z == pe && j + 2 < e);
                r += (q.w > pe) || (q.w == pe && j + 3 < e);
            }
        }
        r += __shfl_xor_sync(0xffffffffu, r, 1);
        if (e < E && half == 0 && r == k - 1) *s_kth = pe;
    }
    __syncthreads();
    const float kth = *s_kth;
    // Slots: an exclusive prefix count, in index order, of the elements above
    // kth and of those equal to it (warp ballots, then the warps' totals).
    int base_gt = 0, base_eq = 0, total_gt = 0;
    {
        // total number of elements above kth (every thread needs it)
        int c = 0;
        for (int e = lane; e < E; e += 32) c += probs[e] > kth;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
        total_gt = c;
    }
    const unsigned below = (1u << lane) - 1u;
    for (int e0 = 0; e0 < E; e0 += blockDim.x) {
        const int e = e0 + tid;
        const float pe = e < E ? probs[e] : -1.0f;
        const unsigned bg = __ballot_sync(0xffffffffu, pe > kth);
        const unsigned be = __ballot_sync(0xffffffffu, pe == kth);
        if (lane == 0) {
            s_cnt[warp] = __popc(bg);
            s_cnt[16 + warp] = __popc(be);
        }
        __syncthreads();
        int pre_gt = base_gt, pre_eq = base_eq, all_gt = 0, all_eq = 0;
        for (int w = 0; w < warps; ++w) {
            if (w < warp) {
                pre_gt += s_cnt[w];
                pre_eq += s_cnt[16 + w];
            }
            all_gt += s_cnt[w];
            all_eq += s_cnt[16 + w];
        }
        if (pe > kth) {
            const int pos = pre_gt + __popc(bg & below);
            s_key[pos] = pe;
            s_idx[pos] = e;
        } else if (pe == kth) {
            const int pos = total_gt + pre_eq + __popc(be & below);
            if (pos < k) {
                s_key[pos] = pe;
                s_idx[pos] = e;
            }
        }
        base_gt += all_gt;
        base_eq += all_eq;
        __syncthreads();
    }
}

// Calls f.template operator()<LANES, ITERS>() for next_pow2(experts) <= 1024.
template <typename F>
__device__ __forceinline__ void dispatch_experts(int experts, F&& f) {
    int p2 = 1;
    while (p2 < experts) p2 <<= 1;
    switch (p2) {
        case 1: f.template operator()<1, 1>(); break;
        case 2: f.template operator()<2, 1>(); break;
        case 4: f.template operator()<4, 1>(); break;
        case 8: f.template operator()<8, 1>(); break;
        case 16: f.template operator()<16, 1>(); break;
        case 32: f.template operator()<32, 1>(); break;
        case 64: f.template operator()<32, 2>(); break;
        case 128: f.template operator()<32, 4>(); break;
        case 256: f.template operator()<32, 8>(); break;
        case 512: f.template operator()<32, 16>(); break;
        default: f.template operator()<32, 32>(); break;
    }
}

}  // namespace drama
