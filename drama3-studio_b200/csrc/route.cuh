// Softmax -> top-k -> renormalise for one row per warp, in the arithmetic
// order of torch's CUDA kernels (see router.cu for the restated steps).
#pragma once

#include "common.cuh"

namespace drama {

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
    float key = lane < k ? s_key[lane] : 0.0f;
    int idx = lane < k ? s_idx[lane] : 0;
    bool valid = lane < k;
    // 32-slot bitonic network (lane = slot); pair (l, l ^ stride).
    auto stage = [&](int stride, bool flag) {
        const float pk = __shfl_xor_sync(kFull, key, stride);
        const int pi = __shfl_xor_sync(kFull, idx, stride);
        const bool pv = __shfl_xor_sync(kFull, valid, stride);
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
#pragma unroll
    for (int size = 2; size < 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1)
            stage(stride, (((lane / (2 * stride)) * stride + (lane % stride)) & (size >> 1)) != 0);
    }
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) stage(stride, false);
    float w = valid ? key : 0.0f;
    if (renormalize) {
        int p2 = 1;
        while (p2 < k) p2 <<= 1;
        float tsum = lane < k ? key : 0.0f;
        for (int off = 1; off < p2; off <<= 1) tsum = tsum + __shfl_down_sync(kFull, tsum, off);
        w = w / __shfl_sync(kFull, tsum, 0);
    }
    out_idx = idx;
    out_w = w;
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
