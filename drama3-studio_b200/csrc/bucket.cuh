// Stable in-CTA bucketing of route IDs (counting sort, index order kept).
#pragma once

#include "common.cuh"

namespace drama {

// ---------------------------------------------------------------------------
// Stable bucket of route IDs inside one CTA (1024 threads). Shared by the
// standalone permutation and the decode preparation kernel.
// smem layout: counts[E] | base[E] | warp_counts[32][E]
// ---------------------------------------------------------------------------
__device__ __forceinline__ void stable_bucket(const void* ids, int ids_dtype, int64_t pairs, int experts,
                              int* smem, int64_t* order64, int32_t* order32, int* dropped) {
    int* counts = smem;
    int* base = smem + experts;
    int* wc = smem + 2 * experts;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < experts; e += blockDim.x) counts[e] = 0;
    for (int e = tid; e < 32 * experts; e += blockDim.x) wc[e] = 0;
    __syncthreads();
    int bad = 0;
    for (int64_t p = tid; p < pairs; p += blockDim.x) {
        const int64_t id = load_index(ids, ids_dtype, p);
        if (id < 0 || id >= experts) ++bad;
        else atomicAdd(&counts[id], 1);
    }
    if (bad) atomicAdd(dropped, bad);
    __syncthreads();
    // Exclusive scan of counts -> base (experts <= 1024, one per thread).
    {
        const int c = tid < experts ? counts[tid] : 0;
        int x = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, off);
            if (lane >= off) x += y;
        }
        __shared__ int warp_tot[32];
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
        const int excl = x - c + (warp ? warp_tot[warp - 1] : 0);
        if (tid < experts) base[tid] = excl;
        __syncthreads();
    }
    const unsigned lt = (1u << lane) - 1u;
    for (int64_t chunk = 0; chunk < pairs; chunk += blockDim.x) {
        const int64_t p = chunk + tid;
        int64_t id = p < pairs ? load_index(ids, ids_dtype, p) : -1;
        if (id >= experts) id = -1;
        if (id < -1) id = -1;
        const unsigned mask = __match_any_sync(0xffffffffu, static_cast<int>(id));
        const int leader = __ffs(mask) - 1;
        const int rank = __popc(mask & lt);
        if (id >= 0 && lane == leader) wc[warp * experts + id] = __popc(mask);
        __syncthreads();
        if (id >= 0) {
            int pos = base[id] + rank;
            for (int w = 0; w < warp; ++w) pos += wc[w * experts + id];
            if (order64) order64[pos] = p;
            else order32[pos] = static_cast<int32_t>(p);
        }
        __syncthreads();
        if (id >= 0 && lane == leader) {
            atomicAdd(&base[id], __popc(mask));
            wc[warp * experts + id] = 0;
        }
        __syncthreads();
    }
}


}  // namespace drama
