// K3: router softmax/top-k/renormalise and the stable route permutation.
//
// route_topk restates BackboneDecodeGraph._route_impl's routing lines
// (src/drama_low_vram/backbone_graph.py:319-323) with torch's CUDA arithmetic
// order, so indices (and their order, ties included) equal what the reference
// computes on the GPU:
//   * softmax: one warp per row, lane l holds elements l + 32*i; exp(x - max)
//     summed per lane in i order, then a xor butterfly; p = e / sum;
//   * topk selection: all values above the k-th largest in index order, then
//     values equal to it in index order;
//   * topk ordering: the 32-slot key/value bitonic network torch uses to sort
//     k <= 32 results (descending; ties resolved by the network);
//   * renormalisation: pairwise tree sum of the k weights (shfl_down 1,2,4..).
// permute_routes restates the host routing of
// ExpertOffloadManager._forward_partitioned (src/drama_low_vram/offload.py:
// 1206-1211): stable argsort by expert plus bincount.
#include <cstdio>

#include "common.cuh"
#include "kernels.h"
#include "route.cuh"
#include "bucket.cuh"

namespace drama {

namespace {


// One warp per token row; LANES lanes x ITERS values cover next_pow2(E).
template <int LANES, int ITERS>
__global__ void __launch_bounds__(256) route_topk_kernel(RouteArgs a) {
    __shared__ float s_key[8][32];
    __shared__ int s_idx[8][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;
    grid_dependency_wait();
    grid_launch_dependents();
    if (row >= a.tokens) return;
    const int E = a.experts;

    int idx = 0;
    float w = 0.0f;
    route_row<LANES, ITERS>([&](int i) { return load_any(a.logits, a.logits_dtype, row * static_cast<int64_t>(E) + i); },
                            E, a.top_k, a.renormalize != 0, lane, s_key[warp], s_idx[warp], idx, w);
    const int k = a.top_k;
    if (lane < k) {
        const int64_t o = row * k + lane;
        store_index(a.ids, a.ids_dtype, o, idx);
        store_any(a.weights, a.weights_dtype, o, w);
    }
}

template <int LANES, int ITERS>
cudaError_t launch_route(const RouteArgs& a, cudaStream_t s) {
    const unsigned blocks = static_cast<unsigned>((a.tokens + 7) / 8);
    return launch_pdl(route_topk_kernel<LANES, ITERS>, dim3(blocks), dim3(256), 0, s, a);
}

}  // namespace

cudaError_t route_topk(const RouteArgs& a, cudaStream_t s) {
    int p2 = 1;
    while (p2 < a.experts) p2 <<= 1;
    switch (p2) {
        case 1: return launch_route<1, 1>(a, s);
        case 2: return launch_route<2, 1>(a, s);
        case 4: return launch_route<4, 1>(a, s);
        case 8: return launch_route<8, 1>(a, s);
        case 16: return launch_route<16, 1>(a, s);
        case 32: return launch_route<32, 1>(a, s);
        case 64: return launch_route<32, 2>(a, s);
        case 128: return launch_route<32, 4>(a, s);
        case 256: return launch_route<32, 8>(a, s);
        case 512: return launch_route<32, 16>(a, s);
        default: return launch_route<32, 32>(a, s);
    }
}

namespace {

__global__ void __launch_bounds__(1024) permute_kernel(PermuteArgs a) {
    extern __shared__ int smem[];
    __shared__ int dropped;
    grid_dependency_wait();
    grid_launch_dependents();
    if (threadIdx.x == 0) dropped = 0;
    __syncthreads();
    stable_bucket(a.ids, a.ids_dtype, a.pairs, a.experts, smem, a.order, nullptr, &dropped);
    // counts survive in smem[0..E); base now holds the exclusive end offsets.
    for (int e = threadIdx.x; e < a.experts; e += blockDim.x) {
        const int c = smem[e];
        const int end = smem[a.experts + e];
        a.counts[e] = c;
        a.offsets[e] = end - c;
        if (e == a.experts - 1) a.offsets[a.experts] = end;
    }
    if (threadIdx.x == 0 && a.status) a.status[0] = dropped;
}

// The same stable permutation for many pairs over many CTAs: each CTA takes
// a chunk of kWideChunk consecutive pairs; the first launch counts each
// chunk's pairs per expert, the second places a chunk's pairs of expert e
// after expert e's pairs of every earlier chunk (so the order stays the
// pairs' index order within each expert) and records each pair's position.
constexpr int kWideChunk = 1024;

__global__ void __launch_bounds__(kWideChunk) permute_count_kernel(PermuteArgs a, int* chunk_counts) {
    extern __shared__ int s_counts[];
    grid_dependency_wait();
    grid_launch_dependents();
    for (int e = threadIdx.x; e < a.experts; e += blockDim.x) s_counts[e] = 0;
    __syncthreads();
    const int64_t p = static_cast<int64_t>(blockIdx.x) * kWideChunk + threadIdx.x;
    if (p < a.pairs) {
        const int64_t id = load_index(a.ids, a.ids_dtype, p);
        if (id >= 0 && id < a.experts) atomicAdd(&s_counts[id], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < a.experts; e += blockDim.x)
        chunk_counts[static_cast<int64_t>(blockIdx.x) * a.experts + e] = s_counts[e];
}

__global__ void __launch_bounds__(kWideChunk) permute_place_kernel(PermuteArgs a, const int* chunk_counts,
                                                                    int64_t* position) {
    extern __shared__ int smem[];
    int* base = smem;                  // [E] first position of this chunk's pairs of each expert
    int* wc = smem + a.experts;        // [32][E] per-warp counts of the current pass
    __shared__ int warp_tot[32];
    grid_dependency_wait();
    grid_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, E = a.experts;
    const int chunks = gridDim.x, me = blockIdx.x;
    // total and earlier-chunk counts per expert (one expert per thread)
    int total = 0, before = 0;
    if (tid < E) {
        for (int b = 0; b < chunks; ++b) {
            const int c = chunk_counts[static_cast<int64_t>(b) * E + tid];
            total += c;
            if (b < me) before += c;
        }
    }
    // exclusive scan of the totals over experts
    int x = total;
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
    const int start = x - total + (warp ? warp_tot[warp - 1] : 0);
    if (tid < E) {
        base[tid] = start + before;
        if (me == 0) {
            a.counts[tid] = total;
            a.offsets[tid] = start;
            if (tid == E - 1) a.offsets[E] = start + total;
        }
    }
    if (me == 0 && tid == 0 && a.status) a.status[0] = static_cast<int32_t>(a.pairs - warp_tot[31]);
    for (int e = tid; e < 32 * E; e += blockDim.x) wc[e] = 0;
    __syncthreads();
    // stable ranks inside the chunk (index order within each expert)
    const int64_t p = static_cast<int64_t>(me) * kWideChunk + tid;
    int64_t id = p < a.pairs ? load_index(a.ids, a.ids_dtype, p) : -1;
    if (id < 0 || id >= E) id = -1;
    const unsigned mask = __match_any_sync(0xffffffffu, static_cast<int>(id));
    const int rank = __popc(mask & ((1u << lane) - 1u));
    if (id >= 0 && lane == __ffs(mask) - 1) wc[warp * E + id] = __popc(mask);
    __syncthreads();
    if (p < a.pairs) {
        int64_t pos = -1;
        if (id >= 0) {
            int q = base[id] + rank;
            for (int w = 0; w < warp; ++w) q += wc[w * E + id];
            a.order[q] = p;
            pos = q;
        }
        if (position) position[p] = pos;
    }
}

}  // namespace

size_t bucket_smem_bytes(int experts) { return static_cast<size_t>(34) * experts * sizeof(int); }

size_t permute_wide_scratch_bytes(int64_t pairs, int experts) {
    return static_cast<size_t>((pairs + kWideChunk - 1) / kWideChunk) * experts * sizeof(int);
}

cudaError_t permute_routes_wide(const PermuteArgs& a, int* chunk_counts, int64_t* position, cudaStream_t s) {
    if (a.experts > kWideChunk) return cudaErrorInvalidValue;
    static bool configured = false;  // benign race: same value from any thread
    if (!configured) {
        const cudaError_t err = cudaFuncSetAttribute(permute_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     static_cast<int>(33 * kWideChunk * sizeof(int)));
        if (err != cudaSuccess) return err;
        configured = true;
    }
    const unsigned chunks = static_cast<unsigned>((a.pairs + kWideChunk - 1) / kWideChunk);
    if (chunks == 0) return cudaSuccess;
    cudaError_t err = launch_pdl(permute_count_kernel, dim3(chunks), dim3(kWideChunk), a.experts * sizeof(int), s, a,
                                 chunk_counts);
    if (err != cudaSuccess) return err;
    return launch_pdl(permute_place_kernel, dim3(chunks), dim3(kWideChunk), 33 * a.experts * sizeof(int), s, a,
                      static_cast<const int*>(chunk_counts), position);
}

cudaError_t permute_routes(const PermuteArgs& a, cudaStream_t s) {
    const size_t smem = bucket_smem_bytes(a.experts);
    static bool configured = false;  // benign race: same value from any thread
    if (!configured) {
        const cudaError_t err = cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     static_cast<int>(bucket_smem_bytes(1024)));
        if (err != cudaSuccess) return err;
        configured = true;
    }
    return launch_pdl(permute_kernel, dim3(1), dim3(1024), smem, s, a);
}

}  // namespace drama
