// Expert-parallel dispatch and combine around the grouped expert GEMMs.
//
// Experts are sharded in blocks of E/G over G ranks: contiguous by id, or by a
// placement table (rank-major position of every expert, e.g. chosen from
// observed route counts so that the ranks receive similar numbers of rows). Each rank owns
// a slice of the tokens; every (token, slot) pair whose expert lives on rank d
// sends the token's hidden row to d, d runs its experts on what it received,
// and the bf16 down rows travel back to the owner, which sums them in route
// slot order. This is the per-GPU form of the reference's partitioned expert
// call (src/drama_low_vram/offload.py:1206-1276): argsort by expert, one
// expert group at a time, fp32 partials summed in slot order at 1242-1244.
// The reference itself is single-GPU; the exchange has no counterpart there.
//
// The exchange buffers have a fixed capacity of `cap` rows per destination
// rank, so a step needs no host-side count exchange and the whole decode step
// (dispatch, all-to-all, experts, all-to-all, combine) can be captured in one
// CUDA graph. Unused rows carry the local expert id E/G, which the grouped
// GEMM's permute drops.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "peer.cuh"

namespace drama {
namespace {

constexpr int kPlanThreads = 1024;

// Rank-major position of pair p's expert: placement[id] (a permutation of
// [0, experts) giving each expert's rank * E/G + local id), or id itself when
// placement is null; -1 for an id or a placement entry outside [0, experts).
__device__ __forceinline__ int64_t ep_position(const void* ids, int ids_dtype, int64_t p, int experts,
                                               const int32_t* placement) {
    const int64_t id = load_index(ids, ids_dtype, p);
    if (id < 0 || id >= experts) return -1;
    const int64_t pos = placement ? static_cast<int64_t>(__ldg(placement + id)) : id;
    return pos >= 0 && pos < experts ? pos : -1;
}
constexpr int kPlanWarps = kPlanThreads / 32;

// One CTA: destination rank of every pair, its row in the send buffer (pairs
// keep their order inside a destination), and the receiver-local expert id of
// every send row. Deterministic: the same ids always give the same rows.
__global__ void __launch_bounds__(kPlanThreads)
ep_plan_kernel(const void* ids, int ids_dtype, int64_t pairs, int experts, int ranks, const int32_t* placement,
               int64_t cap, __nv_bfloat16* send_rows, int64_t row_stride, int H, int32_t* send_ids,
               int32_t* pair_rows, int32_t* status) {
    __shared__ int warp_tot[kMaxEpRanks][kPlanWarps];
    __shared__ int dropped, overflow;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per_rank = experts / ranks;
    if (tid == 0) dropped = overflow = 0;
    // the receiver-local id of every send row: in send_ids, or in the row's tail
    auto id_slot = [&](int64_t row) -> int32_t* {
        return send_ids ? send_ids + row : reinterpret_cast<int32_t*>(send_rows + row * row_stride + H);
    };
    for (int64_t i = tid; i < ranks * cap; i += kPlanThreads) *id_slot(i) = per_rank;
    const int64_t chunk = (pairs + kPlanThreads - 1) / kPlanThreads;
    const int64_t p0 = min(pairs, tid * chunk), p1 = min(pairs, p0 + chunk);
    int count[kMaxEpRanks];
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) count[d] = 0;
    int bad = 0;
    for (int64_t p = p0; p < p1; ++p) {
        const int64_t pos = ep_position(ids, ids_dtype, p, experts, placement);
        if (pos < 0) { ++bad; continue; }
        const int d = static_cast<int>(pos / per_rank);
#pragma unroll
        for (int r = 0; r < kMaxEpRanks; ++r) count[r] += (r == d);
    }
    // Exclusive scan of every destination's counts over the threads, in order.
    int base[kMaxEpRanks];
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) {
        int v = count[d];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += n;
        }
        if (lane == 31) warp_tot[d][warp] = v;
        base[d] = v - count[d];
    }
    __syncthreads();
    if (warp < kMaxEpRanks) {
        int v = warp_tot[warp][lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += n;
        }
        warp_tot[warp][lane] = v - warp_tot[warp][lane];
    }
    __syncthreads();
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) base[d] += warp_tot[d][warp];
    int over = 0;
    for (int64_t p = p0; p < p1; ++p) {
        const int64_t pos = ep_position(ids, ids_dtype, p, experts, placement);
        int32_t row = -1;
        if (pos >= 0) {
            const int d = static_cast<int>(pos / per_rank);
            int slot = 0;
#pragma unroll
            for (int r = 0; r < kMaxEpRanks; ++r)
                if (r == d) slot = base[r]++;
            if (slot < cap) {
                row = static_cast<int32_t>(d * cap + slot);
                *id_slot(row) = static_cast<int32_t>(pos - static_cast<int64_t>(d) * per_rank);
            } else {
                ++over;
            }
        }
        pair_rows[p] = row;
    }
    if (bad) atomicAdd(&dropped, bad);
    if (over) atomicAdd(&overflow, over);
    __syncthreads();
    if (tid == 0 && status) {
        status[0] = dropped;
        status[1] = overflow;
    }
}

// send_rows[pair_rows[p]] = hidden[p / top_k], 16 bytes per thread step.
__global__ void ep_pack_kernel(const __nv_bfloat16* hidden, int64_t pairs, int top_k, int H,
                               const int32_t* pair_rows, __nv_bfloat16* send_rows, int64_t row_stride) {
    const int vec = H / 8;
    const int64_t n = pairs * vec;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = i / vec;
        const int c = static_cast<int>(i - p * vec) * 8;
        const int32_t row = __ldg(pair_rows + p);
        if (row < 0) continue;
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(hidden + (p / top_k) * H + c));
        *reinterpret_cast<uint4*>(send_rows + static_cast<int64_t>(row) * row_stride + c) = q;
    }
}

// out[t] = bf16(residual[t] + bf16(sum over slots s, in order, of
// bf16 rows[pair_rows[t*k+s]] * w[t*k+s])), fp32 accumulation. Pairs without a
// row (dropped ids, or a row outside [0, row_count)) contribute zero. residual
// may be null.
__global__ void ep_combine_kernel(const __nv_bfloat16* rows, int64_t row_count, const int32_t* pair_rows,
                                  const void* weights,
                                  int weights_dtype, int64_t tokens, int top_k, int H,
                                  const __nv_bfloat16* residual, __nv_bfloat16* out, PeerWait wait) {
    peer_wait_cta(wait);  // rows written by other ranks (peer exchange): their return flags first
    const bool peer = wait.flags != nullptr;
    const int vec = H / 8;
    const int64_t n = tokens * vec;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / vec;
        const int c = static_cast<int>(i - t * vec) * 8;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < top_k; ++s) {
            const int64_t p = t * top_k + s;
            const int32_t row = __ldg(pair_rows + p);
            if (row < 0 || row >= row_count) continue;
            const uint4* src = reinterpret_cast<const uint4*>(rows + static_cast<int64_t>(row) * H + c);
            combine_accumulate(acc, peer ? __ldcg(src) : __ldg(src), load_any(weights, weights_dtype, p));
        }
        uint32_t o[4];
        if (residual) {
            const uint4 r = __ldg(reinterpret_cast<const uint4*>(residual + t * H + c));
            const uint32_t rv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const __nv_bfloat162 m = __floats2bfloat162_rn(acc[2 * u], acc[2 * u + 1]);
                const float lo = __uint_as_float(rv[u] << 16) + __low2float(m);
                const float hi = __uint_as_float(rv[u] & 0xffff0000u) + __high2float(m);
                const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
                o[u] = *reinterpret_cast<const uint32_t*>(&v);
            }
        } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const __nv_bfloat162 v = __floats2bfloat162_rn(acc[2 * u], acc[2 * u + 1]);
                o[u] = *reinterpret_cast<const uint32_t*>(&v);
            }
        }
        *reinterpret_cast<uint4*>(out + t * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

int grid_for(int64_t work, int sm_count) {
    const int64_t blocks = (work + 255) / 256;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(sm_count) * 8)));
}

}  // namespace

cudaError_t ep_dispatch_launch(const void* hidden, int64_t tokens, int H, const void* ids, int ids_dtype, int top_k,
                               int experts, int ranks, const int32_t* placement, int64_t cap, void* send_rows,
                               int64_t row_stride, int32_t* send_ids, int32_t* pair_rows, int32_t* status,
                               int sm_count, cudaStream_t s) {
    const int64_t pairs = tokens * top_k;
    ep_plan_kernel<<<1, kPlanThreads, 0, s>>>(ids, ids_dtype, pairs, experts, ranks, placement, cap,
                                              static_cast<__nv_bfloat16*>(send_rows), row_stride, H, send_ids,
                                              pair_rows, status);
    if (pairs > 0)
        ep_pack_kernel<<<grid_for(pairs * (H / 8), sm_count), 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(hidden), pairs, top_k, H, pair_rows,
            static_cast<__nv_bfloat16*>(send_rows), row_stride);
    return cudaGetLastError();
}

cudaError_t ep_combine_launch(const void* rows, int64_t row_count, const int32_t* pair_rows, const void* weights,
                              int weights_dtype, int64_t tokens, int top_k, int H, const void* residual, void* out,
                              int sm_count, cudaStream_t s, const int32_t* wait_flags, const int32_t* wait_epoch,
                              int wait_ranks, int32_t* status, int64_t wait_ns) {
    PeerWait w;
    w.flags = wait_flags;
    w.epoch = wait_epoch;
    w.ranks = wait_ranks;
    w.bit = 2;
    w.status = status;
    w.limit_ns = peer_wait_limit(wait_ns);
    if (tokens > 0 || wait_flags)
        ep_combine_kernel<<<grid_for(tokens * (H / 8), sm_count), 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(rows), row_count, pair_rows, weights, weights_dtype, tokens, top_k, H,
            static_cast<const __nv_bfloat16*>(residual), static_cast<__nv_bfloat16*>(out), w);
    return cudaGetLastError();
}

}  // namespace drama
