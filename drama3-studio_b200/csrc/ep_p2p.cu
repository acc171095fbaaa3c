// Expert-parallel exchange over NVLink peer memory (no NCCL on the data path).
//
// Each rank holds three buffers that every other rank maps (CUDA IPC):
//   recv    [ranks][cap][H + 8] bf16: rows sent to this rank; block s is
//           written by rank s, row j = (hidden row, then the receiver-local
//           expert id as an int32 in the 16-byte tail);
//   back    [ranks][cap][H] bf16: the down projections of this rank's rows,
//           block d written by rank d at the positions this rank used;
//   signals [3 * ranks] int32: [s] dispatch flag and [ranks + s] row count
//           written by rank s, [2 * ranks + d] return flag written by rank d.
// A flag holds the step counter (epoch) of the write it announces; every
// rank runs the same sequence of layers, so the counters move in lockstep.
//
// A layer is four launches:
//   dispatch (this file): every CTA numbers all (token, slot) pairs (a block
//     scan, redundant per CTA) and stores its share of the real rows into the
//     owners' recv buffers over NVLink; the last CTA to finish advances the
//     epoch and publishes the counts and, after a system-scope fence, the
//     flags;
//   expert rows (expert_rows.cu): the row-prep kernel waits for every
//     source's flag and skips the rows past each count; the second GEMM
//     stores each result row straight into the source's back buffer and its
//     last CTA publishes the return flags;
//   combine (expert_parallel.cu): waits for every return flag, then sums the
//   route slots from the local back buffer.
// Every wait gives up after the descriptor's wait_ns (2 s when 0) of global
// time and records status[2]; the step's result is then invalid but no kernel
// hangs. Waits are on flags
// written by other GPUs (never by another launch on the same GPU).
//
// Reuse is safe without further flags: rank A writes rank B's recv block of
// layer l + 1 only after B's return flag of layer l, which B publishes after
// its row prep of layer l copied that block away.
#include "common.cuh"
#include "kernels.h"
#include "peer.cuh"

namespace drama {
namespace {

constexpr int kDispThreads = 512;
constexpr int kDispWarps = kDispThreads / 32;

__global__ void __launch_bounds__(kDispThreads)
p2p_dispatch_kernel(DramaB200EpPeers peers, const __nv_bfloat16* hidden, const void* ids, int ids_dtype,
                    int64_t pairs, int top_k, const int32_t* placement, int32_t* pair_rows, int32_t* status) {
    __shared__ int s_row[kP2pMaxPairs], s_tag[kP2pMaxPairs];
    __shared__ int warp_tot[kMaxEpRanks][kDispWarps];
    __shared__ int s_total[kMaxEpRanks];
    __shared__ int dropped, overflow;
    __shared__ bool s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = peers.ranks, me = peers.rank, H = peers.hidden, experts = peers.experts;
    const int per_rank = experts / G;
    const int64_t cap = peers.capacity;
    if (tid == 0) dropped = overflow = 0;

    // 1. destination and row of every pair (pairs keep their order inside a
    // destination); same placement rule as the NCCL path's plan kernel
    auto position = [&](int64_t p) -> int64_t {
        const int64_t id = load_index(ids, ids_dtype, p);
        if (id < 0 || id >= experts) return -1;
        const int64_t pos = placement ? static_cast<int64_t>(__ldg(placement + id)) : id;
        return pos >= 0 && pos < experts ? pos : -1;
    };
    const int64_t chunk = (pairs + kDispThreads - 1) / kDispThreads;
    const int64_t p0 = min(pairs, tid * chunk), p1 = min(pairs, p0 + chunk);
    int count[kMaxEpRanks];
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) count[d] = 0;
    int bad = 0;
    for (int64_t p = p0; p < p1; ++p) {
        const int64_t pos = position(p);
        if (pos < 0) { ++bad; continue; }
        const int d = static_cast<int>(pos / per_rank);
#pragma unroll
        for (int r = 0; r < kMaxEpRanks; ++r) count[r] += (r == d);
    }
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
        int v = lane < kDispWarps ? warp_tot[warp][lane] : 0;
        const int own = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += n;
        }
        if (lane < kDispWarps) warp_tot[warp][lane] = v - own;
        if (lane == 31) s_total[warp] = v;
    }
    __syncthreads();
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) base[d] += warp_tot[d][warp];
    int over = 0;
    for (int64_t p = p0; p < p1; ++p) {
        const int64_t pos = position(p);
        int row = -1, tag = 0;
        if (pos >= 0) {
            const int d = static_cast<int>(pos / per_rank);
            int slot = 0;
#pragma unroll
            for (int r = 0; r < kMaxEpRanks; ++r)
                if (r == d) slot = base[r]++;
            if (slot < cap) {
                row = static_cast<int>(d * cap + slot);
                tag = static_cast<int>(pos - static_cast<int64_t>(d) * per_rank);
            } else {
                ++over;
            }
        }
        s_row[p] = row;
        s_tag[p] = tag;
        if (blockIdx.x == 0) pair_rows[p] = row;
    }
    if (blockIdx.x == 0) {
        if (bad) atomicAdd(&dropped, bad);
        if (over) atomicAdd(&overflow, over);
    }
    __syncthreads();
    if (blockIdx.x == 0 && tid == 0 && status) {
        status[0] = dropped;
        status[1] = overflow;
    }

    // 2. this CTA's share of the real rows into the owners' recv buffers
    const int64_t stride = H + 8;
    const int vec = H / 8 + 1;  // H/8 chunks of the row and the tag chunk
    const int64_t n = pairs * vec;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + tid; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = i / vec;
        const int c = static_cast<int>(i - p * vec);
        const int row = s_row[p];
        if (row < 0) continue;
        const int64_t d = row / cap, j = row - d * cap;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(peers.recv[d]) + (me * cap + j) * stride;
        const uint4 q = c < H / 8 ? __ldg(reinterpret_cast<const uint4*>(hidden + (p / top_k) * H) + c)
                                  : make_uint4(static_cast<uint32_t>(s_tag[p]), 0u, 0u, 0u);
        reinterpret_cast<uint4*>(dst)[c] = q;
    }

    // 3. the last CTA: new epoch, the counts, then the flags
    __threadfence_system();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(peers.done, 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (s_last && tid == 0) {
        __threadfence_system();
        const int e = *peers.epoch + 1;
        *peers.epoch = e;
        for (int d = 0; d < G; ++d) peers.signals[d][G + me] = s_total[d] < cap ? s_total[d] : static_cast<int>(cap);
        __threadfence_system();
        for (int d = 0; d < G; ++d) st_release_sys(peers.signals[d] + me, e);
        *peers.done = 0;
    }
}

}  // namespace

cudaError_t ep_p2p_dispatch_launch(const DramaB200EpPeers& peers, const void* hidden, int64_t tokens,
                                   const void* ids, int ids_dtype, int top_k, const int32_t* placement,
                                   int32_t* pair_rows, int32_t* status, int sm_count, cudaStream_t s) {
    const int64_t pairs = tokens * top_k;
    const int64_t work = pairs * (peers.hidden / 8 + 1);
    int grid = static_cast<int>((work + kDispThreads - 1) / kDispThreads);
    grid = grid < 1 ? 1 : (grid > sm_count ? sm_count : grid);
    p2p_dispatch_kernel<<<grid, kDispThreads, 0, s>>>(peers, static_cast<const __nv_bfloat16*>(hidden), ids,
                                                      ids_dtype, pairs, top_k, placement, pair_rows, status);
    return cudaGetLastError();
}

}  // namespace drama
