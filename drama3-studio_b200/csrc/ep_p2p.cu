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
// Per layer: the plan kernel advances the epoch and numbers each (token,
// slot) pair's row in its destination block; the pack kernel stores the real
// rows (no padding) into the owners' recv buffers over NVLink, and its last
// CTA publishes the counts and, after a system-scope fence, the flags. The
// owner waits for every source's flag (bounded), marks the rows past each
// count as unused, runs the expert-rows GEMMs whose second GEMM stores each
// result row straight into the source rank's back buffer, and a signal kernel
// publishes the return flags; the combine waits for them (bounded) and sums
// the route slots from its local back buffer.
//
// Every wait gives up after kWaitNs of global time, records status[2] and
// returns; the step's result is then wrong but no kernel hangs. Waits are on
// flags written by other GPUs only (never by another launch on this GPU).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace drama {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ int ld_acquire_sys(const int32_t* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int32_t* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Spin until *flag == want or kWaitNs pass; false on timeout.
__device__ __forceinline__ bool wait_flag(const int32_t* flag, int want) {
    const unsigned long long start = global_ns();
    while (ld_acquire_sys(flag) != want) {
        if (global_ns() - start > kWaitNs) return false;
        __nanosleep(200);
    }
    return true;
}

// One CTA: advance the epoch; destination block and row of every pair (pairs
// keep their order inside a destination), its receiver-local id, and the row
// count per destination. Same placement rule as ep_plan_kernel.
__global__ void __launch_bounds__(kPlanThreads)
p2p_plan_kernel(const void* ids, int ids_dtype, int64_t pairs, int experts, int ranks, const int32_t* placement,
                int64_t cap, int32_t* epoch, int32_t* pair_rows, int32_t* pair_tags, int32_t* send_counts,
                int32_t* status) {
    __shared__ int warp_tot[kMaxEpRanks][kPlanWarps];
    __shared__ int dropped, overflow;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per_rank = experts / ranks;
    if (tid == 0) {
        dropped = overflow = 0;
        *epoch = *epoch + 1;
    }
    const int64_t chunk = (pairs + kPlanThreads - 1) / kPlanThreads;
    const int64_t p0 = min(pairs, tid * chunk), p1 = min(pairs, p0 + chunk);
    auto position = [&](int64_t p) -> int64_t {
        const int64_t id = load_index(ids, ids_dtype, p);
        if (id < 0 || id >= experts) return -1;
        const int64_t pos = placement ? static_cast<int64_t>(__ldg(placement + id)) : id;
        return pos >= 0 && pos < experts ? pos : -1;
    };
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
        int v = warp_tot[warp][lane];
        const int own = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += n;
        }
        warp_tot[warp][lane] = v - own;
        if (lane == 31 && warp < ranks) send_counts[warp] = static_cast<int32_t>(v < cap ? v : cap);
    }
    __syncthreads();
#pragma unroll
    for (int d = 0; d < kMaxEpRanks; ++d) base[d] += warp_tot[d][warp];
    int over = 0;
    for (int64_t p = p0; p < p1; ++p) {
        const int64_t pos = position(p);
        int32_t row = -1, tag = 0;
        if (pos >= 0) {
            const int d = static_cast<int>(pos / per_rank);
            int slot = 0;
#pragma unroll
            for (int r = 0; r < kMaxEpRanks; ++r)
                if (r == d) slot = base[r]++;
            if (slot < cap) {
                row = static_cast<int32_t>(d * cap + slot);
                tag = static_cast<int32_t>(pos - static_cast<int64_t>(d) * per_rank);
            } else {
                ++over;
            }
        }
        pair_rows[p] = row;
        pair_tags[p] = tag;
    }
    if (bad) atomicAdd(&dropped, bad);
    if (over) atomicAdd(&overflow, over);
    __syncthreads();
    if (tid == 0 && status) {
        status[0] = dropped;
        status[1] = overflow;
    }
}

// Real rows into the owners' recv buffers (16 bytes per thread step); the
// last CTA to finish publishes the counts, then the flags.
__global__ void p2p_pack_kernel(DramaB200EpPeers peers, const __nv_bfloat16* hidden, int64_t pairs, int top_k,
                                const int32_t* pair_rows, const int32_t* pair_tags, const int32_t* send_counts) {
    __shared__ bool s_last;
    const int H = peers.hidden, G = peers.ranks, me = peers.rank;
    const int64_t cap = peers.capacity, stride = H + 8;
    const int vec = H / 8 + 1;  // H/8 chunks of the row and the tag chunk
    const int64_t n = pairs * vec;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = i / vec;
        const int c = static_cast<int>(i - p * vec);
        const int32_t row = __ldg(pair_rows + p);
        if (row < 0) continue;
        const int64_t d = row / cap, j = row - d * cap;
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(peers.recv[d]) + (me * cap + j) * stride;
        uint4 q;
        if (c < H / 8) {
            q = __ldg(reinterpret_cast<const uint4*>(hidden + (p / top_k) * H) + c);
        } else {
            q = make_uint4(static_cast<uint32_t>(__ldg(pair_tags + p)), 0u, 0u, 0u);
        }
        reinterpret_cast<uint4*>(dst)[c] = q;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(peers.done, 1) == static_cast<int>(gridDim.x) - 1;
    __syncthreads();
    if (s_last && threadIdx.x == 0) {
        __threadfence_system();
        const int e = *peers.epoch;
        for (int d = 0; d < G; ++d) peers.signals[d][G + me] = send_counts[d];
        __threadfence_system();
        for (int d = 0; d < G; ++d) st_release_sys(peers.signals[d] + me, e);
        *peers.done = 0;
    }
}

// Wait for every source's dispatch flag, then mark the rows past each
// source's count as unused (receiver-local id = experts / ranks).
__global__ void p2p_receive_kernel(DramaB200EpPeers peers, int32_t* status) {
    __shared__ int s_count[kMaxEpRanks];
    const int G = peers.ranks, me = peers.rank, tid = threadIdx.x;
    const int32_t* sig = peers.signals[me];
    const int e = *peers.epoch;
    if (tid < G) {
        if (!wait_flag(sig + tid, e) && status) atomicOr(status + 2, 1);
        s_count[tid] = ld_acquire_sys(sig + G + tid);
    }
    __syncthreads();
    const int64_t cap = peers.capacity, stride = peers.hidden + 8;
    const int unused = peers.experts / G;
    __nv_bfloat16* recv = static_cast<__nv_bfloat16*>(peers.recv[me]);
    for (int64_t r = tid; r < G * cap; r += blockDim.x) {
        const int64_t s = r / cap, j = r - s * cap;
        if (j >= s_count[s]) *reinterpret_cast<int32_t*>(recv + r * stride + peers.hidden) = unused;
    }
}

// After the second GEMM stored this rank's results into the sources' back
// buffers (and fenced them): publish the return flags.
__global__ void p2p_signal_back_kernel(DramaB200EpPeers peers) {
    const int G = peers.ranks, me = peers.rank;
    __threadfence_system();
    const int e = *peers.epoch;
    for (int d = 0; d < G; ++d) st_release_sys(peers.signals[d] + 2 * G + me, e);
}

__global__ void p2p_wait_back_kernel(DramaB200EpPeers peers, int32_t* status) {
    const int G = peers.ranks, me = peers.rank, tid = threadIdx.x;
    const int e = *peers.epoch;
    if (tid < G && !wait_flag(peers.signals[me] + 2 * G + tid, e) && status) atomicOr(status + 2, 2);
}

int pack_grid(int64_t work, int sm_count) {
    const int64_t blocks = (work + 255) / 256;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(sm_count) * 4)));
}

}  // namespace

cudaError_t ep_p2p_dispatch_launch(const DramaB200EpPeers& peers, const void* hidden, int64_t tokens,
                                   const void* ids, int ids_dtype, int top_k, const int32_t* placement,
                                   int32_t* pair_rows, int32_t* scratch, int32_t* status, int sm_count,
                                   cudaStream_t s) {
    const int64_t pairs = tokens * top_k;
    int32_t* pair_tags = scratch;
    int32_t* send_counts = scratch + pairs;
    p2p_plan_kernel<<<1, kPlanThreads, 0, s>>>(ids, ids_dtype, pairs, peers.experts, peers.ranks, placement,
                                               peers.capacity, peers.epoch, pair_rows, pair_tags, send_counts,
                                               status);
    p2p_pack_kernel<<<pack_grid(pairs * (peers.hidden / 8 + 1), sm_count), 256, 0, s>>>(
        peers, static_cast<const __nv_bfloat16*>(hidden), pairs, top_k, pair_rows, pair_tags, send_counts);
    return cudaGetLastError();
}

cudaError_t ep_p2p_receive_launch(const DramaB200EpPeers& peers, int32_t* status, cudaStream_t s) {
    p2p_receive_kernel<<<1, 256, 0, s>>>(peers, status);
    return cudaGetLastError();
}

cudaError_t ep_p2p_signal_back_launch(const DramaB200EpPeers& peers, cudaStream_t s) {
    p2p_signal_back_kernel<<<1, 1, 0, s>>>(peers);
    return cudaGetLastError();
}

cudaError_t ep_p2p_wait_back_launch(const DramaB200EpPeers& peers, int32_t* status, cudaStream_t s) {
    p2p_wait_back_kernel<<<1, 32, 0, s>>>(peers, status);
    return cudaGetLastError();
}

}  // namespace drama
