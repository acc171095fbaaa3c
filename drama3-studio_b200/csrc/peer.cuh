// System-scope flags between GPUs that map each other's memory (CUDA IPC):
// release stores, acquire loads and a wait bounded in global time.
#pragma once

#include "common.cuh"

namespace drama {

constexpr unsigned long long kPeerWaitNs = 2000000000ull;  // default limit of a wait: 2 s

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
// Spin until *flag == want or limit_ns pass; false on timeout.
__device__ __forceinline__ bool wait_flag(const int32_t* flag, int want, unsigned long long limit_ns) {
    const unsigned long long start = global_ns();
    while (ld_acquire_sys(flag) != want) {
        if (global_ns() - start > limit_ns) return false;
        __nanosleep(200);
    }
    return true;
}

// Flags one kernel waits for before it reads peer-written data: threads
// t < ranks of every CTA wait for flags[t] == *epoch, then the CTA syncs.
// A wait gives up after limit_ns and ORs `bit` into status[2] (status may be
// null).
struct PeerWait {
    const int32_t* flags = nullptr;  // null: nothing to wait for
    const int32_t* epoch = nullptr;
    int ranks = 0;
    int bit = 0;
    int32_t* status = nullptr;
    unsigned long long limit_ns = kPeerWaitNs;
};

// The wait limit a peer descriptor asks for: wait_ns, or the default when 0.
__host__ __device__ inline unsigned long long peer_wait_limit(int64_t wait_ns) {
    return wait_ns > 0 ? static_cast<unsigned long long>(wait_ns) : kPeerWaitNs;
}

__device__ __forceinline__ void peer_wait_cta(const PeerWait& w) {
    if (!w.flags) return;
    if (static_cast<int>(threadIdx.x) < w.ranks) {
        if (!wait_flag(w.flags + threadIdx.x, *w.epoch, w.limit_ns) && w.status) atomicOr(w.status + 2, w.bit);
    }
    __syncthreads();
}

}  // namespace drama
