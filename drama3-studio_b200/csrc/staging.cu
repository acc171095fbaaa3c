// Host -> HBM expert staging on a copy stream (the transfer half of the
// reference's _StagingPool.stage, src/drama_low_vram/offload.py:543-651).
//
// The reference gathers the requested experts into a pinned host buffer and
// then issues one H2D copy on the compute stream (offload.py:596-636), so the
// DMA and the expert kernels serialise. Here the caller's host store is itself
// page-locked (cudaHostAlloc'd, or cudaHostRegister'ed over an mmap), each
// expert's bytes go straight from the store into its arena slot, copies that
// continue one another in both address spaces are merged into one DMA, and
// everything runs on a caller-chosen copy stream bracketed by events, so the
// compute stream only waits for the bytes it is about to read.
//
// A pageable source would turn cudaMemcpyAsync into a staged, synchronous
// copy and quietly remove the overlap, so it is rejected instead; so is a
// source that starts in a window registered here and runs past its end, and
// no merged DMA crosses from one registered window into another.
#include <unistd.h>

#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace drama {
namespace {

// Windows page-locked through drama_b200_host_register: [start, end).
std::mutex g_windows_mutex;
std::map<uintptr_t, uintptr_t> g_windows;

// The registered window holding byte p, or {0, 0} when p lies in none of them
// (memory page-locked by its allocator, e.g. cudaHostAlloc).
std::pair<uintptr_t, uintptr_t> window_of(const void* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    std::lock_guard<std::mutex> lock(g_windows_mutex);
    auto it = g_windows.upper_bound(a);
    if (it == g_windows.begin()) return {0, 0};
    --it;
    if (a < it->second) return {it->first, it->second};
    return {0, 0};
}

int pointer_kind(const void* p, cudaMemoryType* type, int* device) {
    cudaPointerAttributes attr{};
    const cudaError_t err = cudaPointerGetAttributes(&attr, p);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail("cudaPointerGetAttributes(%p): %s", p, cudaGetErrorString(err));
    }
    *type = attr.type;
    *device = attr.device;
    return 0;
}

}  // namespace
}  // namespace drama

using namespace drama;

extern "C" {

int drama_b200_stage_copies(const void* const* host_src, void* const* dev_dst, const uint64_t* bytes, int count,
                            void* copy_stream, void* wait_event, void* done_event) {
    if (count < 0) return fail("copy count must be non-negative, got %d", count);
    if (count > 0 && (!host_src || !dev_dst || !bytes)) return fail("copy arrays must not be null");
    int dst_device = -1;
    for (int i = 0; i < count; ++i) {
        if (!host_src[i] || !dev_dst[i]) return fail("copy %d has a null pointer", i);
        if (bytes[i] == 0) return fail("copy %d has zero bytes", i);
        cudaMemoryType type;
        int device = -1;
        // both ends: a registered range may cover the start of a source but not its end
        const void* last = static_cast<const char*>(host_src[i]) + (bytes[i] - 1);
        for (const void* q : {host_src[i], last}) {
            if (pointer_kind(q, &type, &device)) return -1;
            if (type != cudaMemoryTypeHost)
                return fail("copy %d: source byte %p is not page-locked host memory (pin it or cudaHostRegister it)",
                            i, q);
        }
        // a source that starts in a registered window must end in it: the bytes
        // after it may belong to another registration or none, and a DMA across
        // the boundary would turn into a staged, synchronous copy
        const auto window = window_of(host_src[i]);
        if (window.second && reinterpret_cast<uintptr_t>(last) >= window.second)
            return fail("copy %d: source runs past the end of its registered host window", i);
        if (pointer_kind(dev_dst[i], &type, &device)) return -1;
        if (type != cudaMemoryTypeDevice) return fail("copy %d: destination %p is not device memory", i, dev_dst[i]);
        if (dst_device < 0) dst_device = device;
        if (device != dst_device) return fail("copy %d: destinations span devices %d and %d", i, dst_device, device);
    }
    cudaStream_t stream = static_cast<cudaStream_t>(copy_stream);
    if (wait_event) {
        const cudaError_t err = cudaStreamWaitEvent(stream, static_cast<cudaEvent_t>(wait_event), 0);
        if (err != cudaSuccess) return fail("cudaStreamWaitEvent: %s", cudaGetErrorString(err));
    }
    int i = 0;
    while (i < count) {
        const char* src = static_cast<const char*>(host_src[i]);
        char* dst = static_cast<char*>(dev_dst[i]);
        uint64_t run = bytes[i];
        int j = i + 1;
        // merge copies that continue one another in both address spaces and
        // lie in the same registered window (or both in allocator-pinned memory)
        const auto window = window_of(src);
        while (j < count && static_cast<const char*>(host_src[j]) == src + run &&
               static_cast<char*>(dev_dst[j]) == dst + run && window_of(host_src[j]) == window) {
            run += bytes[j];
            ++j;
        }
        const cudaError_t err = cudaMemcpyAsync(dst, src, run, cudaMemcpyHostToDevice, stream);
        if (err != cudaSuccess) return fail("cudaMemcpyAsync of %llu bytes: %s", (unsigned long long)run,
                                            cudaGetErrorString(err));
        i = j;
    }
    if (done_event) {
        const cudaError_t err = cudaEventRecord(static_cast<cudaEvent_t>(done_event), stream);
        if (err != cudaSuccess) return fail("cudaEventRecord: %s", cudaGetErrorString(err));
    }
    return 0;
}

int drama_b200_host_register(void* host_ptr, uint64_t bytes, int read_only, void** registered_base,
                              uint64_t* registered_bytes) {
    if (!host_ptr || bytes == 0) return fail("host_ptr and a non-zero byte count are required");
    if (!registered_base || !registered_bytes) return fail("registered_base and registered_bytes are required");
    const long page = sysconf(_SC_PAGESIZE);
    if (page <= 0) return fail("sysconf(_SC_PAGESIZE) failed");
    const uintptr_t p = reinterpret_cast<uintptr_t>(host_ptr);
    const uintptr_t start = p / page * page;
    const uintptr_t end = (p + bytes + page - 1) / page * page;
    unsigned flags = cudaHostRegisterPortable;
    if (read_only) {
        int dev = 0, supported = 0;
        cudaError_t err = cudaGetDevice(&dev);
        if (err == cudaSuccess) err = cudaDeviceGetAttribute(&supported, cudaDevAttrHostRegisterReadOnlySupported, dev);
        if (err != cudaSuccess) return fail("querying read-only host registration: %s", cudaGetErrorString(err));
        if (!supported) return fail("device %d cannot register read-only host memory", dev);
        flags |= cudaHostRegisterReadOnly;
    }
    const cudaError_t err = cudaHostRegister(reinterpret_cast<void*>(start), end - start, flags);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail("cudaHostRegister of %llu bytes at %p: %s", (unsigned long long)(end - start),
                    reinterpret_cast<void*>(start), cudaGetErrorString(err));
    }
    {
        std::lock_guard<std::mutex> lock(g_windows_mutex);
        g_windows[start] = end;
    }
    *registered_base = reinterpret_cast<void*>(start);
    *registered_bytes = end - start;
    return 0;
}

int drama_b200_host_locked(const void* host_ptr, uint64_t bytes, int* locked) {
    if (!locked) return fail("locked is required");
    *locked = 0;
    if (!host_ptr || bytes == 0) return fail("host_ptr and a non-zero byte count are required");
    const void* last = static_cast<const char*>(host_ptr) + (bytes - 1);
    for (const void* q : {host_ptr, last}) {
        cudaPointerAttributes attr{};
        if (cudaPointerGetAttributes(&attr, q) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        if (attr.type != cudaMemoryTypeHost) return 0;
    }
    *locked = 1;
    return 0;
}

int drama_b200_host_unregister(void* registered_base) {
    if (!registered_base) return fail("registered_base is required");
    const cudaError_t err = cudaHostUnregister(registered_base);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail("cudaHostUnregister(%p): %s", registered_base, cudaGetErrorString(err));
    }
    std::lock_guard<std::mutex> lock(g_windows_mutex);
    g_windows.erase(reinterpret_cast<uintptr_t>(registered_base));
    return 0;
}

}  // extern "C"
