// extern "C" entry points: validation first, then launches on the caller's
// stream. Status/error conventions follow the reference's native ABI v1
// (native/src/runtime.cpp:278-290: status 0/-1 plus a thread-local message).
#include <cuda.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace drama {

namespace {
thread_local std::string g_error;
int g_sm_count[64] = {0};

bool float_dtype(int d) { return d == DRAMA_B200_F32 || d == DRAMA_B200_F16 || d == DRAMA_B200_BF16; }
bool index_dtype(int d) { return d == DRAMA_B200_I32 || d == DRAMA_B200_I64; }
size_t dtype_size(int d) {
    switch (d) {
        case DRAMA_B200_F32: case DRAMA_B200_I32: return 4;
        case DRAMA_B200_I64: return 8;
        default: return 2;
    }
}
bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
    if (!a || !b || !na || !nb) return false;
    const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + nb && y < x + na;
}
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count_current(int* out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return fail("cudaGetDevice: %s", cudaGetErrorString(err));
    if (dev < 0 || dev >= 64) return fail("device ordinal %d out of range", dev);
    if (!g_sm_count[dev]) {
        int major = 0, count = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        err = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
        if (err != cudaSuccess) return fail("device query: %s", cudaGetErrorString(err));
        if (major != 10) return fail("device %d is sm_%d0; this library is built for sm_100a only", dev, major);
        g_sm_count[dev] = count;
    }
    *out = g_sm_count[dev];
    return 0;
}
}  // namespace

void set_error(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_error = buf;
}

int fail(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_error = buf;
    return -1;
}

int check_launch(const char* what) {
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail("%s launch failed: %s", what, cudaGetErrorString(err));
    return 0;
}

namespace {

int validate_decode_common(const void* x, int x_dtype, int64_t tokens, int top_k, const void* ids,
                           int ids_dtype, const void* weights, int weights_dtype, const void* out,
                           const float* pair_out, int hidden, int intermediate, int slots,
                           int64_t max_pairs = kMaxDecodePairs, const char* path = "decode") {
    if (!x || !ids || !weights) return fail("x, ids and weights are required");
    if (!out && !pair_out) return fail("either out or pair_out is required");
    if (!float_dtype(x_dtype)) return fail("x must be float32, float16 or bfloat16");
    if (!float_dtype(weights_dtype)) return fail("routing weights must be floating point");
    if (!index_dtype(ids_dtype)) return fail("expert IDs must be int32 or int64");
    if (tokens < 0 || top_k < 1) return fail("tokens must be >= 0 and top_k >= 1");
    if (tokens * top_k > max_pairs)
        return fail("%s supports at most %lld (token, slot) pairs; got %lld", path, static_cast<long long>(max_pairs),
                    static_cast<long long>(tokens * top_k));
    if (hidden < 128 || hidden % 128 || intermediate < 128 || intermediate % 128)
        return fail("hidden and intermediate must be positive multiples of 128");
    if (slots < 1 || slots > kMaxSlots) return fail("slots must be in [1, %d]", kMaxSlots);
    const size_t xb = static_cast<size_t>(tokens) * hidden * dtype_size(x_dtype);
    if (out && overlaps(out, xb, x, xb)) return fail("output must not overlap the hidden states");
    if (pair_out && overlaps(pair_out, static_cast<size_t>(tokens) * top_k * hidden * 4, x, xb))
        return fail("pair output must not overlap the hidden states");
    return 0;
}

// Validation and argument block of the FP8 decode entry points (with a
// workspace or with the library's static scratch).
int prepare_fp8_decode(const DramaB200Fp8Bank* bank, const void* x, int x_dtype, int64_t tokens, int top_k,
                       const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                       float* pair_out, DecodeArgs* out_args, int64_t max_pairs = kMaxDecodePairs,
                       const char* path = "decode") {
    if (!bank) return fail("bank is required");
    const DramaB200Fp8Bank& b = *bank;
    if (validate_decode_common(x, x_dtype, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out, pair_out,
                               b.hidden, b.intermediate, b.slots, max_pairs, path))
        return -1;
    if (!b.w13 || !b.w13_scale || !b.w2 || !b.w2_scale) return fail("FP8 bank pointers are required");
    if (!aligned16(b.w13) || !aligned16(b.w2) || b.w13_row_stride % 16 || b.w2_row_stride % 16 ||
        b.w13_slot_stride % 16 || b.w2_slot_stride % 16)
        return fail("FP8 weight rows must start on 16-byte boundaries");
    if (b.w13_row_stride < b.hidden || b.w2_row_stride < b.intermediate ||
        b.w13_slot_stride < b.w13_row_stride * 2 * b.intermediate ||
        b.w2_slot_stride < b.w2_row_stride * b.hidden)
        return fail("FP8 weight strides are smaller than the bank geometry");
    if (b.w13_scale_row_stride < b.hidden / 128 || b.w2_scale_row_stride < b.intermediate / 128)
        return fail("FP8 scale strides are smaller than the bank geometry");
    DecodeArgs& a = *out_args;
    a = DecodeArgs{};
    a.format = 0;
    a.fp8 = b;
    a.x = x;
    a.x_dtype = x_dtype;
    a.tokens = tokens;
    a.top_k = top_k;
    a.ids = ids;
    a.ids_dtype = ids_dtype;
    a.weights = weights;
    a.weights_dtype = weights_dtype;
    a.out = out;
    a.pair_out = pair_out;
    a.hidden = b.hidden;
    a.intermediate = b.intermediate;
    a.slots = b.slots;
    return 0;
}

// Scratch need of a decode call on the current device (0 on failure, with the error set).
size_t decode_scratch_need(const DecodeArgs& a, int* sms) {
    if (sm_count_current(sms)) return 0;
    return decode_workspace_layout(a.tokens, a.top_k, a.hidden, a.intermediate, *sms, 0, nullptr, nullptr);
}

int finish_decode(DecodeArgs& a, void* workspace, size_t workspace_bytes, void* stream) {
    if (a.tokens == 0) return 0;
    int sms = 0;
    const size_t need = decode_scratch_need(a, &sms);
    if (!need) return -1;
    if (!workspace || workspace_bytes < need)
        return fail("decode workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    decode_workspace_layout(a.tokens, a.top_k, a.hidden, a.intermediate, sms, 0, static_cast<char*>(workspace), &a.ws);
    a.ctas = sms * kDecodeCtasPerSm;
    const cudaError_t err = decode_launch(a, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("decode launch failed: %s", cudaGetErrorString(err));
    return 0;
}

}  // namespace
}  // namespace drama

using namespace drama;

extern "C" {

int drama_b200_abi(void) { return DRAMA_B200_ABI_VERSION; }

const char* drama_b200_error(void) { return g_error.c_str(); }

int drama_b200_device_check(int device, int* sm_count) {
    cudaDeviceProp prop;
    const cudaError_t err = cudaGetDeviceProperties(&prop, device);
    if (err != cudaSuccess) return fail("cudaGetDeviceProperties(%d): %s", device, cudaGetErrorString(err));
    if (prop.major != 10) return fail("device %d (%s) is sm_%d%d; drama_b200 needs sm_100", device, prop.name, prop.major, prop.minor);
    if (sm_count) *sm_count = prop.multiProcessorCount;
    return 0;
}

int drama_b200_route_topk(const void* logits, int logits_dtype, int64_t tokens, int experts, int top_k,
                          int renormalize, void* ids, int ids_dtype, void* weights, int weights_dtype,
                          void* stream) {
    if (!logits || !ids || !weights) return fail("logits, ids and weights are required");
    if (!float_dtype(logits_dtype) || !float_dtype(weights_dtype)) return fail("logits/weights dtype must be floating point");
    if (!index_dtype(ids_dtype)) return fail("ids must be int32 or int64");
    if (tokens < 0 || experts < 1 || experts > 1024) return fail("experts must be in [1, 1024]");
    if (top_k < 1 || top_k > 32 || top_k > experts) return fail("top_k must be in [1, min(32, experts)]");
    if (renormalize != 0 && renormalize != 1) return fail("renormalize must be 0 or 1");
    const size_t lb = static_cast<size_t>(tokens) * experts * dtype_size(logits_dtype);
    if (overlaps(ids, tokens * top_k * dtype_size(ids_dtype), logits, lb) ||
        overlaps(weights, tokens * top_k * dtype_size(weights_dtype), logits, lb))
        return fail("router outputs must not overlap the logits");
    if (tokens == 0) return 0;
    RouteArgs a{logits, logits_dtype, tokens, experts, top_k, renormalize, ids, ids_dtype, weights, weights_dtype};
    const cudaError_t err = route_topk(a, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("route_topk launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_permute_routes(const void* ids, int ids_dtype, int64_t pairs, int experts, int64_t* order,
                              int64_t* counts, int64_t* offsets, int32_t* status, void* stream) {
    if (!ids || !order || !counts || !offsets) return fail("ids, order, counts and offsets are required");
    if (!index_dtype(ids_dtype)) return fail("ids must be int32 or int64");
    if (pairs < 0 || pairs > (int64_t(1) << 24)) return fail("pairs must be in [0, 2^24]");
    if (experts < 1 || experts > 1024) return fail("experts must be in [1, 1024]");
    PermuteArgs a{ids, ids_dtype, pairs, experts, order, counts, offsets, status};
    const cudaError_t err = permute_routes(a, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("permute_routes launch failed: %s", cudaGetErrorString(err));
    return 0;
}

size_t drama_b200_permute_routes_wide_scratch_bytes(int64_t pairs, int experts) {
    return pairs < 0 || experts < 1 ? 0 : permute_wide_scratch_bytes(pairs, experts);
}

int drama_b200_permute_routes_wide(const void* ids, int ids_dtype, int64_t pairs, int experts, int64_t* order,
                                   int64_t* counts, int64_t* offsets, int64_t* position, void* scratch,
                                   size_t scratch_bytes, int32_t* status, void* stream) {
    if (!ids || !order || !counts || !offsets) return fail("ids, order, counts and offsets are required");
    if (!index_dtype(ids_dtype)) return fail("ids must be int32 or int64");
    if (pairs < 0 || pairs > (int64_t(1) << 24)) return fail("pairs must be in [0, 2^24]");
    if (experts < 1 || experts > 1024) return fail("experts must be in [1, 1024]");
    const size_t need = permute_wide_scratch_bytes(pairs, experts);
    if (need && (!scratch || scratch_bytes < need))
        return fail("permutation scratch too small: need %zu bytes, got %zu", need, scratch_bytes);
    if (scratch && !aligned16(scratch)) return fail("scratch must be 16-byte aligned");
    PermuteArgs a{ids, ids_dtype, pairs, experts, order, counts, offsets, status};
    const cudaError_t err = permute_routes_wide(a, static_cast<int*>(scratch), position,
                                                static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("permute_routes_wide launch failed: %s", cudaGetErrorString(err));
    return 0;
}

size_t drama_b200_decode_workspace_bytes(int64_t tokens, int top_k, int hidden, int intermediate) {
    int sms = 0;
    if (sm_count_current(&sms)) sms = 148;
    const size_t decode = decode_workspace_layout(tokens, top_k, hidden, intermediate, sms, 0, nullptr, nullptr);
    // the bf16 INT4 path runs on the W8A8 schedule and its scratch
    const size_t rows = w8a8_workspace_layout(tokens, top_k, hidden, intermediate, nullptr, nullptr);
    return decode > rows ? decode : rows;
}

size_t drama_b200_decode_status_offset(void) { return 0; }

int drama_b200_fp8_decode(const DramaB200Fp8Bank* bank, const void* x, int x_dtype, int64_t tokens,
                          int top_k, const void* ids, int ids_dtype, const void* weights, int weights_dtype,
                          void* out, float* pair_out, void* workspace, size_t workspace_bytes, void* stream) {
    DecodeArgs a{};
    if (prepare_fp8_decode(bank, x, x_dtype, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out, pair_out,
                           &a))
        return -1;
    return finish_decode(a, workspace, workspace_bytes, stream);
}

size_t drama_b200_fp8_w8a8_workspace_bytes(int64_t tokens, int top_k, int hidden, int intermediate) {
    return fp8_w8a8_workspace_layout(tokens, top_k, hidden, intermediate, nullptr, nullptr);
}

int drama_b200_fp8_w8a8_decode(const DramaB200Fp8Bank* bank, const void* x, int64_t tokens, int top_k,
                               const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                               float* pair_out, void* x_fp8_out, float* x_scale_out, void* workspace,
                               size_t workspace_bytes, void* stream) {
    DecodeArgs a{};
    if (prepare_fp8_decode(bank, x, DRAMA_B200_BF16, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out,
                           pair_out, &a))
        return -1;
    if (tokens == 0) return 0;
    const size_t need = fp8_w8a8_workspace_layout(tokens, top_k, a.hidden, a.intermediate, nullptr, nullptr);
    if (!workspace || workspace_bytes < need)
        return fail("W8A8 workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    Fp8W8a8Workspace ws;
    fp8_w8a8_workspace_layout(tokens, top_k, a.hidden, a.intermediate, static_cast<char*>(workspace), &ws);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = fp8_w8a8_launch(a.fp8, x, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out, pair_out,
                                      ws, s);
    if (err == cudaSuccess && x_fp8_out)
        err = cudaMemcpyAsync(x_fp8_out, ws.xq, static_cast<size_t>(tokens) * a.hidden, cudaMemcpyDeviceToDevice, s);
    if (err == cudaSuccess && x_scale_out)
        err = cudaMemcpyAsync(x_scale_out, ws.xs, static_cast<size_t>(tokens) * (a.hidden / 128) * 4,
                              cudaMemcpyDeviceToDevice, s);
    if (err != cudaSuccess) return fail("W8A8 decode launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_fp8_w8a8_prefill_supported(int hidden, int intermediate, int experts) {
    return fp8_prefill_tc_supported(hidden, intermediate, experts) ? 1 : 0;
}

size_t drama_b200_fp8_w8a8_prefill_workspace_bytes(int64_t tokens, int top_k, int hidden, int intermediate,
                                                   int experts) {
    return fp8_prefill_tc_workspace_layout(tokens, top_k, hidden, intermediate, experts, nullptr, nullptr) + 1024;
}

int drama_b200_fp8_w8a8_prefill(const DramaB200Fp8Bank* bank, const void* x, int64_t tokens, int top_k,
                                const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                                float* pair_out, void* workspace, size_t workspace_bytes, void* stream) {
    DecodeArgs a{};
    if (prepare_fp8_decode(bank, x, DRAMA_B200_BF16, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out,
                           pair_out, &a, kMaxPrefillPairs, "the W8A8 prefill"))
        return -1;
    if (top_k > 32) return fail("the W8A8 prefill takes top_k in [1, 32]");
    if (!fp8_prefill_tc_supported(a.hidden, a.intermediate, a.slots))
        return fail("the tcgen05 prefill needs hidden a multiple of 256, hidden and intermediate <= 2048, "
                    "intermediate a multiple of 128 and at most 512 experts");
    if (tokens == 0) return 0;
    // the buffers start on 1024-byte boundaries: up to 1023 bytes of the workspace lead in
    const size_t need = fp8_prefill_tc_workspace_layout(tokens, top_k, a.hidden, a.intermediate, a.slots, nullptr,
                                                        nullptr) + 1024;
    if (!workspace || workspace_bytes < need)
        return fail("W8A8 prefill workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(workspace) + 1023) & ~uintptr_t(1023));
    if (pair_out && (reinterpret_cast<uintptr_t>(pair_out) & 31u)) return fail("pair_out must be 32-byte aligned");
    if (!aligned16(x)) return fail("hidden rows must start on 16-byte boundaries");
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    Fp8PrefillWorkspace ws;
    fp8_prefill_tc_workspace_layout(tokens, top_k, a.hidden, a.intermediate, a.slots, base, &ws);
    const cudaError_t err = fp8_prefill_tc_launch(a.fp8, x, tokens, top_k, ids, ids_dtype, weights, weights_dtype,
                                                  out, pair_out, ws, sms, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("W8A8 prefill launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_int4_decode(const DramaB200Int4Bank* bank, const void* x, int x_dtype, int64_t tokens,
                           int top_k, const void* ids, int ids_dtype, const void* weights, int weights_dtype,
                           void* out, float* pair_out, void* workspace, size_t workspace_bytes, void* stream) {
    if (!bank) return fail("bank is required");
    const DramaB200Int4Bank& b = *bank;
    if (validate_decode_common(x, x_dtype, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out, pair_out,
                               b.hidden, b.intermediate, b.slots))
        return -1;
    if (!b.w13 || !b.w13_scale || !b.w2 || !b.w2_scale) return fail("INT4 bank pointers are required");
    if (b.scale_dtype != DRAMA_B200_BF16 && b.scale_dtype != DRAMA_B200_F16)
        return fail("INT4 scales must be bfloat16 or float16");
    if (!aligned16(b.w13) || !aligned16(b.w2) || b.w13_row_stride % 4 || b.w2_row_stride % 4 ||
        b.w13_slot_stride % 4 || b.w2_slot_stride % 4)
        return fail("INT4 weight rows must start on 16-byte boundaries");
    if (b.w13_row_stride < b.hidden / 8 || b.w2_row_stride < b.intermediate / 8 ||
        b.w13_slot_stride < b.w13_row_stride * 2 * b.intermediate ||
        b.w2_slot_stride < b.w2_row_stride * b.hidden)
        return fail("INT4 weight strides are smaller than the bank geometry");
    if (x_dtype == DRAMA_B200_BF16 && b.hidden % 256 == 0 && b.intermediate % 256 == 0) {
        // bf16 rows: grouping + split-K GEMVs with the reference's per-element bf16 weights
        if (tokens == 0) return 0;
        int sms = 0;
        if (sm_count_current(&sms)) return -1;
        const size_t need = w8a8_workspace_layout(tokens, top_k, b.hidden, b.intermediate, nullptr, nullptr);
        if (!workspace || workspace_bytes < need)
            return fail("decode workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
        if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
        W8a8Workspace ws{};
        w8a8_workspace_layout(tokens, top_k, b.hidden, b.intermediate, static_cast<char*>(workspace), &ws);
        const cudaError_t err =
            int4_layer_supported(tokens, top_k, b, x_dtype)
                // one row of the reference's shape: the whole layer in one launch
                ? int4_layer_launch(b, x, ids, ids_dtype, weights, weights_dtype, out, x_dtype, pair_out,
                                    ws.layer_part, ws.layer_tickets, ws.status, static_cast<cudaStream_t>(stream))
                : int4_rows_launch(b, x, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out, x_dtype,
                                   pair_out, ws, sms, static_cast<cudaStream_t>(stream));
        if (err != cudaSuccess) return fail("INT4 launch failed: %s", cudaGetErrorString(err));
        return 0;
    }
    DecodeArgs a{};
    a.format = 1;
    a.int4 = b;
    a.x = x;
    a.x_dtype = x_dtype;
    a.tokens = tokens;
    a.top_k = top_k;
    a.ids = ids;
    a.ids_dtype = ids_dtype;
    a.weights = weights;
    a.weights_dtype = weights_dtype;
    a.out = out;
    a.pair_out = pair_out;
    a.hidden = b.hidden;
    a.intermediate = b.intermediate;
    a.slots = b.slots;
    return finish_decode(a, workspace, workspace_bytes, stream);
}

size_t drama_b200_w8a8_workspace_bytes(int64_t tokens, int top_k, int hidden, int intermediate) {
    return w8a8_workspace_layout(tokens, top_k, hidden, intermediate, nullptr, nullptr);
}

int drama_b200_w8a8_decode(const DramaB200W8a8Bank* bank, const void* x, int x_dtype, int64_t tokens, int top_k,
                           const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                           float* pair_out, void* workspace, size_t workspace_bytes, void* stream) {
    if (!bank) return fail("bank is required");
    const DramaB200W8a8Bank& b = *bank;
    if (validate_decode_common(x, x_dtype, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out, pair_out,
                               b.hidden, b.intermediate, b.slots))
        return -1;
    if (x_dtype != DRAMA_B200_BF16) return fail("W8A8 hidden rows must be bfloat16");
    if (b.mode < 1 || b.mode > 3) return fail("W8A8 mode must be 1, 2 or 3; got %d", b.mode);
    if (b.hidden % 256 || b.intermediate % 256)
        return fail("W8A8 needs hidden and intermediate sizes that are multiples of 256 (ConvRot groups)");
    if (!b.w13 || !b.w13_scale || !b.w2 || !b.w2_scale) return fail("W8A8 bank pointers are required");
    const int H = b.hidden, I = b.intermediate;
    struct RoleCheck { const char* name; const void* w; const void* sc; int64_t ws, wr, ss, sr; int n, k; };
    const RoleCheck roles[2] = {
        {"w13", b.w13, b.w13_scale, b.w13_slot_stride, b.w13_row_stride, b.w13_scale_slot_stride,
         b.w13_scale_row_stride, 2 * I, H},
        {"w2", b.w2, b.w2_scale, b.w2_slot_stride, b.w2_row_stride, b.w2_scale_slot_stride, b.w2_scale_row_stride, H,
         I}};
    for (const RoleCheck& r : roles) {
        const int64_t row_bytes = b.mode == 1 ? r.k : b.mode == 2 ? 3 * static_cast<int64_t>(r.k) / 4 : r.k / 2;
        const int64_t scale_bytes = b.mode == 1 ? 4 : r.k / 16 + (b.mode == 3 ? 8 : 4);
        const int64_t align = b.mode == 1 ? 16 : 8;  // 16-byte rows (mode 1) / 8-byte nibble loads
        if (reinterpret_cast<uintptr_t>(r.w) % align || r.wr % align || r.ws % align)
            return fail("%s weight rows must start on %lld-byte boundaries", r.name, static_cast<long long>(align));
        if (reinterpret_cast<uintptr_t>(r.sc) % 4 || r.sr % 4 || r.ss % 4)
            return fail("%s scale rows must start on 4-byte boundaries", r.name);
        if (r.wr < row_bytes || r.ws < r.wr * r.n || r.sr < scale_bytes || r.ss < r.sr * r.n)
            return fail("%s strides are smaller than the mode-%d bank geometry", r.name, b.mode);
        if (b.mode == 3 && r.n < 16) return fail("%s: the W4A8 codebook needs at least 16 rows", r.name);
    }
    if (tokens == 0) return 0;
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const size_t need = w8a8_workspace_layout(tokens, top_k, H, I, nullptr, nullptr);
    if (!workspace || workspace_bytes < need)
        return fail("W8A8 workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    W8a8Workspace ws{};
    w8a8_workspace_layout(tokens, top_k, H, I, static_cast<char*>(workspace), &ws);
    const cudaError_t err = w8a8_decode_launch(b, x, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out,
                                               x_dtype, pair_out, ws, sms, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("W8A8 launch failed: %s", cudaGetErrorString(err));
    return 0;
}

size_t drama_b200_shared_expert_workspace_bytes(int64_t tokens, int hidden, int intermediate) {
    return shared_expert_workspace_layout(tokens, hidden, intermediate, nullptr, nullptr);
}

int drama_b200_shared_expert(const DramaB200SharedExpert* mlp, const void* x, int64_t tokens, const void* routed,
                             const void* residual, void* out, void* workspace, size_t workspace_bytes, void* stream) {
    if (!mlp) return fail("mlp is required");
    const DramaB200SharedExpert& m = *mlp;
    if (!m.gate_proj || !m.up_proj || !m.down_proj || !m.gate_weight) return fail("shared expert weights are required");
    if (!x || !out) return fail("x and out are required");
    if (tokens < 0 || tokens > kMaxSharedTokens) return fail("tokens must be in [0, %d]", kMaxSharedTokens);
    if (m.hidden < 128 || m.hidden % 128 || m.intermediate < 128 || m.intermediate % 128)
        return fail("hidden and intermediate must be positive multiples of 128");
    const void* rows[3] = {m.gate_proj, m.up_proj, m.down_proj};
    const int64_t strides[3] = {m.gate_row_stride, m.up_row_stride, m.down_row_stride};
    const int64_t widths[3] = {m.hidden, m.hidden, m.intermediate};
    for (int i = 0; i < 3; ++i) {
        if (!aligned16(rows[i]) || strides[i] % 8) return fail("weight rows must start on 16-byte boundaries");
        if (strides[i] < widths[i]) return fail("a weight row stride is smaller than its row");
    }
    const void* acts[4] = {x, routed, residual, out};
    for (const void* p : acts)
        if (p && !aligned16(p)) return fail("activation rows must be 16-byte aligned");
    const size_t xb = static_cast<size_t>(tokens) * m.hidden * 2;
    if (overlaps(out, xb, x, xb)) return fail("output must not overlap x");
    if (tokens == 0) return 0;
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const size_t need = shared_expert_workspace_layout(tokens, m.hidden, m.intermediate, nullptr, nullptr);
    if (!workspace || workspace_bytes < need)
        return fail("shared expert workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    SharedWorkspace ws{};
    shared_expert_workspace_layout(tokens, m.hidden, m.intermediate, static_cast<char*>(workspace), &ws);
    const cudaError_t err = shared_expert_launch(m, x, tokens, routed, residual, out, ws, sms,
                                                 static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("shared expert launch failed: %s", cudaGetErrorString(err));
    return 0;
}

size_t drama_b200_moe_layer_workspace_bytes(int64_t tokens, int top_k, int hidden, int intermediate,
                                             int experts) {
    int sms = 0;
    if (sm_count_current(&sms)) sms = 148;
    return decode_workspace_layout(tokens, top_k, hidden, intermediate, sms, experts, nullptr, nullptr);
}

namespace {
// Validation and argument blocks shared by the fused layer entry points.
int prepare_moe_layer(const DramaB200Fp8Bank* bank, const void* gate, const void* next_gate, const float* gamma,
                      float eps, const void* hidden_in, void* hidden_out, int64_t tokens, int top_k,
                      int64_t* ids_out, void* weights_out, void* normed_out, void* moe_out, void* workspace,
                      size_t workspace_bytes, MoeLayerArgs* m, DecodeArgs* d) {
    if (!bank || !gate || !gamma || !hidden_in || !hidden_out) return fail("bank, gate, gamma and hidden buffers are required");
    const DramaB200Fp8Bank& b = *bank;
    const int H = b.hidden, E = b.slots;
    if (tokens < 0 || top_k < 1 || top_k > 32 || top_k > E) return fail("top_k must be in [1, min(32, experts)]");
    if (tokens * top_k > kMaxLayerPairs) return fail("the fused MoE layer supports at most %d (token, slot) pairs", kMaxLayerPairs);
    if (H % 256 || H < 256 || H > 4096 || b.intermediate % 128 || b.intermediate < 128)
        return fail("hidden must be a multiple of 256 up to 4096 and intermediate a multiple of 128");
    if (tokens * H * 4 + 8192 > 200 * 1024) return fail("tokens * hidden too large for the router's shared memory");
    if (E < 1 || E > 1024) return fail("experts must be in [1, 1024]");
    if (!(eps > 0.0f)) return fail("eps must be positive");
    if (!b.w13 || !b.w13_scale || !b.w2 || !b.w2_scale) return fail("FP8 bank pointers are required");
    if (!aligned16(b.w13) || !aligned16(b.w2) || !aligned16(gate) || b.w13_row_stride % 16 || b.w2_row_stride % 16 ||
        b.w13_slot_stride % 16 || b.w2_slot_stride % 16)
        return fail("FP8 weight rows and the router weight must start on 16-byte boundaries");
    if (next_gate && !aligned16(next_gate)) return fail("next router weight must be 16-byte aligned");
    if (!aligned16(hidden_in) || !aligned16(hidden_out) || (normed_out && !aligned16(normed_out)) ||
        (moe_out && !aligned16(moe_out)))
        return fail("hidden, normed and moe rows must start on 16-byte boundaries");
    const size_t hb = static_cast<size_t>(tokens) * H * 2;
    if (overlaps(hidden_out, hb, hidden_in, hb)) return fail("hidden_out must not overlap hidden_in");
    if (tokens == 0) return 1;
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const size_t need = decode_workspace_layout(tokens, top_k, H, b.intermediate, sms, E, nullptr, nullptr);
    if (!workspace || workspace_bytes < need)
        return fail("MoE layer workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    *d = DecodeArgs{};
    decode_workspace_layout(tokens, top_k, H, b.intermediate, sms, E, static_cast<char*>(workspace), &d->ws);
    d->format = 0;
    d->fp8 = b;
    d->x = hidden_in;
    d->x_dtype = DRAMA_B200_BF16;
    d->tokens = tokens;
    d->top_k = top_k;
    d->out = hidden_out;
    d->residual = hidden_in;
    d->moe_out = moe_out;
    d->hidden = H;
    d->intermediate = b.intermediate;
    d->slots = E;
    d->ctas = sms * kDecodeCtasPerSm;
    *m = MoeLayerArgs{};
    m->hidden_in = static_cast<const __nv_bfloat16*>(hidden_in);
    m->hidden_out = static_cast<__nv_bfloat16*>(hidden_out);
    m->gamma = gamma;
    m->gate = static_cast<const __nv_bfloat16*>(gate);
    m->next_gate = static_cast<const __nv_bfloat16*>(next_gate);
    m->eps = eps;
    m->tokens = tokens;
    m->experts = E;
    m->top_k = top_k;
    m->hidden = H;
    m->intermediate = b.intermediate;
    m->ws = d->ws;
    m->ids_out = ids_out;
    m->weights_out = static_cast<__nv_bfloat16*>(weights_out);
    m->normed_out = static_cast<__nv_bfloat16*>(normed_out);
    m->router_ctas = kRouterCtas < E ? kRouterCtas : E;
    return 0;
}
}  // namespace

namespace {
DecodeLayerArgs one_launch_layer(const MoeLayerArgs& m, const DecodeArgs& d, void* moe_out, const void* normed_in,
                                 const void* logits_in) {
    DecodeLayerArgs a{};
    RoutedLayerArgs& r = a.layer;
    r.bank = d.fp8;
    r.hidden_in = m.hidden_in;
    r.hidden_out = m.hidden_out;
    r.gamma = m.gamma;
    r.gate = m.gate;
    r.eps = m.eps;
    r.E = m.experts;
    r.k = m.top_k;
    r.H = m.hidden;
    r.I = m.intermediate;
    r.ws = d.ws;
    r.ids_out = m.ids_out;
    r.weights_out = m.weights_out;
    r.normed_out = m.normed_out;
    r.moe_out = static_cast<__nv_bfloat16*>(moe_out);
    a.normed_in = static_cast<const __nv_bfloat16*>(normed_in);
    a.logits_in = static_cast<const __nv_bfloat16*>(logits_in);
    a.part = d.ws.layer_part;
    a.tickets = d.ws.layer_tickets;
    return a;
}
}  // namespace

int drama_b200_fp8_moe_layer(const DramaB200Fp8Bank* bank, const void* gate, const void* next_gate,
                             const float* gamma, float eps, const void* hidden_in, void* hidden_out,
                             int64_t tokens, int top_k, int64_t* ids_out, void* weights_out,
                             void* normed_out, void* moe_out, void* workspace, size_t workspace_bytes,
                             void* stream) {
    MoeLayerArgs m;
    DecodeArgs d;
    const int st = prepare_moe_layer(bank, gate, next_gate, gamma, eps, hidden_in, hidden_out, tokens, top_k,
                                     ids_out, weights_out, normed_out, moe_out, workspace, workspace_bytes, &m, &d);
    if (st) return st < 0 ? -1 : 0;
    cudaError_t err;
    if (decode_layer_supported(tokens, top_k, m.hidden, m.intermediate, m.experts)) {
        // one hidden row: the whole layer in one launch
        err = decode_layer_launch(one_launch_layer(m, d, moe_out, nullptr, nullptr), static_cast<cudaStream_t>(stream));
    } else if (routed_layer_supported(tokens, top_k, m.hidden, m.intermediate, m.experts)) {
        // one hidden row: router + gate/up and down + combine, two launches
        RoutedLayerArgs r{};
        r.bank = d.fp8;
        r.hidden_in = m.hidden_in;
        r.hidden_out = m.hidden_out;
        r.gamma = m.gamma;
        r.gate = m.gate;
        r.eps = m.eps;
        r.E = m.experts;
        r.k = top_k;
        r.H = m.hidden;
        r.I = m.intermediate;
        r.ws = d.ws;
        r.ids_out = m.ids_out;
        r.weights_out = m.weights_out;
        r.normed_out = m.normed_out;
        r.moe_out = static_cast<__nv_bfloat16*>(moe_out);
        err = routed_layer_launch(r, d.ctas / kDecodeCtasPerSm, static_cast<cudaStream_t>(stream));
    } else {
        err = moe_router_launch(m, static_cast<cudaStream_t>(stream));
        if (err == cudaSuccess) err = decode_experts_launch(d, static_cast<cudaStream_t>(stream));
    }
    if (err != cudaSuccess) return fail("MoE layer launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_moe_layer_launches(int64_t tokens, int top_k, int hidden, int intermediate, int experts) {
    if (decode_layer_supported(tokens, top_k, hidden, intermediate, experts)) return 1;
    if (routed_layer_supported(tokens, top_k, hidden, intermediate, experts)) return 2;
    return 3;
}

int drama_b200_fp8_moe_layer_logits(const DramaB200Fp8Bank* bank, const void* normed, const void* logits,
                                    const void* hidden_in, void* hidden_out, int64_t tokens, int top_k,
                                    int64_t* ids_out, void* weights_out, void* moe_out, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (!normed || !logits) return fail("normed row and router logits are required");
    if (!aligned16(normed) || !aligned16(logits)) return fail("normed row and logits must be 16-byte aligned");
    if (tokens != 1) return fail("the logits-driven layer runs one decode row (tokens == 1), got %lld",
                                 static_cast<long long>(tokens));
    MoeLayerArgs m;
    DecodeArgs d;
    // The router weight and gamma are not read; the normalised row stands in for both pointers.
    const float one = 1.0f;
    const int st = prepare_moe_layer(bank, normed, nullptr, &one, 1e-6f, hidden_in, hidden_out, tokens, top_k,
                                     ids_out, weights_out, nullptr, moe_out, workspace, workspace_bytes, &m, &d);
    if (st) return st < 0 ? -1 : 0;
    if (!decode_layer_supported(tokens, top_k, m.hidden, m.intermediate, m.experts))
        return fail("the logits-driven layer supports hidden %% 512 == 0 up to 2048, intermediate %% 16 == 0, "
                    "top_k <= 16 (got hidden %d, intermediate %d, top_k %d)", m.hidden, m.intermediate, top_k);
    m.gamma = nullptr;
    m.gate = nullptr;
    const cudaError_t err =
        decode_layer_launch(one_launch_layer(m, d, moe_out, normed, logits), static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("MoE layer launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_fp8_moe_router(const DramaB200Fp8Bank* bank, const void* gate, const void* next_gate,
                              const float* gamma, float eps, const void* hidden_in, int64_t tokens, int top_k,
                              int64_t* ids_out, void* weights_out, void* normed_out, void* workspace,
                              size_t workspace_bytes, void* stream) {
    MoeLayerArgs m;
    DecodeArgs d;
    // hidden_out is unused by the router; any non-overlapping pointer passes validation.
    const int st = prepare_moe_layer(bank, gate, next_gate, gamma, eps, hidden_in, workspace, tokens, top_k,
                                     ids_out, weights_out, normed_out, nullptr, workspace, workspace_bytes, &m, &d);
    if (st) return st < 0 ? -1 : 0;
    const cudaError_t err = moe_router_launch(m, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("MoE router launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_fp8_moe_experts(const DramaB200Fp8Bank* bank, const void* hidden_in, void* hidden_out,
                               int64_t tokens, int top_k, void* moe_out, void* workspace, size_t workspace_bytes,
                               void* stream) {
    MoeLayerArgs m;
    DecodeArgs d;
    static const float one = 1.0f;
    const int st = prepare_moe_layer(bank, hidden_in, nullptr, &one, 1e-6f, hidden_in, hidden_out, tokens, top_k,
                                     nullptr, nullptr, nullptr, moe_out, workspace, workspace_bytes, &m, &d);
    if (st) return st < 0 ? -1 : 0;
    const cudaError_t err = decode_experts_launch(d, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("MoE experts launch failed: %s", cudaGetErrorString(err));
    return 0;
}

size_t drama_b200_prefill_workspace_bytes(int64_t tokens, int top_k, int hidden, int intermediate, int experts) {
    return prefill_workspace_layout(tokens, top_k, hidden, intermediate, experts, nullptr, nullptr);
}

size_t drama_b200_prefill_status_offset(void) { return 0; }

int drama_b200_fp8_prefill(const DramaB200Fp8Bank* bank, const void* x, int64_t tokens, int top_k, const void* ids,
                           int ids_dtype, const void* weights, int weights_dtype, void* out, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (!bank || !x || !ids || !weights || !out) return fail("bank, x, ids, weights and out are required");
    const DramaB200Fp8Bank& b = *bank;
    if (!index_dtype(ids_dtype)) return fail("expert IDs must be int32 or int64");
    if (!float_dtype(weights_dtype)) return fail("routing weights must be floating point");
    if (tokens < 0 || top_k < 1 || top_k > 32) return fail("tokens must be >= 0 and top_k in [1, 32]");
    if (tokens * top_k > (int64_t(1) << 24)) return fail("prefill supports at most 2^24 (token, slot) pairs");
    if (b.hidden % 256 || b.hidden < 256 || b.intermediate % 128 || b.intermediate < 128)
        return fail("prefill needs hidden a multiple of 256 and intermediate a multiple of 128");
    if (b.slots < 1 || b.slots > 1024) return fail("slots must be in [1, 1024]");
    if (!b.w13 || !b.w13_scale || !b.w2 || !b.w2_scale) return fail("FP8 bank pointers are required");
    if (!aligned16(b.w13) || !aligned16(b.w2) || !aligned16(x) || !aligned16(out) || b.w13_row_stride % 16 ||
        b.w2_row_stride % 16 || b.w13_slot_stride % 16 || b.w2_slot_stride % 16)
        return fail("FP8 weight rows and the hidden rows must start on 16-byte boundaries");
    if (b.w13_row_stride < b.hidden || b.w2_row_stride < b.intermediate ||
        b.w13_slot_stride < b.w13_row_stride * 2 * b.intermediate || b.w2_slot_stride < b.w2_row_stride * b.hidden)
        return fail("FP8 weight strides are smaller than the bank geometry");
    if (b.w13_scale_row_stride < b.hidden / 128 || b.w2_scale_row_stride < b.intermediate / 128)
        return fail("FP8 scale strides are smaller than the bank geometry");
    const size_t xb = static_cast<size_t>(tokens) * b.hidden * 2;
    if (overlaps(out, xb, x, xb)) return fail("output must not overlap the hidden states");
    if (tokens == 0) return 0;
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const size_t need = prefill_workspace_layout(tokens, top_k, b.hidden, b.intermediate, b.slots, nullptr, nullptr);
    if (!workspace || workspace_bytes < need)
        return fail("prefill workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    PrefillWorkspace ws;
    prefill_workspace_layout(tokens, top_k, b.hidden, b.intermediate, b.slots, static_cast<char*>(workspace), &ws);
    const cudaError_t err = prefill_launch(b, x, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out, ws, sms,
                                           static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("prefill launch failed: %s", cudaGetErrorString(err));
    return 0;
}

size_t drama_b200_expert_rows_workspace_bytes(int64_t rows, int hidden, int intermediate, int experts) {
    return expert_rows_workspace_layout(rows, hidden, intermediate, experts, nullptr, nullptr);
}

int drama_b200_fp8_expert_rows(const DramaB200Fp8Bank* bank, const void* x, int64_t x_row_stride, int64_t rows,
                               const void* ids, int ids_dtype, void* out, void* workspace, size_t workspace_bytes,
                               void* stream) {
    if (!bank || !x || !out) return fail("bank, x and out are required");
    const DramaB200Fp8Bank& b = *bank;
    if (ids && !index_dtype(ids_dtype)) return fail("expert IDs must be int32 or int64");
    if (x_row_stride % 8 || x_row_stride < b.hidden || (!ids && x_row_stride < b.hidden + 8))
        return fail("x_row_stride must be a multiple of 8, at least hidden (hidden + 8 for tagged rows)");
    if (rows < 0 || rows > (int64_t(1) << 24)) return fail("rows must be in [0, 2^24]");
    if (b.hidden % 128 || b.hidden < 128 || b.intermediate % 128 || b.intermediate < 128)
        return fail("hidden and intermediate must be positive multiples of 128");
    if (b.slots < 1 || b.slots > 1024) return fail("slots must be in [1, 1024]");
    if (!b.w13 || !b.w13_scale || !b.w2 || !b.w2_scale) return fail("FP8 bank pointers are required");
    if (!aligned16(b.w13) || !aligned16(b.w2) || !aligned16(x) || !aligned16(out) || b.w13_row_stride % 16 ||
        b.w2_row_stride % 16 || b.w13_slot_stride % 16 || b.w2_slot_stride % 16)
        return fail("FP8 weight rows and the hidden rows must start on 16-byte boundaries");
    if (b.w13_row_stride < b.hidden || b.w2_row_stride < b.intermediate ||
        b.w13_slot_stride < b.w13_row_stride * 2 * b.intermediate || b.w2_slot_stride < b.w2_row_stride * b.hidden)
        return fail("FP8 weight strides are smaller than the bank geometry");
    if (b.w13_scale_row_stride < b.hidden / 128 || b.w2_scale_row_stride < b.intermediate / 128)
        return fail("FP8 scale strides are smaller than the bank geometry");
    const size_t xb = static_cast<size_t>(rows) * x_row_stride * 2, ob = static_cast<size_t>(rows) * b.hidden * 2;
    if (overlaps(out, ob, x, xb)) return fail("output must not overlap the hidden rows");
    if (rows == 0) return 0;
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const size_t need = expert_rows_workspace_layout(rows, b.hidden, b.intermediate, b.slots, nullptr, nullptr);
    if (!workspace || workspace_bytes < need)
        return fail("expert-rows workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    RowsWorkspace ws;
    expert_rows_workspace_layout(rows, b.hidden, b.intermediate, b.slots, static_cast<char*>(workspace), &ws);
    const cudaError_t err = expert_rows_launch(b, x, x_row_stride, rows, ids, ids_dtype, out, ws, sms,
                                               static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("expert-rows launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_ep_dispatch(const void* hidden, int64_t tokens, int hidden_size, const void* ids, int ids_dtype,
                           int top_k, int experts, int ranks, const int32_t* placement, int64_t capacity,
                           void* send_rows, int64_t send_row_stride, int32_t* send_ids, int32_t* pair_rows,
                           int32_t* status, void* stream) {
    if (!hidden || !ids || !send_rows || !pair_rows) return fail("hidden, ids, send_rows and pair_rows are required");
    if (send_row_stride % 8 || send_row_stride < hidden_size || (!send_ids && send_row_stride < hidden_size + 8))
        return fail("send_row_stride must be a multiple of 8, at least hidden (hidden + 8 without send_ids)");
    if (!index_dtype(ids_dtype)) return fail("expert IDs must be int32 or int64");
    if (tokens < 0 || top_k < 1 || top_k > 32) return fail("tokens must be >= 0 and top_k in [1, 32]");
    if (tokens * top_k > (int64_t(1) << 24)) return fail("dispatch supports at most 2^24 (token, slot) pairs");
    if (hidden_size < 8 || hidden_size % 8) return fail("hidden size must be a positive multiple of 8");
    if (ranks < 1 || ranks > kMaxEpRanks) return fail("ranks must be in [1, %d]", kMaxEpRanks);
    if (experts < ranks || experts % ranks || experts > (1 << 20))
        return fail("experts (%d) must be a multiple of ranks (%d) and at most 2^20", experts, ranks);
    if (capacity < 1 || capacity * ranks > INT32_MAX) return fail("capacity must be in [1, 2^31 / ranks)");
    if (!aligned16(hidden) || !aligned16(send_rows)) return fail("hidden rows must start on 16-byte boundaries");
    const size_t hb = static_cast<size_t>(tokens) * hidden_size * 2;
    const size_t sb = static_cast<size_t>(capacity) * ranks * send_row_stride * 2;
    if (overlaps(send_rows, sb, hidden, hb)) return fail("send rows must not overlap the hidden states");
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const cudaError_t err = ep_dispatch_launch(hidden, tokens, hidden_size, ids, ids_dtype, top_k, experts, ranks,
                                               placement, capacity, send_rows, send_row_stride, send_ids, pair_rows,
                                               status, sms, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("dispatch launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_ep_buffers_alloc(int ranks, int64_t capacity, int hidden, void** recv, void** back,
                                int32_t** signals, int32_t** counters) {
    if (!recv || !back || !signals || !counters) return fail("output pointers are required");
    if (ranks < 1 || ranks > kMaxEpRanks || capacity < 1 || hidden < 8 || hidden % 8)
        return fail("ranks in [1, %d], capacity >= 1 and hidden a positive multiple of 8", kMaxEpRanks);
    *recv = *back = nullptr;
    *signals = *counters = nullptr;
    const size_t rows = static_cast<size_t>(ranks) * capacity;
    cudaError_t err = cudaMalloc(recv, rows * (hidden + 8) * 2);
    if (err == cudaSuccess) err = cudaMalloc(back, rows * hidden * 2);
    if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void**>(signals), 256);
    if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void**>(counters), 256);
    if (err == cudaSuccess) err = cudaMemset(*signals, 0, 256);
    if (err == cudaSuccess) err = cudaMemset(*counters, 0, 256);
    if (err == cudaSuccess) err = cudaMemset(*recv, 0, rows * (hidden + 8) * 2);
    if (err != cudaSuccess) {
        cudaFree(*recv);
        cudaFree(*back);
        cudaFree(*signals);
        cudaFree(*counters);
        *recv = *back = nullptr;
        *signals = *counters = nullptr;
        return fail("allocating the exchange buffers: %s", cudaGetErrorString(err));
    }
    return 0;
}

int drama_b200_ep_buffers_free(void* recv, void* back, int32_t* signals, int32_t* counters) {
    cudaFree(recv);
    cudaFree(back);
    cudaFree(signals);
    cudaFree(counters);
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail("freeing the exchange buffers: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_ipc_handle(const void* device_ptr, void* handle_out) {
    if (!device_ptr || !handle_out) return fail("device_ptr and handle_out are required");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    cudaIpcMemHandle_t h;
    const cudaError_t err = cudaIpcGetMemHandle(&h, const_cast<void*>(device_ptr));
    if (err != cudaSuccess) return fail("cudaIpcGetMemHandle: %s", cudaGetErrorString(err));
    memcpy(handle_out, &h, sizeof(h));
    return 0;
}

int drama_b200_ipc_open(const void* handle, void** device_ptr) {
    if (!handle || !device_ptr) return fail("handle and device_ptr are required");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t err = cudaIpcOpenMemHandle(device_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return fail("cudaIpcOpenMemHandle: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_ipc_close(void* device_ptr) {
    const cudaError_t err = cudaIpcCloseMemHandle(device_ptr);
    if (err != cudaSuccess) return fail("cudaIpcCloseMemHandle: %s", cudaGetErrorString(err));
    return 0;
}

namespace {
constexpr long long kMaxPeerWaitNs = 60'000'000'000LL;  // one minute

int check_peers(const DramaB200EpPeers* peers) {
    if (!peers) return fail("peers are required");
    const DramaB200EpPeers& q = *peers;
    if (q.ranks < 1 || q.ranks > kMaxEpRanks || q.rank < 0 || q.rank >= q.ranks)
        return fail("ranks must be in [1, %d] and rank in [0, ranks)", kMaxEpRanks);
    if (q.capacity < 1 || q.capacity * q.ranks > INT32_MAX) return fail("capacity must be in [1, 2^31 / ranks)");
    if (q.hidden < 8 || q.hidden % 8) return fail("hidden must be a positive multiple of 8");
    if (q.experts < q.ranks || q.experts % q.ranks) return fail("experts must be a multiple of ranks");
    for (int r = 0; r < q.ranks; ++r)
        if (!q.recv[r] || !q.back[r] || !q.signals[r]) return fail("rank %d's exchange buffers are missing", r);
    if (!q.epoch || !q.done) return fail("epoch and done counters are required");
    if (q.wait_ns < 0 || q.wait_ns > kMaxPeerWaitNs) return fail("wait_ns must be in [0, %lld]", kMaxPeerWaitNs);
    return 0;
}
}  // namespace

int drama_b200_ep_p2p_dispatch(const DramaB200EpPeers* peers, const void* hidden, int64_t tokens, const void* ids,
                               int ids_dtype, int top_k, const int32_t* placement, int32_t* pair_rows,
                               int32_t* status, void* stream) {
    if (check_peers(peers)) return -1;
    if (!hidden || !ids || !pair_rows) return fail("hidden, ids and pair_rows are required");
    if (!index_dtype(ids_dtype)) return fail("expert IDs must be int32 or int64");
    if (tokens < 0 || top_k < 1 || top_k > 32) return fail("tokens must be >= 0 and top_k in [1, 32]");
    if (tokens * top_k > peers->capacity) return fail("capacity must be at least tokens * top_k");
    if (tokens * top_k > kP2pMaxPairs) return fail("the peer dispatch handles at most %d pairs per rank", kP2pMaxPairs);
    if (!aligned16(hidden)) return fail("hidden rows must start on 16-byte boundaries");
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const cudaError_t err = ep_p2p_dispatch_launch(*peers, hidden, tokens, ids, ids_dtype, top_k, placement,
                                                   pair_rows, status, sms, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("peer dispatch launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_fp8_expert_rows_p2p(const DramaB200Fp8Bank* bank, const DramaB200EpPeers* peers, void* workspace,
                                   size_t workspace_bytes, int32_t* status, void* stream) {
    if (check_peers(peers)) return -1;
    if (!bank) return fail("bank is required");
    const DramaB200Fp8Bank& b = *bank;
    if (b.hidden != peers->hidden) return fail("bank hidden size %d differs from the exchange's %d", b.hidden,
                                               peers->hidden);
    if (b.slots != peers->experts / peers->ranks) return fail("the bank must hold experts / ranks slots");
    if (b.hidden % 128 || b.intermediate % 128 || b.intermediate < 128)
        return fail("hidden and intermediate must be positive multiples of 128");
    if (!b.w13 || !b.w13_scale || !b.w2 || !b.w2_scale) return fail("FP8 bank pointers are required");
    if (!aligned16(b.w13) || !aligned16(b.w2) || b.w13_row_stride % 16 || b.w2_row_stride % 16 ||
        b.w13_slot_stride % 16 || b.w2_slot_stride % 16)
        return fail("FP8 weight rows must start on 16-byte boundaries");
    const int64_t rows = peers->capacity * peers->ranks;
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const size_t need = expert_rows_workspace_layout(rows, b.hidden, b.intermediate, b.slots, nullptr, nullptr);
    if (!workspace || workspace_bytes < need)
        return fail("expert-rows workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail("workspace must be 256-byte aligned");
    RowsWorkspace ws;
    expert_rows_workspace_layout(rows, b.hidden, b.intermediate, b.slots, static_cast<char*>(workspace), &ws);
    const int me = peers->rank;
    RowsReceive rc;
    rc.signals = peers->signals[me];
    rc.epoch = peers->epoch;
    rc.ranks = peers->ranks;
    rc.cap = peers->capacity;
    rc.unused = b.slots;
    rc.status = status;
    rc.wait_ns = peers->wait_ns;
    RowsScatter sc;
    sc.ranks = peers->ranks;
    sc.rank = me;
    sc.cap = peers->capacity;
    for (int r = 0; r < peers->ranks; ++r) {
        sc.dst[r] = static_cast<__nv_bfloat16*>(peers->back[r]);
        sc.signals[r] = peers->signals[r];
    }
    sc.done = peers->done + 16;   // the GEMM's own arrival counter, 64 bytes after the dispatch's
    sc.epoch = peers->epoch;
    const cudaError_t err = expert_rows_launch(b, peers->recv[me], b.hidden + 8, rows, nullptr, DRAMA_B200_I32,
                                               nullptr, ws, sms, static_cast<cudaStream_t>(stream), &sc, &rc);
    if (err != cudaSuccess) return fail("peer expert-rows launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_ep_p2p_combine(const DramaB200EpPeers* peers, const int32_t* pair_rows, const void* weights,
                              int weights_dtype, int64_t tokens, int top_k, const void* residual, void* out,
                              int32_t* status, void* stream) {
    if (check_peers(peers)) return -1;
    if (!pair_rows || !weights || !out) return fail("pair_rows, weights and out are required");
    if (!float_dtype(weights_dtype)) return fail("routing weights must be floating point");
    if (tokens < 0 || top_k < 1 || top_k > 32) return fail("tokens must be >= 0 and top_k in [1, 32]");
    if (!aligned16(out) || (residual && !aligned16(residual))) return fail("out and residual must be 16-byte aligned");
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const int me = peers->rank;
    const cudaError_t err = ep_combine_launch(peers->back[me], peers->capacity * peers->ranks, pair_rows, weights,
                                              weights_dtype, tokens, top_k, peers->hidden, residual, out, sms,
                                              static_cast<cudaStream_t>(stream), peers->signals[me] + 2 * peers->ranks,
                                              peers->epoch, peers->ranks, status, peers->wait_ns);
    if (err != cudaSuccess) return fail("peer combine launch failed: %s", cudaGetErrorString(err));
    return 0;
}

int drama_b200_ep_combine(const void* rows, int64_t row_count, const int32_t* pair_rows, const void* weights,
                          int weights_dtype, int64_t tokens, int top_k, int hidden_size, const void* residual,
                          void* out, void* stream) {
    if (!rows || !pair_rows || !weights || !out) return fail("rows, pair_rows, weights and out are required");
    if (row_count < 0) return fail("row_count must be non-negative");
    if (!float_dtype(weights_dtype)) return fail("routing weights must be floating point");
    if (tokens < 0 || top_k < 1 || top_k > 32) return fail("tokens must be >= 0 and top_k in [1, 32]");
    if (hidden_size < 8 || hidden_size % 8) return fail("hidden size must be a positive multiple of 8");
    if (!aligned16(rows) || !aligned16(out) || (residual && !aligned16(residual)))
        return fail("rows, residual and out must start on 16-byte boundaries");
    const size_t ob = static_cast<size_t>(tokens) * hidden_size * 2;
    if (overlaps(out, ob, rows, static_cast<size_t>(row_count) * hidden_size * 2))
        return fail("output must not overlap the expert rows");
    if (residual && residual != out && overlaps(out, ob, residual, ob))
        return fail("output may be the residual itself but must not partly overlap it");
    int sms = 0;
    if (sm_count_current(&sms)) return -1;
    const cudaError_t err = ep_combine_launch(rows, row_count, pair_rows, weights, weights_dtype, tokens, top_k, hidden_size,
                                              residual, out, sms, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail("combine launch failed: %s", cudaGetErrorString(err));
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// FP8 decode for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc or hand over a workspace: a host
// binding with no device allocator of its own, or a serving process whose
// memory manager has reserved the device for its banks and caches and allows
// no further allocation (a cudaMalloc there would also synchronise the
// device). This variant of drama_b200_fp8_decode keeps its scratch in the
// array below, which every GPU that loads the library holds until the process
// exits. Host code cannot use the array's name as a device address; the
// address comes from cudaGetSymbolAddress, once per device.
// ---------------------------------------------------------------------------
constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

namespace drama {
namespace {
std::mutex g_static_mutex;
struct StaticBase {
    CUcontext ctx;
    void* ptr;
};
StaticBase g_static_base[64] = {};

// The context current on this thread (null when none is), through the
// driver entry point the runtime exposes.
int current_context(CUcontext* ctx) {
    using GetCurrent = CUresult (*)(CUcontext*);
    static GetCurrent fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult found{};
        const cudaError_t err = cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &found);
        if (err != cudaSuccess || found != cudaDriverEntryPointSuccess || !p)
            return fail("cuCtxGetCurrent is not available from the driver");
        fn = reinterpret_cast<GetCurrent>(p);
    }
    if (fn(ctx) != CUDA_SUCCESS) return fail("cuCtxGetCurrent failed");
    return 0;
}

// The array's device address in the current context. It is looked up on
// the first call in each context (cudaGetSymbolAddress) and kept per
// context, so a device reset or another context on the same device gets its
// own address. No clear is needed: every decode call rewrites the status
// words and zeroes its split-K and combine counters before the expert kernels
// read them (decode_prep_kernel), so the array's previous contents are never
// read.
int static_scratch(void** out) {
    int dev = 0;
    const cudaError_t derr = cudaGetDevice(&dev);
    if (derr != cudaSuccess) return fail("cudaGetDevice: %s", cudaGetErrorString(derr));
    if (dev < 0 || dev >= 64) return fail("device ordinal %d out of range", dev);
    CUcontext ctx = nullptr;
    if (current_context(&ctx)) return -1;
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (!ctx || !g_static_base[dev].ptr || g_static_base[dev].ctx != ctx) {
        void* ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (err != cudaSuccess) return fail("cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(err));
        if (current_context(&ctx)) return -1;  // the lookup binds the device's primary context if none was current
        g_static_base[dev] = {ctx, ptr};
    }
    *out = g_static_base[dev].ptr;
    return 0;
}
}  // namespace
}  // namespace drama

extern "C" {

size_t drama_b200_static_scratch_bytes(void) { return kStaticScratchBytes; }

int drama_b200_fp8_decode_static(const DramaB200Fp8Bank* bank, const void* x, int x_dtype, int64_t tokens,
                                 int top_k, const void* ids, int ids_dtype, const void* weights,
                                 int weights_dtype, void* out, float* pair_out, void* stream) {
    DecodeArgs a{};
    if (prepare_fp8_decode(bank, x, x_dtype, tokens, top_k, ids, ids_dtype, weights, weights_dtype, out, pair_out,
                           &a))
        return -1;
    if (tokens == 0) return 0;
    int sms = 0;
    const size_t need = decode_scratch_need(a, &sms);
    if (!need) return -1;
    if (need > kStaticScratchBytes)
        return fail("decode of %lld tokens x top-%d at hidden %d, intermediate %d needs %zu bytes of scratch; "
                    "the library's static scratch holds %zu (use drama_b200_fp8_decode with a workspace)",
                    static_cast<long long>(tokens), top_k, a.hidden, a.intermediate, need, kStaticScratchBytes);
    void* base = nullptr;
    if (static_scratch(&base)) return -1;
    return finish_decode(a, base, kStaticScratchBytes, stream);
}

}  // extern "C"
