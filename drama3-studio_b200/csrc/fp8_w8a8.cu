// The official FP8 W8A8 expert contract on the GPU: the arithmetic of the
// reference's production decode backend (src/drama_low_vram/fp8_decode.py:
// 114-147 forward / quantized_pairs, decode_gemm 24-58; the CPU statement of
// it is native/src/runtime.cpp:162-237 and fp8_cpu_reference.py:14-52):
//
//   x (bf16 row) -> 1x128 blocks: scale = max(amax, 1e-10) * (1/448),
//                   q = e4m3(x / scale) (round to nearest even, saturating)
//   gu[n] = sum over K blocks b of fma(dot_b(W13[n], q) * scale_b, S13[n/128][b], acc)
//   gate, up = bf16(gu); h = (gate / (1 + exp(-gate))) * up       (fp32)
//   h -> 1x128 blocks as x
//   down[n] = sum over I blocks of fma(dot_b(W2[n], hq) * hscale_b, S2[n/128][b], acc)
//   partial = down * route weight (fp32); out[t] = bf16(sum over slots in slot order)
//
// dot_b is a 128-term product sum of E4M3 values; here it is four
// mma.m16n8k32 E4M3 tensor-core steps (the products are exact; the order of
// the additions inside the tensor core is the hardware's), so results agree
// with the sequential CPU sum to within fp32 rounding of the block sums.
//
// Launches: quantise the token rows; gate/up cells (pair, 8 gate + 8 up
// rows), one warp each, weights streamed with 16-byte loads straight into
// the FP8 A fragments (no conversion); quantise the SwiGLU rows; down cells
// (pair, 16 rows), route weight applied; slot-ordered combine.
#include "common.cuh"
#include "kernels.h"

namespace drama {
namespace {

constexpr int kQWarps = 4;  // warps per CTA of the cell kernels

__device__ __forceinline__ void mma_e4m3_16832(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp32 -> E4M3 byte, round to nearest even, saturating to +-448.
__device__ __forceinline__ uint32_t e4m3_byte(float v) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
    return r & 0xffu;
}

// One 1x128 block of `v` (thread k of a 128-thread group holds value k):
// the block scale and this thread's byte.
__device__ __forceinline__ uint32_t quantize_block(float v, float* s_red4, float* scale_out) {
    const int k = threadIdx.x & 127, lane = k & 31, w = k >> 5;
    float m = fabsf(v);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) s_red4[w] = m;
    __syncthreads();
    const float amax = fmaxf(fmaxf(fmaxf(s_red4[0], s_red4[1]), fmaxf(s_red4[2], s_red4[3])), 1e-10f);
    const float scale = __fmul_rn(amax, 1.0f / 448.0f);
    *scale_out = scale;
    return e4m3_byte(__fdiv_rn(v, scale));
}

struct W8Args {
    DramaB200Fp8Bank bank;
    const __nv_bfloat16* x;
    int64_t tokens;
    int top_k, H, I;
    const void* ids;
    int ids_dtype;
    const void* weights;
    int weights_dtype;
    uint8_t* xq;       // [T][H]
    float* xs;         // [T][H/128]
    float* h;          // [P][I]
    uint8_t* hq;       // [P][I]
    float* hs;         // [P][I/128]
    float* pair_out;   // [P][H] weighted fp32 partials
    __nv_bfloat16* out;  // [T][H] or null
    int32_t* status;   // [0] pairs with an out-of-range id (contribute zero)
};

// grid (T, H/128), block 128
__global__ void __launch_bounds__(128) w8_quant_x_kernel(W8Args a) {
    __shared__ float s_red[4];
    const int t = blockIdx.x, b = blockIdx.y, k = threadIdx.x;
    const int64_t i = static_cast<int64_t>(t) * a.H + b * 128 + k;
    float scale;
    const uint32_t q = quantize_block(__bfloat162float(a.x[i]), s_red, &scale);
    a.xq[i] = static_cast<uint8_t>(q);
    if (k == 0) a.xs[static_cast<int64_t>(t) * (a.H / 128) + b] = scale;
}

// A tile's rows r0 (MMA rows 0-7 at lane row g) and r1 (rows 8-15) times the
// quantised row q over K = 128 * nb columns, promoted per block with the
// activation scales sa[] and the rows' block scales. K permutation: in each
// 64-column span lane t takes columns 16t..16t+15 of both operands, bytes 0-7
// to the first k32 step and bytes 8-15 to the second.
__device__ __forceinline__ void tile_dot(const uint8_t* r0, const uint8_t* r1, const uint8_t* q, const float* sa,
                                         const float* s0, const float* s1, int nb, int g, int t, float& acc0,
                                         float& acc1) {
    for (int b = 0; b < nb; ++b) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int span = 0; span < 2; ++span) {
            const int col = b * 128 + span * 64 + 16 * t;
            const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(r0 + col));
            const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(r1 + col));
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if (g == 0) x = __ldg(reinterpret_cast<const uint4*>(q + col));
            const uint32_t A0[4] = {w0.x, w1.x, w0.y, w1.y};
            const uint32_t A1[4] = {w0.z, w1.z, w0.w, w1.w};
            mma_e4m3_16832(d, A0, x.x, x.y);
            mma_e4m3_16832(d, A1, x.z, x.w);
        }
        acc0 = fmaf(__fmul_rn(d[0], sa[b]), s0[b], acc0);
        acc1 = fmaf(__fmul_rn(d[2], sa[b]), s1[b], acc1);
    }
}

__device__ __forceinline__ bool pair_route(const W8Args& a, int p, int& expert, float& w) {
    expert = static_cast<int>(load_index(a.ids, a.ids_dtype, p));
    w = load_any(a.weights, a.weights_dtype, p);
    return expert >= 0 && expert < a.bank.slots;
}

// cells: (pair p, j) for j < I/8: gate rows 8j.. and up rows I + 8j..; one warp each
__global__ void __launch_bounds__(kQWarps * 32) w8_up_kernel(W8Args a) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int cell = blockIdx.x * kQWarps + (threadIdx.x >> 5);
    const int per = a.I / 8, P = static_cast<int>(a.tokens) * a.top_k;
    if (cell >= P * per) return;
    const int p = cell / per, j = cell - p * per;
    int expert;
    float w;
    const int row = j * 8 + g;
    if (!pair_route(a, p, expert, w)) {
        if (t == 0) a.h[static_cast<int64_t>(p) * a.I + row] = 0.0f;
        return;
    }
    const DramaB200Fp8Bank& b = a.bank;
    const int KB = a.H / 128, token = p / a.top_k;
    const uint8_t* base = static_cast<const uint8_t*>(b.w13) + expert * b.w13_slot_stride;
    const float* sbase = b.w13_scale + expert * b.w13_scale_slot_stride;
    const float* sg = sbase + ((j * 8) >> 7) * b.w13_scale_row_stride;
    const float* su = sbase + ((a.I + j * 8) >> 7) * b.w13_scale_row_stride;
    float gate = 0.0f, up = 0.0f;
    tile_dot(base + static_cast<int64_t>(row) * b.w13_row_stride,
             base + static_cast<int64_t>(a.I + row) * b.w13_row_stride, a.xq + static_cast<int64_t>(token) * a.H,
             a.xs + static_cast<int64_t>(token) * KB, sg, su, KB, g, t, gate, up);
    if (t == 0) {
        const float gb = __bfloat162float(__float2bfloat16_rn(gate));
        const float ub = __bfloat162float(__float2bfloat16_rn(up));
        a.h[static_cast<int64_t>(p) * a.I + row] = __fmul_rn(__fdiv_rn(gb, __fadd_rn(1.0f, expf(-gb))), ub);
    }
}

// grid (P, I/128), block 128
__global__ void __launch_bounds__(128) w8_quant_h_kernel(W8Args a) {
    __shared__ float s_red[4];
    const int p = blockIdx.x, b = blockIdx.y, k = threadIdx.x;
    const int64_t i = static_cast<int64_t>(p) * a.I + b * 128 + k;
    float scale;
    const uint32_t q = quantize_block(a.h[i], s_red, &scale);
    a.hq[i] = static_cast<uint8_t>(q);
    if (k == 0) a.hs[static_cast<int64_t>(p) * (a.I / 128) + b] = scale;
}

// cells: (pair p, 16-row tile n of H); the route weight applied in fp32
__global__ void __launch_bounds__(kQWarps * 32) w8_down_kernel(W8Args a) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int cell = blockIdx.x * kQWarps + (threadIdx.x >> 5);
    const int per = a.H / 16, P = static_cast<int>(a.tokens) * a.top_k;
    if (cell >= P * per) return;
    const int p = cell / per, n = (cell - p * per) * 16;
    int expert;
    float w;
    float* dst = a.pair_out + static_cast<int64_t>(p) * a.H + n;
    if (!pair_route(a, p, expert, w)) {
        if (t == 0) {
            dst[g] = 0.0f;
            dst[g + 8] = 0.0f;
        }
        if (lane == 0 && (cell - p * per) == 0) atomicAdd(a.status, 1);
        return;
    }
    const DramaB200Fp8Bank& b = a.bank;
    const int KB = a.I / 128;
    const uint8_t* base = static_cast<const uint8_t*>(b.w2) + expert * b.w2_slot_stride;
    const float* s = b.w2_scale + expert * b.w2_scale_slot_stride + (n >> 7) * b.w2_scale_row_stride;
    float d0 = 0.0f, d1 = 0.0f;
    tile_dot(base + static_cast<int64_t>(n + g) * b.w2_row_stride, base + static_cast<int64_t>(n + g + 8) * b.w2_row_stride,
             a.hq + static_cast<int64_t>(p) * a.I, a.hs + static_cast<int64_t>(p) * KB, s, s, KB, g, t, d0, d1);
    if (t == 0) {
        dst[g] = __fmul_rn(d0, w);
        dst[g + 8] = __fmul_rn(d1, w);
    }
}

// out[t][c] = bf16(sum over slots, in slot order, of pair_out[t*k + s][c])
__global__ void w8_combine_kernel(W8Args a) {
    const int64_t total = a.tokens * a.H;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t token = i / a.H, c = i - token * a.H;
        float acc = 0.0f;
        for (int s = 0; s < a.top_k; ++s) acc = __fadd_rn(acc, a.pair_out[(token * a.top_k + s) * a.H + c]);
        a.out[i] = __float2bfloat16_rn(acc);
    }
}

}  // namespace

size_t fp8_w8a8_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, char* base,
                                 Fp8W8a8Workspace* ws) {
    const int64_t P = tokens * top_k;
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return p;
    };
    Fp8W8a8Workspace w{};
    w.status = reinterpret_cast<int32_t*>(take(16));
    w.xq = reinterpret_cast<uint8_t*>(take(tokens * hidden));
    w.xs = reinterpret_cast<float*>(take(tokens * (hidden / 128) * 4));
    w.h = reinterpret_cast<float*>(take(P * intermediate * 4));
    w.hq = reinterpret_cast<uint8_t*>(take(P * intermediate));
    w.hs = reinterpret_cast<float*>(take(P * (intermediate / 128) * 4));
    w.pair_out = reinterpret_cast<float*>(take(P * hidden * 4));
    if (ws) *ws = w;
    return off;
}

cudaError_t fp8_w8a8_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t tokens, int top_k, const void* ids,
                            int ids_dtype, const void* weights, int weights_dtype, void* out, float* pair_out,
                            const Fp8W8a8Workspace& ws, cudaStream_t s) {
    W8Args a{};
    a.bank = bank;
    a.x = static_cast<const __nv_bfloat16*>(x);
    a.tokens = tokens;
    a.top_k = top_k;
    a.H = bank.hidden;
    a.I = bank.intermediate;
    a.ids = ids;
    a.ids_dtype = ids_dtype;
    a.weights = weights;
    a.weights_dtype = weights_dtype;
    a.xq = ws.xq;
    a.xs = ws.xs;
    a.h = ws.h;
    a.hq = ws.hq;
    a.hs = ws.hs;
    a.pair_out = pair_out ? pair_out : ws.pair_out;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.status = ws.status;
    const int P = static_cast<int>(tokens) * top_k;
    cudaError_t err = cudaMemsetAsync(ws.status, 0, 16, s);
    if (err != cudaSuccess) return err;
    w8_quant_x_kernel<<<dim3(static_cast<unsigned>(tokens), a.H / 128), 128, 0, s>>>(a);
    const int up_cells = P * (a.I / 8), dn_cells = P * (a.H / 16);
    w8_up_kernel<<<(up_cells + kQWarps - 1) / kQWarps, kQWarps * 32, 0, s>>>(a);
    w8_quant_h_kernel<<<dim3(P, a.I / 128), 128, 0, s>>>(a);
    w8_down_kernel<<<(dn_cells + kQWarps - 1) / kQWarps, kQWarps * 32, 0, s>>>(a);
    if (out) {
        const int64_t total = tokens * a.H;
        const int blocks = static_cast<int>((total + 255) / 256 < 1184 ? (total + 255) / 256 : 1184);
        w8_combine_kernel<<<blocks, 256, 0, s>>>(a);
    }
    return cudaGetLastError();
}

}  // namespace drama
