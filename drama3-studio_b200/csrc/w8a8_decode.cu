// W8A8 expert FFN, modes 1-3 of the reference's QuantizedExpertBackend
// (src/drama_low_vram/quantized_kernels.py:115-189 _quant_gemm, 15-45
// rotate_quantize, 217-248 the backend): INT8-ConvRot, W6A8 and W4A8 with a
// 16-level codebook.
//
// Arithmetic (the reference's CUDA path):
//   activations: each 256-column group of a row is rotated by
//     kron(H4, H4, H4, H4) / 16 and rounded to bf16, then quantised per row
//     to int8 with s = max(amax, 1e-12) / 127, q = clamp(rint(r / s), +-127);
//   weights: int8 (mode 1) or clamp(rint(level * fp8 relative scale), +-127)
//     (modes 2/3) with an fp32 channel scale per output row;
//   projection = bf16((float(int32 sum) * s) * channel).
// The int32 sums are exact, so they do not depend on the summation order.
// The rotation runs as four radix-4 stages in float64 and is rounded once,
// which equals the correctly rounded product for all practical inputs.
//
// Launches (one stream, in order, chained by programmatic dependent launch):
//   prep   : CTA 0 groups the route slots into expert groups of <= 8 pairs
//            (one warp with match_any for <= 32 pairs, else a stable bucket;
//            a column's result does not depend on its group, so any grouping
//            gives the same bits); CTAs 1..T rotate and quantise one token row
//            each;
//   gemv   : gate/up projections. A cell is (group, 8 gate rows j..j+7 in
//            MMA rows 0-7 and their 8 up rows in MMA rows 8-15): a warp
//            streams the tile's weights with 16-byte loads, dequantises them
//            in registers into mma.m16n8k32 s8 fragments whose N dimension
//            holds the group's tokens (weights read once per group). When
//            there are too few cells to occupy the GPU (batch 1), a CTA of up
//            to 8 warps shares one cell, each warp a contiguous part of K, and
//            warp 0 adds the int32 sums from shared memory (exact in any
//            order) and applies the epilogue, which writes the SwiGLU rows
//            bf16(bf16(silu(gate)) * up) [P][I];
//   rotate : SwiGLU rows -> int8 + scale;
//   gemv   : down projections, rounded to bf16 and weighted in fp32; the
//            warp that finishes the last cell of a 16-row tile of H sums the
//            route slots of those rows in slot order in fp32 (the combine).
//
// K permutation: within each 64-column span, thread t of a quad takes the 16
// consecutive columns 16t..16t+15 of both its weight rows and its token row,
// and feeds bytes 0-7 to the first k32 MMA and bytes 8-15 to the second. A and
// B use the same permutation, so every product still pairs equal columns.
#include "common.cuh"
#include "grouped.cuh"
#include "kernels.h"
#include "bucket.cuh"
#include "int4.cuh"

namespace drama {
namespace {

constexpr int kW8GemvThreads = 128;
constexpr int kW8Unroll = 4;  // split-K granule: 64-column spans per register batch (K % 256 == 0)
constexpr int kW8Group = 8;
constexpr int kW8TargetWarps = 4736;  // 148 SMs x 32 warps: the split-K target

__device__ __forceinline__ void w8_fence() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ld_nc_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ld_nc_v2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_nc_u8(const void* p) {
    uint16_t v;
    asm volatile("ld.global.nc.u8 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// FP8 E4M3 byte -> float (exact), via the f16x2 conversion.
__device__ __forceinline__ float fp8_to_float(uint32_t byte) {
    const uint32_t h2 = e4m3x2_to_f16x2(byte & 0xffu);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xffffu)));
}

// Packed-half helpers (round-to-nearest; each is one explicit instruction, never contracted).
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// clamp to [1536 - 127, 1536 + 127] = [1409, 1663]
__device__ __forceinline__ uint32_t h2_clamp_grid(uint32_t a) {
    uint32_t d;
    asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(0x65816581u));  // 1409
    asm("min.f16x2 %0, %1, %2;" : "=r"(d) : "r"(d), "r"(0x667F667Fu));  // 1663
    return d;
}

// clamp(rint(level * rel), +-127) (fp32 product, like the reference) in the
// low byte: the lower clamp first (-127 is an integer, so the order does not
// matter), then one round-to-nearest-even conversion that saturates at 127.
__device__ __forceinline__ uint32_t grid_byte(float level, float rel) {
    const float v = fmaxf(__fmul_rn(level, rel), -127.0f);
    uint32_t q;
    asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(q) : "f"(v));
    return q;
}

// ---------------------------------------------------------------------------
// ConvRot rotation + per-row int8 quantisation of one row, by a whole CTA
// (blockDim a multiple of 256; chunks of 256 columns in passes)
// ---------------------------------------------------------------------------
__constant__ double kH4[4][4] = {{1, 1, 1, -1}, {1, 1, -1, 1}, {1, -1, 1, 1}, {-1, 1, 1, 1}};

// row = bf16 [K]. s_v: blockDim doubles; s_row: K floats.
__device__ void rotate_row(const __nv_bfloat16* row, int K, int8_t* q, float* qs, double* s_v, float* s_row) {
    __shared__ float s_red[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
    const int j = tid & 255;
    double* v = s_v + (tid - j);  // this thread's 256-value chunk buffer
    float amax = 0.0f;
    for (int c0 = 0; c0 < K; c0 += nthr) {
        const int col = c0 + tid;
        const bool live = col < K;  // K and nthr are multiples of 256: whole chunks are live or idle
        if (live) {
            v[j] = static_cast<double>(__bfloat162float(row[col]));
        }
        __syncthreads();
#pragma unroll
        for (int st = 0; st < 4; ++st) {  // base-4 digit st, least significant first
            const int stride = 1 << (2 * st);
            const int d = (j >> (2 * st)) & 3;
            const int base = j - d * stride;
            double acc = 0.0;
            if (live) {
                acc = kH4[0][d] * v[base];
                acc = acc + kH4[1][d] * v[base + stride];
                acc = acc + kH4[2][d] * v[base + 2 * stride];
                acc = acc + kH4[3][d] * v[base + 3 * stride];
            }
            __syncthreads();
            if (live) v[j] = acc;
            __syncthreads();
        }
        if (live) {
            const float rv = __bfloat162float(__double2bfloat16(v[j] * 0.0625));
            s_row[col] = rv;
            amax = fmaxf(amax, fabsf(rv));
        }
        __syncthreads();
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) s_red[warp] = amax;
    __syncthreads();
    float m = s_red[0];
    for (int w = 1; w < nthr / 32; ++w) m = fmaxf(m, s_red[w]);
    const float scale = __fdiv_rn(fmaxf(m, 1e-12f), 127.0f);
    for (int col = tid; col < K; col += nthr) {
        float r = rintf(__fdiv_rn(s_row[col], scale));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        q[col] = static_cast<int8_t>(r);
    }
    if (tid == 0) *qs = scale;
}

// ---------------------------------------------------------------------------
// prep (CTA 0): groups of <= 8 pairs per slot (the FP8/INT4 decode's records)
// and the split-K counters; CTAs 1..T: token rows -> int8
// ---------------------------------------------------------------------------
struct W8PrepArgs {
    const void* ids;
    int ids_dtype;
    const void* weights;
    int weights_dtype;
    const __nv_bfloat16* x;
    int64_t pairs;
    int slots, hidden, intermediate;
    float* pair_out;  // zeroed rows for dropped pairs
    W8a8Workspace ws;
};

// The rest of CTA 0's work once the groups exist: counts, counters, weights,
// zero partials for pairs whose slot is out of range.
__device__ void w8a8_prep_tail(const W8PrepArgs& a, int groups, int dropped) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        a.ws.num_groups[0] = groups;
        a.ws.status[0] = dropped;
    }
    for (int i = tid; i < a.hidden / 16; i += blockDim.x) a.ws.cmb_cnt[i] = 0;
    for (int64_t p = tid; p < a.pairs; p += blockDim.x) a.ws.wts[p] = load_any(a.weights, a.weights_dtype, p);
    if (dropped) {
        for (int64_t p = 0; p < a.pairs; ++p) {
            const int64_t id = load_index(a.ids, a.ids_dtype, p);
            if (id < 0 || id >= a.slots)
                for (int n = tid; n < a.hidden; n += blockDim.x) a.pair_out[p * a.hidden + n] = 0.0f;
        }
    }
}

__global__ void __launch_bounds__(1024) w8a8_prep_kernel(W8PrepArgs a) {
    grid_launch_dependents();  // programmatic dependent launch: the next kernel may start its launch
    grid_dependency_wait();    // the previous kernel's results are visible from here
    extern __shared__ __align__(16) unsigned char smem_w8prep[];
    if (blockIdx.x > 0) {  // rotate token row blockIdx.x - 1
        double* s_v = reinterpret_cast<double*>(smem_w8prep);
        float* s_row = reinterpret_cast<float*>(s_v + blockDim.x);
        const int64_t t = blockIdx.x - 1;
        rotate_row(a.x + t * a.hidden, a.hidden, a.ws.xq + t * a.hidden, a.ws.xs + t, s_v, s_row);
        return;
    }
    int* smem = reinterpret_cast<int*>(smem_w8prep);
    __shared__ int dropped;
    __shared__ int warp_tot[32];
    __shared__ int s_groups;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = a.slots;
    if (tid == 0) dropped = 0;
    __syncthreads();
    if (a.pairs <= 32) {
        // one warp: lanes are pairs; equal ids form groups of <= 8 in lane order
        if (warp == 0) {
            const int64_t id = lane < a.pairs ? load_index(a.ids, a.ids_dtype, lane) : -2;
            const bool valid = id >= 0 && id < S;
            const int key = valid ? static_cast<int>(id) : -2 - lane;  // invalid lanes stay alone
            const unsigned mask = __match_any_sync(0xffffffffu, key);
            const bool leader = valid && lane == __ffs(mask) - 1;
            const int ng = leader ? (__popc(mask) + kW8Group - 1) / kW8Group : 0;
            int base = ng;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, base, off);
                if (lane >= off) base += y;
            }
            const int total = __shfl_sync(0xffffffffu, base, 31);
            base -= ng;
            if (leader) {
                unsigned rest = mask;
                for (int j = 0; j < ng; ++j) {
                    uint32_t packed[4] = {0u, 0u, 0u, 0u};
                    int cnt = 0;
                    while (rest && cnt < kW8Group) {
                        const int member = __ffs(rest) - 1;
                        rest &= rest - 1;
                        packed[cnt >> 1] |= static_cast<uint32_t>(member) << (16 * (cnt & 1));
                        ++cnt;
                    }
                    a.ws.g_rec[2 * (base + j)] = make_int4(static_cast<int>(id), 0, cnt, 0);
                    a.ws.g_rec[2 * (base + j) + 1] = make_int4(static_cast<int>(packed[0]), static_cast<int>(packed[1]),
                                                               static_cast<int>(packed[2]), static_cast<int>(packed[3]));
                }
            }
            const unsigned bad = __ballot_sync(0xffffffffu, lane < a.pairs && !valid);
            if (lane == 0) {
                s_groups = total;
                dropped = __popc(bad);
            }
        }
        __syncthreads();
        w8a8_prep_tail(a, s_groups, dropped);
        return;
    }
    stable_bucket(a.ids, a.ids_dtype, a.pairs, S, smem, nullptr, a.ws.order, &dropped);
    const int* counts = smem;
    const int* ends = smem + S;
    int ng = 0;
    if (tid < S) ng = (counts[tid] + kW8Group - 1) / kW8Group;
    int x = ng;
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
    const int gbase = x - ng + (warp ? warp_tot[warp - 1] : 0);
    if (tid < S && ng) {
        const int c = counts[tid];
        const int start = ends[tid] - c;
        for (int j = 0; j < ng; ++j) {
            const int cnt = min(kW8Group, c - j * kW8Group);
            uint32_t packed[4] = {0u, 0u, 0u, 0u};
            for (int q = 0; q < cnt; ++q)
                packed[q >> 1] |= static_cast<uint32_t>(a.ws.order[start + j * kW8Group + q] & 0xffff)
                                  << (16 * (q & 1));
            a.ws.g_rec[2 * (gbase + j)] = make_int4(tid, start + j * kW8Group, cnt, 0);
            a.ws.g_rec[2 * (gbase + j) + 1] = make_int4(static_cast<int>(packed[0]), static_cast<int>(packed[1]),
                                                        static_cast<int>(packed[2]), static_cast<int>(packed[3]));
        }
    }
    w8a8_prep_tail(a, warp_tot[31], dropped);
}

// SwiGLU rows -> int8 (one CTA per pair)
__global__ void __launch_bounds__(1024) w8a8_act_kernel(const __nv_bfloat16* up, int I, int8_t* hq, float* hs) {
    grid_launch_dependents();  // programmatic dependent launch: the next kernel may start its launch
    grid_dependency_wait();    // the previous kernel's results are visible from here
    extern __shared__ __align__(16) unsigned char smem_w8act[];
    double* s_v = reinterpret_cast<double*>(smem_w8act);
    float* s_row = reinterpret_cast<float*>(s_v + blockDim.x);
    const int64_t p = blockIdx.x;
    rotate_row(up + p * I, I, hq + p * I, hs + p, s_v, s_row);
}

// ---------------------------------------------------------------------------
// gemv: tasks (group, 16-row tile, K part)
// ---------------------------------------------------------------------------
struct W8Role {
    const uint8_t* w;
    const uint8_t* s;
    int64_t w_slot, w_row, s_slot, s_row;  // bytes
    int n, k;
};

struct W8GemvArgs {
    W8Role role;
    const int4* g_rec;
    const int32_t* num_groups;
    const int8_t* act;        // [rows][k]
    const float* act_scale;   // [rows]
    int top_k;                // up: activation row = pair / top_k; down: row = pair
    int ksplit;               // K parts per tile = warps per CTA when > 1 (spans divisible by ksplit * kW8Unroll)
    __nv_bfloat16* up_out;    // up: [P][n / 2] SwiGLU rows
    float* pair_out;          // down: [P][n]
    const float* wts;         // down: [P]
    int32_t* cmb_cnt;         // down: [n/16] finished cells per row tile
    void* out;                // down: [T][n] combined rows (NULL: pairs only)
    int out_dtype;
    int64_t tokens;
};

// Raw weight bytes of one span for one row, by mode.
template <int MODE> struct SpanRaw;
template <> struct SpanRaw<1> { uint4 v; };
template <> struct SpanRaw<2> { uint2 lo; uint32_t hi; uint32_t rel; };
template <> struct SpanRaw<3> { uint2 lo; uint32_t rel; };

template <int MODE>
__device__ __forceinline__ void load_span(SpanRaw<MODE>& raw, const uint8_t* wrow, const uint8_t* srow, int span,
                                          int t, int k, uint64_t pol) {
    const int k0 = span * 64 + 16 * t;
    if constexpr (MODE == 1) {
        raw.v = ld_stream_v4(wrow + k0, pol);
    } else {
        raw.lo = ld_nc_v2(wrow + k0 / 2);
        if constexpr (MODE == 2) raw.hi = ld_nc_u32(wrow + k / 2 + k0 / 4);
        raw.rel = ld_nc_u8(srow + k0 / 16);
    }
}

// 16 int8 grid values of one row's span slice, as four words (byte j = column 16t + j).
//
// Mode 2 runs two columns per instruction in f16x2, exactly. The 6-bit codes of
// a word's 8 columns are assembled bytewise (low nibbles from the code bytes,
// top bits from the matching nibble of the top-bit word, which one byte permute
// lines up); (1024 + code) is the code OR-ed into 0x6400, minus 1056 gives
// level = code - 32. One fused multiply-add level * rel + 1536 rounds the exact
// value once: where it lies in [1024, 2048) (f16 spacing 1) that is
// 1536 + rint(level * rel), round half to even as the reference's rint of its
// (exact) fp32 product. Rounding is monotone, so clamping the sum to
// [1409, 1663] afterwards equals clamping rint(level * rel) to +-127, and the
// low byte of 0x6400 + 512 + v is v mod 256.
//
// Mode 3 looks the grid values up in a table of the slot's codebook: row r (an
// FP8 relative-scale byte) holds grid_byte(codebook[c], rel(r)) for the codes
// c = 0..15, built with the same grid_byte, so the lookup is exact. Four
// columns take three byte permutes: the low three code bits select from codes
// 0-7 and from codes 8-15, bit 3 picks between the two.
template <int MODE>
__device__ __forceinline__ void dequant_span(const SpanRaw<MODE>& raw, const uint4* tab, uint32_t (&o)[4]) {
    if constexpr (MODE == 1) {
        o[0] = raw.v.x;
        o[1] = raw.v.y;
        o[2] = raw.v.z;
        o[3] = raw.v.w;
    } else if constexpr (MODE == 2) {
        const uint32_t rel2 = e4m3x2_to_f16x2(raw.rel | (raw.rel << 8));
        const uint32_t hi4 = raw.hi >> 4;
        uint32_t r[8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // columns 8h..8h+7: pairs m = 4h + b are columns 2m, 2m + 1
            const uint32_t L = h ? raw.lo.y : raw.lo.x;  // byte b: column 2m low nibble, 2m + 1 high nibble
            // byte b of X: nibble m of the top-bit word in its low nibble (bits 0-1: column 2m, 2-3: 2m + 1)
            const uint32_t X = __byte_perm(raw.hi, hi4, h ? 0x7362u : 0x5140u);
            const uint32_t ce = (L & 0x0F0F0F0Fu) | ((X << 4) & 0x30303030u);         // byte b: code of 2m
            const uint32_t co = ((L >> 4) & 0x0F0F0F0Fu) | ((X << 2) & 0x30303030u);  // byte b: code of 2m + 1
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint32_t pair = __byte_perm(ce, co, b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12));
                const uint32_t codes = (pair & 0x00FF00FFu) | 0x64006400u;  // f16x2 1024 + code
                r[4 * h + b] = h2_clamp_grid(h2_fma(h2_sub(codes, 0x64206420u), rel2, 0x66006600u));
            }
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) o[w] = __byte_perm(r[2 * w], r[2 * w + 1], 0x6420u);
    } else {
        const uint4 T = tab[raw.rel];  // grid bytes of codes 0-15 at this relative scale
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t word = h ? raw.lo.y : raw.lo.x;  // columns 8h..8h+7, nibble j = column 8h + j
            const uint32_t idx = word & 0x77777777u;
            const uint32_t pick = ((word >> 1) & 0x44444444u) | 0x32103210u;  // selector + 4 where code >= 8
            o[2 * h] = __byte_perm(__byte_perm(T.x, T.y, idx), __byte_perm(T.z, T.w, idx), pick);
            o[2 * h + 1] =
                __byte_perm(__byte_perm(T.x, T.y, idx >> 16), __byte_perm(T.z, T.w, idx >> 16), pick >> 16);
        }
    }
}

// Mode 3: the grid table of one slot (256 relative-scale bytes x 16 codes), entries
// e = first, first + n, ... written by threads whose code (e & 15) matches their
// codebook value cb (n and first are such that e & 15 == lane & 15).
__device__ __forceinline__ void build_grid_table(uint8_t* tab, float cb, int first, int n) {
    for (int e = first; e < 4096; e += n) tab[e] = static_cast<uint8_t>(grid_byte(cb, fp8_to_float(e >> 4)));
}

__device__ __forceinline__ int group_pair(const int4& ids4, int c) {
    const uint32_t word = static_cast<uint32_t>(c < 2 ? ids4.x : c < 4 ? ids4.y : c < 6 ? ids4.z : ids4.w);
    return static_cast<int>((word >> (16 * (c & 1))) & 0xffffu);
}

template <int MODE>
__device__ __forceinline__ float channel_scale(const W8Role& r, int slot, int row) {
    const uint8_t* p = r.s + slot * r.s_slot + row * r.s_row + (MODE == 1 ? 0 : r.k / 16);
    return __ldg(reinterpret_cast<const float*>(p));
}

// U: spans whose loads are all issued before the first MMA (4, or 8 when a
// task's span count allows, so a batch-1 task is a single round trip).
template <int MODE, bool DOWN, int U>
__global__ void __launch_bounds__(256) w8a8_gemv_kernel(W8GemvArgs a) {
    grid_launch_dependents();  // programmatic dependent launch: the next kernel may start its launch
    grid_dependency_wait();    // the previous kernel's results are visible from here
    __shared__ int4 s_part[8][32];
    extern __shared__ uint4 s_tab[];  // mode 3: grid tables (w8_table_smem bytes)
    int tab_slot = -1;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, warp = threadIdx.x >> 5;
    const int groups = __ldg(a.num_groups);
    const W8Role& role = a.role;
    // up: cell j's MMA rows g are gate rows 8j + g and rows g + 8 the up rows of the same j, so the epilogue
    // forms the SwiGLU rows; down: cell j is rows 16j..16j+15. Either way 16 weight rows per cell.
    constexpr bool GLU = !DOWN;
    const int tiles = role.n / 16, spans_per = role.k / 64 / a.ksplit;
    const uint64_t pol = policy_evict_first();
    // a.ksplit > 1: the CTA's a.ksplit warps share one cell (warp = K part) and add their int32 sums in
    // shared memory; a.ksplit == 1: every warp owns whole cells
    const bool team = a.ksplit > 1;
    const int first = team ? blockIdx.x : blockIdx.x * (blockDim.x >> 5) + warp;
    const int step = team ? gridDim.x : gridDim.x * (blockDim.x >> 5);
    for (int cell = first; cell < groups * tiles; cell += step) {
        const int kpart = team ? warp : 0;
        const int grp = cell / tiles, tile = cell - grp * tiles;
        const int4 head = __ldg(a.g_rec + 2 * grp);
        const int4 ids4 = __ldg(a.g_rec + 2 * grp + 1);
        const int slot = head.x, count = head.z;
        const int my_pair = g < count ? group_pair(ids4, g) : -1;
        const int8_t* arow =
            my_pair >= 0 ? a.act + static_cast<int64_t>(DOWN ? my_pair : my_pair / a.top_k) * role.k : nullptr;
        const int r0 = GLU ? tile * 8 + g : tile * 16 + g;
        const int r1 = GLU ? role.n / 2 + r0 : r0 + 8;
        const uint8_t* w0 = role.w + slot * role.w_slot + static_cast<int64_t>(r0) * role.w_row;
        const uint8_t* w1 = role.w + slot * role.w_slot + static_cast<int64_t>(r1) * role.w_row;
        const uint8_t* s0 = role.s + slot * role.s_slot + static_cast<int64_t>(r0) * role.s_row;
        const uint8_t* s1 = role.s + slot * role.s_slot + static_cast<int64_t>(r1) * role.s_row;
        const uint4* tab = nullptr;
        if constexpr (MODE == 3) {
            // the slot's grid table: one per CTA when the warps share a cell, else one per warp
            uint4* mine = s_tab + (team ? 0 : warp * 256);
            tab = mine;
            if (slot != tab_slot) {  // uniform over the threads that share the table
                tab_slot = slot;
                const float cb = __ldg(reinterpret_cast<const float*>(
                    role.s + slot * role.s_slot + (lane & 15) * role.s_row + role.k / 16 + 4));
                if (team) {
                    __syncthreads();  // the previous table's readers are done
                    build_grid_table(reinterpret_cast<uint8_t*>(mine), cb, threadIdx.x, blockDim.x);
                    __syncthreads();
                } else {
                    __syncwarp();
                    build_grid_table(reinterpret_cast<uint8_t*>(mine), cb, lane, 32);
                    __syncwarp();
                }
            }
        }
        int acc[4] = {0, 0, 0, 0};
        const int sp_end = (kpart + 1) * spans_per;
        for (int sp = kpart * spans_per; sp < sp_end; sp += U) {
            SpanRaw<MODE> raw0[U], raw1[U];
            uint4 xb[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                load_span<MODE>(raw0[u], w0, s0, sp + u, t, role.k, pol);
                load_span<MODE>(raw1[u], w1, s1, sp + u, t, role.k, pol);
                xb[u] = arow ? __ldg(reinterpret_cast<const uint4*>(arow + (sp + u) * 64 + 16 * t))
                             : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                uint32_t A0[4], A1[4];
                dequant_span<MODE>(raw0[u], tab, A0);
                dequant_span<MODE>(raw1[u], tab, A1);
                const uint32_t a1[4] = {A0[0], A1[0], A0[1], A1[1]};
                const uint32_t a2[4] = {A0[2], A1[2], A0[3], A1[3]};
                mma_s8_16832(acc, a1, xb[u].x, xb[u].y);
                mma_s8_16832(acc, a2, xb[u].z, xb[u].w);
            }
        }
        if (team) {
            s_part[warp][lane] = make_int4(acc[0], acc[1], acc[2], acc[3]);
            __syncthreads();
            if (warp == 0)
                for (int q = 1; q < a.ksplit; ++q) {  // exact integer sums: any order gives the same bits
                    const int4 v = s_part[q][lane];
                    acc[0] += v.x;
                    acc[1] += v.y;
                    acc[2] += v.z;
                    acc[3] += v.w;
                }
        }
        if (!team || warp == 0) {
            // epilogue: acc[0..1] row r0, token columns 2t, 2t+1; acc[2..3] row r1
            const float sb0 = channel_scale<MODE>(role, slot, r0), sb1 = channel_scale<MODE>(role, slot, r1);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int col = 2 * t + c;
                if (col >= count) continue;
                const int pair = group_pair(ids4, col);
                const float sa = __ldg(a.act_scale + (DOWN ? pair : pair / a.top_k));
                // projections rounded to bf16 (the reference kernel's output type)
                const float v0 = __bfloat162float(
                    __float2bfloat16_rn(__fmul_rn(__fmul_rn(__int2float_rn(acc[c]), sa), sb0)));
                const float v1 = __bfloat162float(
                    __float2bfloat16_rn(__fmul_rn(__fmul_rn(__int2float_rn(acc[2 + c]), sa), sb1)));
                if constexpr (DOWN) {
                    const float w = __ldg(a.wts + pair);
                    a.pair_out[static_cast<int64_t>(pair) * role.n + r0] = __fmul_rn(v0, w);
                    a.pair_out[static_cast<int64_t>(pair) * role.n + r1] = __fmul_rn(v1, w);
                } else {  // bf16(bf16(silu(gate)) * up) of row r0
                    const float act = __bfloat162float(__float2bfloat16_rn(v0 / (1.0f + expf(-v0))));
                    a.up_out[static_cast<int64_t>(pair) * (role.n / 2) + r0] = __float2bfloat16_rn(act * v1);
                }
            }
            if constexpr (DOWN) {
                // the last cell of this row tile sums its rows' route slots in slot order
                int old = -1;
                if (a.out) {
                    __syncwarp();
                    if (lane == 0) {
                        w8_fence();
                        old = atomicAdd(a.cmb_cnt + tile, 1);
                    }
                    old = __shfl_sync(0xffffffffu, old, 0);
                }
                if (old == groups - 1) {
                    w8_fence();
                    const int n = role.n;
                    for (int i = lane; i < a.tokens * 16; i += 32) {
                        const int64_t tok = i >> 4;
                        const int row = tile * 16 + (i & 15);
                        float sum = 0.0f;
                        for (int sl = 0; sl < a.top_k; ++sl)
                            sum = __fadd_rn(sum, __ldcg(a.pair_out + (tok * a.top_k + sl) * n + row));
                        store_any(a.out, a.out_dtype, tok * n + row, sum);
                    }
                }
            }
        }
        if (team) __syncthreads();  // s_part is reused by the next cell
    }
}

// Upper bound of expert groups: every group holds >= 1 pair.
int64_t max_groups(int64_t pairs) { return pairs; }

// K parts per tile: split only while the tiles alone leave the GPU idle.
int split_for(int64_t cells, int spans) {
    for (int ks = 8; ks > 1; --ks)
        if (cells * ks <= kW8TargetWarps && spans % (ks * kW8Unroll) == 0) return ks;
    return 1;
}

// Dynamic shared memory of a W8A8 GEMV launch: mode 3 keeps a 4 KB grid table
// per CTA (warps sharing a cell) or per warp.
size_t w8_table_smem(int mode, int ks) { return mode == 3 ? 4096u * (ks > 1 ? 1 : kW8GemvThreads / 32) : 0; }

int rot_threads(int K) { return K < 1024 ? K : 1024; }
size_t rot_smem(int K) { return static_cast<size_t>(rot_threads(K)) * sizeof(double) + K * sizeof(float); }

template <int MODE>
cudaError_t launch_mode(const DramaB200W8a8Bank& b, int64_t tokens, int top_k, void* out, int out_dtype,
                        float* pair_out, const W8a8Workspace& ws, int sm_count, cudaStream_t s) {
    const int64_t P = tokens * top_k;
    const int H = b.hidden, I = b.intermediate;
    const int64_t gmax = max_groups(P);
    // split tiles: one CTA of ks warps per cell; otherwise four single-warp cells per CTA
    auto cta_threads = [](int ks) { return ks > 1 ? 32 * ks : kW8GemvThreads; };
    auto grid_cells = [&](int64_t cells, int ks) {
        const int per_cta = ks > 1 ? 1 : kW8GemvThreads / 32;
        const int64_t ctas = (cells + per_cta - 1) / per_cta;
        const int64_t cap = static_cast<int64_t>(sm_count) * (ks > 1 ? 32 / ks : 16);
        return static_cast<unsigned>(ctas < 1 ? 1 : (ctas > cap ? cap : ctas));
    };
    W8GemvArgs up{};
    up.role = W8Role{static_cast<const uint8_t*>(b.w13), static_cast<const uint8_t*>(b.w13_scale), b.w13_slot_stride,
                     b.w13_row_stride, b.w13_scale_slot_stride, b.w13_scale_row_stride, 2 * I, H};
    up.g_rec = ws.g_rec;
    up.num_groups = ws.num_groups;
    up.act = ws.xq;
    up.act_scale = ws.xs;
    up.top_k = top_k;
    up.ksplit = split_for(gmax * (2 * I / 16), H / 64);  // a cell: 8 gate rows and their 8 up rows
    up.up_out = ws.up;
    const dim3 up_grid(grid_cells(gmax * (2 * I / 16), up.ksplit)), up_block(cta_threads(up.ksplit));
    cudaError_t err = (H / 64 / up.ksplit) % 8 == 0
                          ? launch_pdl(w8a8_gemv_kernel<MODE, false, 8>, up_grid, up_block,
                                       w8_table_smem(MODE, up.ksplit), s, up)
                          : launch_pdl(w8a8_gemv_kernel<MODE, false, 4>, up_grid, up_block,
                                       w8_table_smem(MODE, up.ksplit), s, up);
    if (err != cudaSuccess) return err;
    err = launch_pdl(w8a8_act_kernel, dim3(static_cast<unsigned>(P)), dim3(rot_threads(I)), rot_smem(I), s, ws.up, I,
                     ws.hq, ws.hs);
    if (err != cudaSuccess) return err;
    W8GemvArgs dn{};
    dn.role = W8Role{static_cast<const uint8_t*>(b.w2), static_cast<const uint8_t*>(b.w2_scale), b.w2_slot_stride,
                     b.w2_row_stride, b.w2_scale_slot_stride, b.w2_scale_row_stride, H, I};
    dn.g_rec = ws.g_rec;
    dn.num_groups = ws.num_groups;
    dn.act = ws.hq;
    dn.act_scale = ws.hs;
    dn.top_k = top_k;
    dn.ksplit = split_for(gmax * (H / 16), I / 64);
    dn.pair_out = pair_out;
    dn.wts = ws.wts;
    dn.cmb_cnt = ws.cmb_cnt;
    dn.out = out;
    dn.out_dtype = out_dtype;
    dn.tokens = tokens;
    const dim3 dn_grid(grid_cells(gmax * (H / 16), dn.ksplit)), dn_block(cta_threads(dn.ksplit));
    return (I / 64 / dn.ksplit) % 8 == 0
               ? launch_pdl(w8a8_gemv_kernel<MODE, true, 8>, dn_grid, dn_block, w8_table_smem(MODE, dn.ksplit), s,
                            dn)
               : launch_pdl(w8a8_gemv_kernel<MODE, true, 4>, dn_grid, dn_block, w8_table_smem(MODE, dn.ksplit), s,
                            dn);
}

// ---------------------------------------------------------------------------
// GPTQ W4A16 (mode 0) on the same schedule: grouping, split-K GEMVs with tokens
// as the MMA N dimension, SwiGLU, down GEMV with the fused slot combine.
// Weights are dequantised the way the reference's kernel does it
// (quantized_kernels.py:139-147): w = bf16((code - zp) * scale) per element,
// then bf16 MMAs with fp32 accumulation.
//
// Per 128-column block (one scale group) thread t of a quad takes the 32
// columns 32t..32t+31 of its two weight rows (four int32 words) and of its
// token row. A word's nibbles i and i + 4 become one bf16x2 pair (one shift and
// one LOP3 with the 128.0 bias 0x4300 per pair, then code - zp exactly and one
// rounding of the product with the scale); the token row is paired the same
// way with byte permutes, so each product still joins equal columns.
// ---------------------------------------------------------------------------
struct I4Role {
    const int32_t* w;       // [slots][n][k/8]
    const void* s;          // [slots][n][k/128] bf16 or f16
    const int32_t* z;       // [slots][n/8][k/128] or NULL (8)
    int64_t w_slot, w_row, s_slot, s_row, z_slot, z_row;  // elements
    int s_dtype;
    int n, k;
};

struct I4GemvArgs {
    I4Role role;
    const int4* g_rec;
    const int32_t* num_groups;
    const __nv_bfloat16* act;  // up: x [T][k]; down: SwiGLU rows in gu [P][2I] (row stride act_stride)
    int64_t act_stride;
    int top_k;
    int ksplit;                // warps per team (K shares per tile)
    __nv_bfloat16* gu;         // up: [P][2I]
    float* pair_out;           // down
    const float* wts;
    int32_t* cmb_cnt;
    void* out;
    int out_dtype;
    int64_t tokens;
};

__device__ __forceinline__ float i4_scale(const void* p, int dtype, int64_t i) {
    return dtype == DRAMA_B200_BF16 ? __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(p) + i))
                                    : __half2float(__ldg(static_cast<const __half*>(p) + i));
}

// One 128-column block of one warp: the raw loads of a row pair (rows g and
// g + 8 of a tile) and of the token row, issued one block ahead of the MMAs
// that consume them.
struct I4Rows {
    uint4 q0, q1;    // the two weight rows' 32 nibbles
    float s0, s1;    // scales
    uint32_t z0, z1; // zero points
};
struct I4X {
    uint4 x[4];      // the token row's 32 bf16
};

__device__ __forceinline__ void i4_load_rows(I4Rows& b, const I4Role& role, const int32_t* w0, const int32_t* w1,
                                             int slot, int r0, int r1, int blk, int t, uint64_t pol) {
    b.q0 = ld_stream_v4(w0 + blk * 16 + 4 * t, pol);
    b.q1 = ld_stream_v4(w1 + blk * 16 + 4 * t, pol);
    const int64_t so = slot * role.s_slot + blk;
    b.s0 = i4_scale(role.s, role.s_dtype, so + static_cast<int64_t>(r0) * role.s_row);
    b.s1 = i4_scale(role.s, role.s_dtype, so + static_cast<int64_t>(r1) * role.s_row);
    b.z0 = b.z1 = 8u;
    if (role.z) {
        const int32_t* zp = role.z + slot * role.z_slot + blk;
        b.z0 = (static_cast<uint32_t>(__ldg(zp + (r0 >> 3) * role.z_row)) >> (4 * (r0 & 7))) & 15u;
        b.z1 = (static_cast<uint32_t>(__ldg(zp + (r1 >> 3) * role.z_row)) >> (4 * (r1 & 7))) & 15u;
    }
}

__device__ __forceinline__ void i4_load_x(I4X& b, const __nv_bfloat16* arow, int blk, int t) {
#pragma unroll
    for (int v = 0; v < 4; ++v)
        b.x[v] = arow ? __ldg(reinterpret_cast<const uint4*>(arow + blk * 128 + 32 * t) + v) : make_uint4(0u, 0u, 0u, 0u);
}

template <bool BF16>
__device__ __forceinline__ void i4_mma(const I4Rows& b, const I4X& xb, float (&acc)[4]) {
    const uint32_t zb0 = (0x4300u + b.z0) * 0x10001u, zb1 = (0x4300u + b.z1) * 0x10001u;
    const __nv_bfloat162 sp0 = __floats2bfloat162_rn(b.s0, b.s0);
    const __nv_bfloat162 sp1 = __floats2bfloat162_rn(b.s1, b.s1);
    const uint32_t sc0 = *reinterpret_cast<const uint32_t*>(&sp0);
    const uint32_t sc1 = *reinterpret_cast<const uint32_t*>(&sp1);
    const uint32_t W0[4] = {b.q0.x, b.q0.y, b.q0.z, b.q0.w};
    const uint32_t W1[4] = {b.q1.x, b.q1.y, b.q1.z, b.q1.w};
    const uint32_t X[16] = {xb.x[0].x, xb.x[0].y, xb.x[0].z, xb.x[0].w, xb.x[1].x, xb.x[1].y, xb.x[1].z, xb.x[1].w,
                            xb.x[2].x, xb.x[2].y, xb.x[2].z, xb.x[2].w, xb.x[3].x, xb.x[3].y, xb.x[3].z, xb.x[3].w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {  // word w: columns 8w..8w+7 of this thread's 32
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // pairs (2h, 2h+4) and (2h+1, 2h+5)
            const uint32_t A[4] = {int4_pair<BF16>(W0[w], 2 * h, zb0, sc0, b.s0),
                                   int4_pair<BF16>(W1[w], 2 * h, zb1, sc1, b.s1),
                                   int4_pair<BF16>(W0[w], 2 * h + 1, zb0, sc0, b.s0),
                                   int4_pair<BF16>(W1[w], 2 * h + 1, zb1, sc1, b.s1)};
            // token columns (2h, 2h+4) and (2h+1, 2h+5): low or high halves of x words 4w+h, 4w+h+2
            const uint32_t xa = X[4 * w + h], xc = X[4 * w + h + 2];
            mma_bf16_16816(acc, A, __byte_perm(xa, xc, 0x5410u), __byte_perm(xa, xc, 0x7632u));
        }
    }
}

// The row pairs a warp multiplies: one pair for the down projection; for the
// gate/up projection (GLU) the gate rows g, g + 8 of tile j and the up rows
// I + g, I + g + 8 of the same j, so that SiLU(gate) * up is formed in the
// epilogue and no separate SwiGLU pass is needed.
template <bool GLU>
struct I4Stage {
    I4Rows r[GLU ? 2 : 1];
    I4X x;
};

struct I4RowPtrs {
    const int32_t* w0[2];
    const int32_t* w1[2];
    int r0[2], r1[2];
};

template <bool GLU>
__device__ __forceinline__ void i4_load_stage(I4Stage<GLU>& st, const I4Role& role, const I4RowPtrs& rp,
                                              const __nv_bfloat16* arow, int slot, int blk, int t, uint64_t pol) {
#pragma unroll
    for (int i = 0; i < (GLU ? 2 : 1); ++i)
        i4_load_rows(st.r[i], role, rp.w0[i], rp.w1[i], slot, rp.r0[i], rp.r1[i], blk, t, pol);
    i4_load_x(st.x, arow, blk, t);
}

// Epilogue of one cell (one warp): gate/up -> bf16(bf16(silu(gate)) * up) into
// the gate half of gu (GLU), or down -> weighted fp32 partials followed, for
// the last cell of a row tile, by the slot sum.
template <bool DOWN, bool GLU>
__device__ __forceinline__ void i4_epilogue(const I4GemvArgs& a, const float (&acc)[2][4], const int4& ids4,
                                            int count, int tile, const I4RowPtrs& rp, int groups, int lane, int t) {
    const I4Role& role = a.role;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const int col = 2 * t + c;
        if (col >= count) continue;
        const int pair = group_pair(ids4, col);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = h ? rp.r1[0] : rp.r0[0];
            const float v = __bfloat162float(__float2bfloat16_rn(acc[0][2 * h + c]));  // projection in bf16
            if constexpr (DOWN) {
                a.pair_out[static_cast<int64_t>(pair) * role.n + row] = __fmul_rn(v, __ldg(a.wts + pair));
            } else if constexpr (GLU) {
                const float up = __bfloat162float(__float2bfloat16_rn(acc[1][2 * h + c]));
                const float act = __bfloat162float(__float2bfloat16_rn(v / (1.0f + expf(-v))));
                a.gu[static_cast<int64_t>(pair) * role.n + row] = __float2bfloat16_rn(act * up);
            } else {
                a.gu[static_cast<int64_t>(pair) * role.n + row] = __float2bfloat16_rn(v);
            }
        }
    }
    if constexpr (DOWN) {
        if (a.out) {
            // the last cell of this row tile sums its rows' route slots in slot order
            __syncwarp();
            int old = 0;
            if (lane == 0) {
                w8_fence();
                old = atomicAdd(a.cmb_cnt + tile, 1);
            }
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == groups - 1) {
                w8_fence();
                const int n = role.n;
                for (int i = lane; i < a.tokens * 16; i += 32) {
                    const int64_t tok = i >> 4;
                    const int row = tile * 16 + (i & 15);
                    float sum = 0.0f;
                    for (int sl = 0; sl < a.top_k; ++sl)
                        sum = __fadd_rn(sum, __ldcg(a.pair_out + (tok * a.top_k + sl) * n + row));
                    store_any(a.out, a.out_dtype, tok * n + row, sum);
                }
            }
        }
    }
}

// Row pointers of a cell: tile j of the down rows, or gate tile j plus up tile j.
template <bool GLU>
__device__ __forceinline__ I4RowPtrs i4_rows(const I4Role& role, int slot, int tile, int g) {
    I4RowPtrs rp{};
#pragma unroll
    for (int i = 0; i < (GLU ? 2 : 1); ++i) {
        rp.r0[i] = (i ? role.n / 2 : 0) + tile * 16 + g;
        rp.r1[i] = rp.r0[i] + 8;
        rp.w0[i] = role.w + slot * role.w_slot + static_cast<int64_t>(rp.r0[i]) * role.w_row;
        rp.w1[i] = rp.w0[i] + 8 * role.w_row;
    }
    return rp;
}

// The warps of a CTA form teams of KS (a.ksplit) warps; a team owns one cell
// (group, 16-row tile) at a time and warp q of the team takes the q-th
// contiguous share of the K blocks, streaming it with the next block's loads in
// flight while the current one is multiplied. The shares are added in warp
// order through shared memory, so no global fence or atomic reduces a tile.
// Used when there are few cells (batch 1): one team of up to 8 warps per CTA.
template <bool DOWN, bool BF16>
__global__ void __launch_bounds__(256) int4_gemv_kernel(I4GemvArgs a) {
    constexpr bool GLU = !DOWN;
    grid_launch_dependents();  // programmatic dependent launch: the next kernel may start its launch
    grid_dependency_wait();    // the previous kernel's results are visible from here
    __shared__ float4 s_part[GLU ? 2 : 1][8][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int KS = a.ksplit, teams = (blockDim.x >> 5) / KS, team = warp / KS, q = warp - team * KS;
    const int groups = __ldg(a.num_groups);
    const I4Role& role = a.role;
    const int tiles = role.n / (GLU ? 32 : 16), blocks = role.k / 128;
    const int per = blocks / KS, b_lo = q * per, b_hi = b_lo + per;
    const uint64_t pol = policy_evict_first();
    const int total = groups * tiles;
    // every warp runs the same number of rounds, so the barriers below are uniform
    for (int base = blockIdx.x * teams; base < total; base += gridDim.x * teams) {
        const int cell = base + team;
        const bool live = cell < total;
        const int grp = live ? cell / tiles : 0, tile = live ? cell - grp * tiles : 0;
        const int4 head = __ldg(a.g_rec + 2 * grp);
        const int4 ids4 = __ldg(a.g_rec + 2 * grp + 1);
        const int slot = head.x, count = live ? head.z : 0;
        const int my_pair = g < count ? group_pair(ids4, g) : -1;
        const __nv_bfloat16* arow =
            my_pair >= 0 ? a.act + static_cast<int64_t>(DOWN ? my_pair : my_pair / a.top_k) * a.act_stride
                         : nullptr;
        const I4RowPtrs rp = i4_rows<GLU>(role, slot, tile, g);
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        if (live) {
            I4Stage<GLU> cur, nxt;
            i4_load_stage<GLU>(cur, role, rp, arow, slot, b_lo, t, pol);
            for (int blk = b_lo; blk < b_hi; blk += 2) {
                if (blk + 1 < b_hi) i4_load_stage<GLU>(nxt, role, rp, arow, slot, blk + 1, t, pol);
#pragma unroll
                for (int i = 0; i < (GLU ? 2 : 1); ++i) i4_mma<BF16>(cur.r[i], cur.x, acc[i]);
                if (blk + 1 >= b_hi) break;
                if (blk + 2 < b_hi) i4_load_stage<GLU>(cur, role, rp, arow, slot, blk + 2, t, pol);
#pragma unroll
                for (int i = 0; i < (GLU ? 2 : 1); ++i) i4_mma<BF16>(nxt.r[i], nxt.x, acc[i]);
            }
        }
        if (KS > 1) {
#pragma unroll
            for (int i = 0; i < (GLU ? 2 : 1); ++i)
                s_part[i][warp][lane] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            __syncthreads();
            if (q == 0) {
#pragma unroll
                for (int i = 0; i < (GLU ? 2 : 1); ++i) {
                    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
                    for (int p = 0; p < KS; ++p) {  // warp (= K) order
                        const float4 v = s_part[i][warp + p][lane];
                        acc[i][0] += v.x;
                        acc[i][1] += v.y;
                        acc[i][2] += v.z;
                        acc[i][3] += v.w;
                    }
                }
            }
        }
        if (q == 0 && live) i4_epilogue<DOWN, GLU>(a, acc, ids4, count, tile, rp, groups, lane, t);
        if (KS > 1) __syncthreads();  // s_part is reused by the next cell
    }
}

// Larger batches (many cells): every warp owns whole cells and loads two K
// blocks per round trip.
template <bool DOWN, bool BF16>
__global__ void __launch_bounds__(kW8GemvThreads) int4_gemv_wide_kernel(I4GemvArgs a) {
    constexpr bool GLU = !DOWN;
    grid_launch_dependents();  // programmatic dependent launch: the next kernel may start its launch
    grid_dependency_wait();    // the previous kernel's results are visible from here
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int warps_total = gridDim.x * (kW8GemvThreads / 32);
    const int groups = __ldg(a.num_groups);
    const I4Role& role = a.role;
    const int tiles = role.n / (GLU ? 32 : 16), blocks = role.k / 128;
    const uint64_t pol = policy_evict_first();
    for (int cell = blockIdx.x * (kW8GemvThreads / 32) + (threadIdx.x >> 5); cell < groups * tiles;
         cell += warps_total) {
        const int grp = cell / tiles, tile = cell - grp * tiles;
        const int4 head = __ldg(a.g_rec + 2 * grp);
        const int4 ids4 = __ldg(a.g_rec + 2 * grp + 1);
        const int slot = head.x, count = head.z;
        const int my_pair = g < count ? group_pair(ids4, g) : -1;
        const __nv_bfloat16* arow =
            my_pair >= 0 ? a.act + static_cast<int64_t>(DOWN ? my_pair : my_pair / a.top_k) * a.act_stride
                         : nullptr;
        const I4RowPtrs rp = i4_rows<GLU>(role, slot, tile, g);
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        for (int blk = 0; blk < blocks; blk += 2) {  // blocks is even (K % 256 == 0)
            I4Stage<GLU> s0, s1;
            i4_load_stage<GLU>(s0, role, rp, arow, slot, blk, t, pol);
            i4_load_stage<GLU>(s1, role, rp, arow, slot, blk + 1, t, pol);
#pragma unroll
            for (int i = 0; i < (GLU ? 2 : 1); ++i) {
                i4_mma<BF16>(s0.r[i], s0.x, acc[i]);
                i4_mma<BF16>(s1.r[i], s1.x, acc[i]);
            }
        }
        i4_epilogue<DOWN, GLU>(a, acc, ids4, count, tile, rp, groups, lane, t);
    }
}

// Warps per CTA (= K shares per tile): the most that keep the warps within the
// target and divide the blocks, at most 8.
int int4_warps(int64_t cells, int blocks, int max_ks = 8) {
    for (int ks = max_ks; ks > 1; --ks)
        if (cells * ks <= kW8TargetWarps && blocks % ks == 0) return ks;
    return 1;
}

template <bool BF16>
cudaError_t int4_launch_fmt(const DramaB200Int4Bank& b, const void* x, int64_t tokens, int top_k, void* out,
                            int out_dtype, float* pair_out, const W8a8Workspace& ws, int sm_count, cudaStream_t s) {
    const int64_t P = tokens * top_k;
    const int H = b.hidden, I = b.intermediate;
    const int64_t gmax = max_groups(P);
    auto grid_wide = [&](int64_t cells) {
        const int64_t ctas = (cells + kW8GemvThreads / 32 - 1) / (kW8GemvThreads / 32);
        const int64_t cap = static_cast<int64_t>(sm_count) * 16;
        return static_cast<unsigned>(ctas < 1 ? 1 : (ctas > cap ? cap : ctas));
    };
    // a CTA is one team of ks warps (ks > 1) or four single-warp teams
    auto team_threads = [](int ks) { return 32 * (ks > 1 ? ks : 4); };
    auto grid_cells = [&](int64_t cells, int ks) {
        const int teams = ks > 1 ? 1 : 4;
        const int64_t ctas = (cells + teams - 1) / teams;
        const int64_t cap = static_cast<int64_t>(sm_count) * (ks > 1 ? 32 / ks : 8);  // up to 32 warps per SM
        return static_cast<unsigned>(ctas < 1 ? 1 : (ctas > cap ? cap : ctas));
    };
    I4GemvArgs up{};
    up.role = I4Role{b.w13, b.w13_scale, b.w13_zeros, b.w13_slot_stride, b.w13_row_stride, b.w13_scale_slot_stride,
                     b.w13_scale_row_stride, b.w13_zeros_slot_stride, b.w13_zeros_row_stride, b.scale_dtype, 2 * I, H};
    up.g_rec = ws.g_rec;
    up.num_groups = ws.num_groups;
    up.act = static_cast<const __nv_bfloat16*>(x);
    up.act_stride = H;
    up.top_k = top_k;
    up.gu = ws.up;
    const int64_t up_cells = gmax * (I / 16);  // a cell is gate tile j with up tile j
    // two row pairs per warp: teams of at most 4 warps (one wave), and only while the cells alone are few
    up.ksplit = up_cells * 8 <= kW8TargetWarps ? int4_warps(up_cells, H / 128, 4) : 1;
    cudaError_t err =
        up.ksplit > 1
            ? launch_pdl(int4_gemv_kernel<false, BF16>, dim3(grid_cells(up_cells, up.ksplit)),
                         dim3(team_threads(up.ksplit)), 0, s, up)
            : launch_pdl(int4_gemv_wide_kernel<false, BF16>, dim3(grid_wide(up_cells)), dim3(kW8GemvThreads), 0, s, up);
    if (err != cudaSuccess) return err;
    I4GemvArgs dn{};
    dn.role = I4Role{b.w2, b.w2_scale, b.w2_zeros, b.w2_slot_stride, b.w2_row_stride, b.w2_scale_slot_stride,
                     b.w2_scale_row_stride, b.w2_zeros_slot_stride, b.w2_zeros_row_stride, b.scale_dtype, H, I};
    dn.g_rec = ws.g_rec;
    dn.num_groups = ws.num_groups;
    dn.act = ws.up;
    dn.act_stride = 2 * I;
    dn.top_k = top_k;
    dn.pair_out = pair_out;
    dn.wts = ws.wts;
    dn.cmb_cnt = ws.cmb_cnt;
    dn.out = out;
    dn.out_dtype = out_dtype;
    dn.tokens = tokens;
    const int64_t dn_cells = gmax * (H / 16);
    dn.ksplit = int4_warps(dn_cells, I / 128);
    return dn.ksplit > 1
               ? launch_pdl(int4_gemv_kernel<true, BF16>, dim3(grid_cells(dn_cells, dn.ksplit)),
                            dim3(team_threads(dn.ksplit)), 0, s, dn)
               : launch_pdl(int4_gemv_wide_kernel<true, BF16>, dim3(grid_wide(dn_cells)), dim3(kW8GemvThreads), 0, s,
                            dn);
}

}  // namespace

size_t w8a8_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, char* base,
                             W8a8Workspace* ws) {
    const int64_t P = tokens * top_k;
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return p;
    };
    W8a8Workspace w{};
    w.status = reinterpret_cast<int32_t*>(take(16));
    w.num_groups = reinterpret_cast<int32_t*>(take(16));
    w.order = reinterpret_cast<int32_t*>(take(P * 4));
    w.g_rec = reinterpret_cast<int4*>(take(P * 32));
    w.xq = reinterpret_cast<int8_t*>(take(static_cast<size_t>(tokens) * hidden));
    w.xs = reinterpret_cast<float*>(take(tokens * 4));
    w.up = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(P) * 2 * intermediate * 2));
    w.hq = reinterpret_cast<int8_t*>(take(static_cast<size_t>(P) * intermediate));
    w.hs = reinterpret_cast<float*>(take(P * 4));
    w.wts = reinterpret_cast<float*>(take(P * 4));
    w.pair_out = reinterpret_cast<float*>(take(static_cast<size_t>(P) * hidden * 4));
    w.cmb_cnt = reinterpret_cast<int32_t*>(take(static_cast<size_t>(hidden / 16) * 4));
    // The one-launch INT4 layer's arrival tickets (int4_layer.cu) live in bytes
    // 64..79 of the status chunk: every workspace layout of the library starts
    // with that 256-byte chunk and writes only its first 16 bytes, so tickets
    // that the last arriver leaves at zero stay zero whatever layout (token
    // count, backend) uses the same zero-filled workspace in between.
    w.layer_tickets = base ? w.status + 16 : nullptr;
    if (tokens == 1)  // the layer's partial rows
        w.layer_part = reinterpret_cast<float*>(take(static_cast<size_t>(kMaxLayerUnits) * hidden * 4));
    if (ws) *ws = w;
    return off;
}

cudaError_t w8a8_decode_launch(const DramaB200W8a8Bank& bank, const void* x, int64_t tokens, int top_k,
                               const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                               int out_dtype, float* pair_out, const W8a8Workspace& ws, int sm_count,
                               cudaStream_t s) {
    float* po = pair_out ? pair_out : ws.pair_out;
    W8PrepArgs pa{ids, ids_dtype, weights, weights_dtype, static_cast<const __nv_bfloat16*>(x), tokens * top_k,
                  bank.slots, bank.hidden, bank.intermediate, po, ws};
    // CTA 0 buckets (34 ints per slot); CTAs 1..T rotate a token row with all 1024 threads
    const size_t bucket_smem = static_cast<size_t>(34) * bank.slots * sizeof(int);
    const size_t rot = 1024 * sizeof(double) + static_cast<size_t>(bank.hidden) * sizeof(float);
    const size_t smem = bucket_smem > rot ? bucket_smem : rot;
    static bool configured = false;  // benign race: identical values
    if (!configured) {
        cudaError_t err = cudaFuncSetAttribute(w8a8_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               200 * 1024);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(w8a8_act_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (err != cudaSuccess) return err;
        configured = true;
    }
    cudaError_t err = launch_pdl(w8a8_prep_kernel, dim3(static_cast<unsigned>(1 + tokens)), dim3(1024), smem, s, pa);
    if (err != cudaSuccess) return err;
    switch (bank.mode) {
        case 1: return launch_mode<1>(bank, tokens, top_k, out, out_dtype, po, ws, sm_count, s);
        case 2: return launch_mode<2>(bank, tokens, top_k, out, out_dtype, po, ws, sm_count, s);
        default: return launch_mode<3>(bank, tokens, top_k, out, out_dtype, po, ws, sm_count, s);
    }
}

cudaError_t int4_rows_launch(const DramaB200Int4Bank& bank, const void* x, int64_t tokens, int top_k,
                             const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                             int out_dtype, float* pair_out, const W8a8Workspace& ws, int sm_count, cudaStream_t s) {
    float* po = pair_out ? pair_out : ws.pair_out;
    W8PrepArgs pa{ids, ids_dtype, weights, weights_dtype, static_cast<const __nv_bfloat16*>(x), tokens * top_k,
                  bank.slots, bank.hidden, bank.intermediate, po, ws};
    static bool configured = false;  // benign race: identical values
    if (!configured) {
        const cudaError_t err = cudaFuncSetAttribute(w8a8_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     200 * 1024);
        if (err != cudaSuccess) return err;
        configured = true;
    }
    // CTA 0 alone: the grouping (W4A16 keeps the activations in bf16)
    cudaError_t err = launch_pdl(w8a8_prep_kernel, dim3(1), dim3(1024), static_cast<size_t>(34) * bank.slots * sizeof(int),
                                 s, pa);
    if (err != cudaSuccess) return err;
    return bank.scale_dtype == DRAMA_B200_BF16
               ? int4_launch_fmt<true>(bank, x, tokens, top_k, out, out_dtype, po, ws, sm_count, s)
               : int4_launch_fmt<false>(bank, x, tokens, top_k, out, out_dtype, po, ws, sm_count, s);
}

}  // namespace drama
