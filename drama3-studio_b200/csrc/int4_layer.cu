// GPTQ W4A16 routed experts for one decode row in ONE launch.
//
// The arithmetic is drama_b200_int4_decode's (QuantizedExpertBackend mode 0,
// src/drama_low_vram/quantized_kernels.py:217-248): each weight is
// bf16((code - zero) * scale), gate and up are the bf16 roundings of their
// fp32 sums, SiLU(gate) is rounded to bf16 before the product with up, the
// down projection is rounded to bf16, multiplied by its route weight in fp32
// and the slots are added in slot order.
//
// Schedule (the fused FP8 layer's, decode_layer.cu, without the router): one
// wave of 4-CTA clusters; cluster u owns unit u = (route slot j, part p), a run
// of 12 16-wide tiles of the intermediate dimension of expert ids[j], and CTA
// r of the cluster
//   1. streams the unit's (gate tile, up tile) row pairs, bytes
//      [r H/8, (r+1) H/8) of each packed row (its quarter of K), into 12
//      shared-memory stages that all stay resident (one 5-D tensor-map load
//      each, 128-byte swizzle, no multicast), and the unit's down columns of
//      rows [r H/4, (r+1) H/4) beside them (3-D tensor-map loads);
//   2. dequantises each 128-wide K block in registers and multiplies it with
//      its quarter of the token row on bf16 mma.sync fragments, adds the K
//      blocks per row and stores the sums into every CTA of the cluster
//      (distributed shared memory); after the cluster barrier each CTA sums
//      the quarters in rank order and forms the unit's SiLU(gate) * up;
//   3. multiplies its down rows by those values (dequantised the same way):
//      a partial down projection, stored in fp32;
//   4. takes an arrival ticket (one acquire-release atomic per CTA); the last
//      CTA of quarter r sums, for every row, each slot's parts in part order,
//      rounds, weights, and adds the slots in slot order.
// This file serves the reference's shape (hidden 2048, intermediate 768,
// top-8: four units per slot); int4_layer_supported says when, and every other
// call keeps the grouped three-launch schedule of w8a8_decode.cu.
#include <cooperative_groups.h>

#include "common.cuh"
#include "grouped.cuh"
#include "int4.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace drama {

namespace {

namespace cg = cooperative_groups;

constexpr int kIlCluster = 4;
constexpr int kIlWarps = 16;                       // consumer warps
constexpr int kIlThreads = (kIlWarps + 1) * 32;   // + one TMA producer warp
constexpr int kIlConsumers = kIlWarps * 32;
constexpr int kIlH = 2048, kIlI = 768, kIlK = 8;  // the shape this kernel is built for
constexpr int kIlParts = 4;                       // units per route slot
constexpr int kIlUnits = kIlK * kIlParts;
static_assert(kIlUnits <= kMaxLayerUnits, "partial rows of the workspace");
constexpr int kIlTiles = kIlI / 16 / kIlParts;    // 16-wide intermediate tiles per unit (12)
constexpr int kIlHq = kIlH / kIlCluster;          // this CTA's quarter of H (512)
constexpr int kIlKbq = kIlHq / 128;               // 128-wide K blocks in a quarter (4)
constexpr int kIlStage = 32 * kIlHq / 2;          // 16 gate + 16 up rows x a quarter of K, packed (8 KB)
constexpr int kIlW2Row = kIlTiles * 8;            // a down row's unit columns, packed (96 bytes)
constexpr int kIlW2Box = 256;                     // down rows per tensor-map box
constexpr int kIlCells = kIlTiles * kIlKbq;       // (stage, K block) cells of gate/up (48)
constexpr int kIlRowTiles = kIlHq / 16;           // 16-row tiles of the down projection (32)
static_assert(kIlCells % kIlWarps == 0 && kIlRowTiles % kIlWarps == 0, "cells and row tiles per warp");

// Shared memory from a 1024-byte aligned base: the gate/up stages, the down
// rows, and the small arrays.
constexpr uint32_t kOffStages = 0;
constexpr uint32_t kOffW2 = kOffStages + kIlTiles * kIlStage;         // stages: 96 KB of gate/up rows
constexpr uint32_t kOffX = kOffW2 + kIlHq * kIlW2Row;                 // w2: 48 KB of down rows
// Each offset is the previous one plus the region named beside it. Scales and
// zero words are kept raw (as the bank stores them) and decoded where used.
constexpr int kIlRows13 = 2 * kIlTiles * 16;                             // the unit's gate and up rows (384)
constexpr uint32_t kOffS2 = kOffX + kIlHq * 2;                           // x: this CTA's quarter of the token row
constexpr uint32_t kOffZ2 = kOffS2 + kIlHq * 2 * 2;                      // down scales [512 rows][2 blocks], 16-bit
constexpr uint32_t kOffS13 = kOffZ2 + (kIlHq / 8) * 2 * 4;               // down zero words [64 row groups][2]
constexpr uint32_t kOffZ13 = kOffS13 + kIlRows13 * kIlKbq * 2;           // gate/up scales [384 rows][4 K blocks]
constexpr uint32_t kOffCell = kOffZ13 + (kIlRows13 / 8) * kIlKbq * 4;    // gate/up zero words [48][4]
constexpr uint32_t kOffXch = kOffCell + kIlCells * 32 * 4;               // cell: gate/up cell sums [48][32]
constexpr uint32_t kOffH = kOffXch + kIlCluster * kIlTiles * 32 * 4;     // xch: quarters of the row sums [4][12][32]
constexpr uint32_t kOffBar = kOffH + kIlTiles * 16 * 2;                  // h: SiLU(gate) * up [12][16] bf16
constexpr uint32_t kIlSmem = kOffBar + (kIlTiles + 1) * 8 + 1024;        // barriers, + room to align the base
static_assert(kIlSmem <= 227 * 1024, "one CTA per SM");

struct Int4LayerArgs {
    DramaB200Int4Bank bank;
    const __nv_bfloat16* x;   // [H] the token row
    const void* ids;          // [k]
    int ids_dtype;
    const void* weights;      // [k]
    int weights_dtype;
    void* out;                // [H]
    int out_dtype;
    float* pair_out;          // [k][H] or NULL
    float* part;              // [units][H] fp32 partial down projections
    int32_t* tickets;         // [4] arrivals per quarter, zero between calls
    int32_t* status;          // [4] [0] dropped routes [1] waits that ran out
    CUtensorMap w13_map;      // bytes [slot][gate|up][I][H/256][128]
    CUtensorMap w2_map;       // bytes [slot][H][I/2]
};

__device__ __forceinline__ float bf16_round_i4(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// One packed 16-byte read of a swizzled stage line pair: 16-byte unit u of
// 128-byte line l sits at unit u ^ (l & 7).
__device__ __forceinline__ uint4 i4_stage_read(const uint8_t* stage, int line, int unit) {
    return lds128(stage + line * 128 + ((unit ^ (line & 7)) << 4));
}

// The (128 + zp) bias and the scale (bf16x2 and fp32) of one weight row and
// block from the raw bank values: the 16-bit scale and the zero word whose
// nibble row % 8 is the row's zero point.
template <bool BF16>
__device__ __forceinline__ void il_params(uint32_t sbits, uint32_t zword, int row, uint32_t& zb, uint32_t& sc2,
                                          float& scf) {
    zb = int4_zero_bias((zword >> (4 * (row & 7))) & 15u);
    if constexpr (BF16) {
        sc2 = sbits * 0x10001u;
        scf = __uint_as_float(sbits << 16);
    } else {
        sc2 = 0u;
        scf = __half2float(__ushort_as_half(static_cast<unsigned short>(sbits)));
    }
}

// One 128-wide K block of two weight rows (g and g + 8 of a 16-row tile; 32
// packed nibbles each, columns 32t.. of the block for lane t) against the
// token row's matching 32 values: D[row][col 0] += sum. The nibble order is
// the grouped kernels' (w8a8_decode.cu i4_mma): words of 8 nibbles, pairs
// (i, i + 4) per bf16x2; B holds x in that pair order.
template <bool BF16>
__device__ __forceinline__ void il_block_mma(uint4 q0, uint4 q1, uint32_t zb0, uint32_t sc0, float sf0, uint32_t zb1,
                                             uint32_t sc1, float sf1, const uint32_t (&B)[16], float (&acc)[4]) {
    const uint32_t W0[4] = {q0.x, q0.y, q0.z, q0.w};
    const uint32_t W1[4] = {q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t A[4] = {int4_pair<BF16>(W0[w], 2 * h, zb0, sc0, sf0),
                                   int4_pair<BF16>(W1[w], 2 * h, zb1, sc1, sf1),
                                   int4_pair<BF16>(W0[w], 2 * h + 1, zb0, sc0, sf0),
                                   int4_pair<BF16>(W1[w], 2 * h + 1, zb1, sc1, sf1)};
            mma_bf16_16816(acc, A, B[4 * w + 2 * h], B[4 * w + 2 * h + 1]);
        }
    }
}

template <bool BF16>
__global__ void __launch_bounds__(kIlThreads, 1) int4_layer_kernel(const __grid_constant__ Int4LayerArgs a) {
    extern __shared__ __align__(1024) uint8_t il_smem_raw[];
    __shared__ int s_ids[kIlK];
    __shared__ float s_w[kIlK];
    __shared__ int s_last;

    const DramaB200Int4Bank& b = a.bank;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    cg::cluster_group cluster = cg::this_cluster();
    const int r = static_cast<int>(cluster.block_rank());
    const int unit = static_cast<int>(blockIdx.x) / kIlCluster;
    const int slot_j = unit / kIlParts, part = unit % kIlParts;
    const int tile0 = part * kIlTiles;   // first 16-wide intermediate tile of the unit
    const int blk0 = tile0 >> 3;         // its first 128-wide block of the intermediate dimension
    const int cb = 8 - (tile0 & 7);      // tiles of the unit in block blk0 (the rest are in blk0 + 1)
    int32_t* status = a.status;

    const uint32_t raw_u32 = smem_u32(il_smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
    uint8_t* base = il_smem_raw + (base_u32 - raw_u32);
    __nv_bfloat16* s_x = reinterpret_cast<__nv_bfloat16*>(base + kOffX);
    uint16_t* s_s2 = reinterpret_cast<uint16_t*>(base + kOffS2);
    uint32_t* s_z2 = reinterpret_cast<uint32_t*>(base + kOffZ2);
    uint16_t* s_s13 = reinterpret_cast<uint16_t*>(base + kOffS13);
    uint32_t* s_z13 = reinterpret_cast<uint32_t*>(base + kOffZ13);
    float* s_cell = reinterpret_cast<float*>(base + kOffCell);
    float* s_xch = reinterpret_cast<float*>(base + kOffXch);
    __nv_bfloat16* s_h = reinterpret_cast<__nv_bfloat16*>(base + kOffH);
    const uint32_t full0 = base_u32 + kOffBar, w2_bar = full0 + 8 * kIlTiles;

    if (tid == 0) {
        for (int st = 0; st < kIlTiles; ++st) mbar_init(full0 + 8 * st, 1);
        mbar_init(w2_bar, 1);
        fence_mbar_init();
    }
    cluster.barrier_arrive();  // paired with the wait before the first remote store
    grid_launch_dependents();
    grid_dependency_wait();    // ids, weights and the token row may come from the previous launch

    if (tid < kIlK) {
        const int64_t id = load_index(a.ids, a.ids_dtype, tid);
        const bool ok = id >= 0 && id < b.slots;
        s_ids[tid] = ok ? static_cast<int>(id) : -1;
        s_w[tid] = ok ? load_any(a.weights, a.weights_dtype, tid) : 0.0f;
        if (!ok && blockIdx.x == 0) atomicAdd(status, 1);
    }
    __syncthreads();
    const int expert = s_ids[slot_j] >= 0 ? s_ids[slot_j] : 0;  // a dropped route streams slot 0 and weighs zero

    if (warp == kIlWarps) {
        // Producer: the 12 gate/up stages (stage s = tile tile0 + s: 16 gate
        // and 16 up rows, this CTA's quarter of K) and the down rows.
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            for (int st = 0; st < kIlTiles; ++st) {
                mbar_arrive_expect_tx(full0 + 8 * st, static_cast<uint32_t>(kIlStage));
                tma_load_5d(base_u32 + kOffStages + st * kIlStage, &a.w13_map, 0, 2 * r, (tile0 + st) * 16, 0,
                            expert, full0 + 8 * st, pol);
            }
            mbar_arrive_expect_tx(w2_bar, static_cast<uint32_t>(kIlHq * kIlW2Row));
            for (int bx = 0; bx < kIlHq / kIlW2Box; ++bx)
                tma_load_3d(base_u32 + kOffW2 + bx * kIlW2Box * kIlW2Row, &a.w2_map, tile0 * 8,
                            r * kIlHq + bx * kIlW2Box, expert, w2_bar, pol);
        }
        __syncwarp();
    } else {
        // This CTA's quarter of the token row, and the scales and zero points
        // of every weight row and K block it multiplies: for the unit's gate
        // and up rows a row's four scales of this quarter (8 bytes) and a row
        // group's four zero words (16 bytes); for the down rows the scales and
        // zero words of the unit's two intermediate blocks. The strides allow
        // the vector loads (int4_layer_supported). Every load is issued
        // before the first store, so the staging costs one round trip.
        static_assert(kIlHq / 8 <= kIlConsumers, "one x vector per thread");
        uint4 xv = make_uint4(0u, 0u, 0u, 0u);
        if (tid < kIlHq / 8) xv = __ldg(reinterpret_cast<const uint4*>(a.x + r * kIlHq) + tid);
        const int bhi = min(blk0 + 1, kIlI / 128 - 1);
        constexpr int kS13 = (kIlRows13 + kIlConsumers - 1) / kIlConsumers;  // gate/up scale rows per thread
        constexpr int kS2 = kIlHq * 2 / kIlConsumers;                         // down scales per thread
        static_assert(kIlHq * 2 % kIlConsumers == 0 && (kIlHq / 8) * 2 <= kIlConsumers &&
                          kIlRows13 / 8 <= kIlConsumers, "staging items per thread");
        const uint16_t* s13g = static_cast<const uint16_t*>(b.w13_scale) + expert * b.w13_scale_slot_stride;
        const uint16_t* s2g = static_cast<const uint16_t*>(b.w2_scale) + expert * b.w2_scale_slot_stride;
        uint2 v13[kS13];
        uint16_t v2[kS2];
        uint4 z13 = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
        uint32_t z2 = 0x88888888u;
#pragma unroll
        for (int k = 0; k < kS13; ++k) {
            const int i = tid + kIlConsumers * k;
            if (i < kIlRows13) {
                const int row = (i / (kIlRows13 / 2)) * kIlI + tile0 * 16 + i % (kIlRows13 / 2);
                v13[k] = __ldg(reinterpret_cast<const uint2*>(s13g + static_cast<int64_t>(row) * b.w13_scale_row_stride +
                                                              r * kIlKbq));
            }
        }
#pragma unroll
        for (int k = 0; k < kS2; ++k) {
            const int i = tid + kIlConsumers * k;
            v2[k] = __ldg(s2g + static_cast<int64_t>(r * kIlHq + (i >> 1)) * b.w2_scale_row_stride +
                          ((i & 1) ? bhi : blk0));
        }
        if (b.w13_zeros && tid < kIlRows13 / 8) {
            const int rg = ((tid / (kIlRows13 / 16)) * kIlI + tile0 * 16) / 8 + tid % (kIlRows13 / 16);
            z13 = __ldg(reinterpret_cast<const uint4*>(b.w13_zeros + expert * b.w13_zeros_slot_stride +
                                                       static_cast<int64_t>(rg) * b.w13_zeros_row_stride + r * kIlKbq));
        }
        if (b.w2_zeros && tid < (kIlHq / 8) * 2)
            z2 = static_cast<uint32_t>(__ldg(b.w2_zeros + expert * b.w2_zeros_slot_stride +
                                             static_cast<int64_t>((r * kIlHq) / 8 + (tid >> 1)) * b.w2_zeros_row_stride +
                                             ((tid & 1) ? bhi : blk0)));
#pragma unroll
        for (int k = 0; k < kS13; ++k)
            if (tid + kIlConsumers * k < kIlRows13) reinterpret_cast<uint2*>(s_s13)[tid + kIlConsumers * k] = v13[k];
#pragma unroll
        for (int k = 0; k < kS2; ++k) s_s2[tid + kIlConsumers * k] = v2[k];
        if (tid < kIlRows13 / 8) reinterpret_cast<uint4*>(s_z13)[tid] = z13;
        if (tid < (kIlHq / 8) * 2) s_z2[tid] = z2;
        if (tid < kIlHq / 8) {
            // x in the MMA's pair order: (x0, x4), (x1, x5), (x2, x6), (x3, x7)
            reinterpret_cast<uint4*>(s_x)[tid] =
                make_uint4(__byte_perm(xv.x, xv.z, 0x5410u), __byte_perm(xv.x, xv.z, 0x7632u),
                           __byte_perm(xv.y, xv.w, 0x5410u), __byte_perm(xv.y, xv.w, 0x7632u));
        }
        named_barrier(1, kIlConsumers);

        // Gate/up cells: cell c = warp + 16i is K block c % 4 of stage c / 4
        // (four warps per SMSP hide the dequantisation's dependent latency).
#pragma unroll 1
        for (int i = 0; i < kIlCells / kIlWarps; ++i) {
            const int c = warp + kIlWarps * i, st = c >> 2, kb = c & 3;
            uint32_t zb[4], sc[4];
            float sf[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // gate rows g, g + 8 and up rows g, g + 8 of the stage's tile
                const int row = (q >> 1) * (kIlRows13 / 2) + st * 16 + g + 8 * (q & 1);
                il_params<BF16>(s_s13[row * kIlKbq + kb], s_z13[(row >> 3) * kIlKbq + kb], row, zb[q], sc[q], sf[q]);
            }
            uint32_t X[16];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const uint4 xv = g == 0 ? lds128(s_x + kb * 128 + 32 * t + 8 * v) : make_uint4(0u, 0u, 0u, 0u);
                X[4 * v] = xv.x;
                X[4 * v + 1] = xv.y;
                X[4 * v + 2] = xv.z;
                X[4 * v + 3] = xv.w;
            }
            mbar_wait(full0 + 8 * st, 0, status + 1);
            // lines of the stage: (gate|up, row, 128-byte chunk); lane t's 16
            // bytes of block kb are unit (kb & 1) * 4 + t of chunk kb >> 1
            const uint8_t* stage = base + kOffStages + st * kIlStage;
            const int unit16 = (kb & 1) * 4 + t, chunk = kb >> 1;
            const uint4 qg0 = i4_stage_read(stage, (g)*2 + chunk, unit16);
            const uint4 qg1 = i4_stage_read(stage, (g + 8) * 2 + chunk, unit16);
            const uint4 qu0 = i4_stage_read(stage, (16 + g) * 2 + chunk, unit16);
            const uint4 qu1 = i4_stage_read(stage, (24 + g) * 2 + chunk, unit16);
            float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
            il_block_mma<BF16>(qg0, qg1, zb[0], sc[0], sf[0], zb[1], sc[1], sf[1], X, ag);
            il_block_mma<BF16>(qu0, qu1, zb[2], sc[2], sf[2], zb[3], sc[3], sf[3], X, au);
            if (t == 0) {
                float* dst = s_cell + c * 32;  // c = st * 4 + kb
                dst[g] = ag[0];
                dst[g + 8] = ag[2];
                dst[16 + g] = au[0];
                dst[24 + g] = au[2];
            }
        }
        named_barrier(1, kIlConsumers);
        // This CTA's quarter of every gate/up row sum (K blocks in order),
        // into slot r of every cluster CTA's exchange area.
        cluster.barrier_wait();  // every CTA of the cluster is running
        for (int idx = tid; idx < kIlTiles * 32; idx += kIlConsumers) {
            const int st = idx >> 5, row = idx & 31;
            float v = 0.0f;
#pragma unroll
            for (int kb = 0; kb < kIlKbq; ++kb) v += s_cell[(st * kIlKbq + kb) * 32 + row];
            float* dst = s_xch + (r * kIlTiles + st) * 32 + row;
#pragma unroll
            for (int d = 0; d < kIlCluster; ++d) *cluster.map_shared_rank(dst, d) = v;
        }
    }
    if (warp == kIlWarps) cluster.barrier_wait();
    cluster.sync();  // every quarter of every row sum is in every CTA

    if (warp < kIlWarps) {
        // SiLU(gate) * up of the unit's tiles, quarters summed in rank order,
        // with the reference's bf16 rounding points.
        {
            const int st = tid >> 4, j = tid & 15;
            if (st < kIlTiles) {
                float gsum = 0.0f, usum = 0.0f;
#pragma unroll
                for (int d = 0; d < kIlCluster; ++d) {
                    gsum += s_xch[(d * kIlTiles + st) * 32 + j];
                    usum += s_xch[(d * kIlTiles + st) * 32 + 16 + j];
                }
                const float gate = bf16_round_i4(gsum);
                const float up = bf16_round_i4(usum);
                const float act = bf16_round_i4(gate / (1.0f + expf(-gate)));
                const __nv_bfloat16 hv = __float2bfloat16_rn(act * up);
                // h in the down MMA's pair order: 64-column chunk, lane, word,
                // pair, half
                const int lc = st * 16 + j;
                s_h[(((lc >> 6) * 4 + ((lc >> 4) & 3)) * 2 + ((lc >> 3) & 1)) * 8 + (lc & 3) * 2 + ((lc >> 2) & 1)] = hv;
            }
        }
        mbar_wait(w2_bar, 0, status + 1);
        named_barrier(1, kIlConsumers);  // h and the down rows in shared memory
        // Partial down projection: warp w takes 16-row tiles w + 16u of the
        // quarter. In each 64-column chunk of the unit's columns lane (g, t)
        // dequantises two words (columns 16t..16t+15) of rows g and g + 8 and
        // reads h in the same pair order. The scale is applied per weight, so
        // the chunks accumulate in one MMA chain per row tile; a chunk never
        // straddles a 128-column block (units start on 64-column boundaries).
        constexpr int kU = kIlRowTiles / kIlWarps;
        constexpr int kChunks = kIlTiles * 16 / 64;
        static_assert(kIlTiles * 16 % 64 == 0, "64-column chunks");
        const uint8_t* w2s = base + kOffW2;
        float d[kU][4];
#pragma unroll
        for (int u = 0; u < kU; ++u) d[u][0] = d[u][1] = d[u][2] = d[u][3] = 0.0f;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
            const int bi = 4 * c < cb ? 0 : 1;  // chunk c starts at tile 4c
            const uint4 hb0 = lds128(s_h + (c * 4 + t) * 16);
            const uint4 hb1 = lds128(s_h + (c * 4 + t) * 16 + 8);
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int row = (warp + kIlWarps * u) * 16 + g;
                const uint2 w0 = lds64(w2s + row * kIlW2Row + c * 32 + 8 * t);
                const uint2 w1 = lds64(w2s + (row + 8) * kIlW2Row + c * 32 + 8 * t);
                uint32_t z0, s0, z1, s1;
                float f0, f1;
                il_params<BF16>(s_s2[row * 2 + bi], s_z2[(row >> 3) * 2 + bi], row, z0, s0, f0);
                il_params<BF16>(s_s2[(row + 8) * 2 + bi], s_z2[((row + 8) >> 3) * 2 + bi], row + 8, z1, s1, f1);
                const uint32_t A0[4] = {int4_pair<BF16>(w0.x, 0, z0, s0, f0), int4_pair<BF16>(w1.x, 0, z1, s1, f1),
                                        int4_pair<BF16>(w0.x, 1, z0, s0, f0), int4_pair<BF16>(w1.x, 1, z1, s1, f1)};
                mma_bf16_16816(d[u], A0, hb0.x, hb0.y);
                const uint32_t A1[4] = {int4_pair<BF16>(w0.x, 2, z0, s0, f0), int4_pair<BF16>(w1.x, 2, z1, s1, f1),
                                        int4_pair<BF16>(w0.x, 3, z0, s0, f0), int4_pair<BF16>(w1.x, 3, z1, s1, f1)};
                mma_bf16_16816(d[u], A1, hb0.z, hb0.w);
                const uint32_t A2[4] = {int4_pair<BF16>(w0.y, 0, z0, s0, f0), int4_pair<BF16>(w1.y, 0, z1, s1, f1),
                                        int4_pair<BF16>(w0.y, 1, z0, s0, f0), int4_pair<BF16>(w1.y, 1, z1, s1, f1)};
                mma_bf16_16816(d[u], A2, hb1.x, hb1.y);
                const uint32_t A3[4] = {int4_pair<BF16>(w0.y, 2, z0, s0, f0), int4_pair<BF16>(w1.y, 2, z1, s1, f1),
                                        int4_pair<BF16>(w0.y, 3, z0, s0, f0), int4_pair<BF16>(w1.y, 3, z1, s1, f1)};
                mma_bf16_16816(d[u], A3, hb1.z, hb1.w);
            }
        }
        float* pr = a.part + static_cast<int64_t>(unit) * kIlH + r * kIlHq;
        if (t == 0) {
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int nt = warp + kIlWarps * u;
                __stcg(pr + nt * 16 + g, d[u][0]);
                __stcg(pr + nt * 16 + g + 8, d[u][2]);
            }
        }
        // Ticket: the CTA barrier orders every thread's partial stores before
        // thread 0's release; its acquire orders the last arriver's reads.
        named_barrier(1, kIlConsumers);
        if (tid == 0) s_last = atomic_add_acq_rel_gpu(a.tickets + r, 1) == kIlUnits - 1;
        named_barrier(1, kIlConsumers);
        if (s_last) {
            // Last CTA of quarter r: column tid of every unit's partial
            // (unit u = j P + p), all loads in flight before
            // the first store; then for each column each slot's parts in part
            // order, rounded, weighted, slots added in slot order.
            static_assert(kIlHq == kIlConsumers, "one column per consumer thread");
            if (tid == 0) a.tickets[r] = 0;
            const int n = r * kIlHq + tid;
            float v[kIlUnits];
#pragma unroll
            for (int u = 0; u < kIlUnits; ++u) v[u] = __ldcg(a.part + static_cast<int64_t>(u) * kIlH + n);
            float y0 = 0.0f;
#pragma unroll
            for (int j = 0; j < kIlK; ++j) {
                float s0 = 0.0f;
#pragma unroll
                for (int p = 0; p < kIlParts; ++p) s0 += v[j * kIlParts + p];
                const bool routed = s_ids[j] >= 0;
                const float pw0 = routed ? __fmul_rn(bf16_round_i4(s0), s_w[j]) : 0.0f;
                if (a.pair_out) a.pair_out[static_cast<int64_t>(j) * kIlH + n] = pw0;
                y0 = __fadd_rn(y0, pw0);
            }
            store_any(a.out, a.out_dtype, n, y0);
        }
    }
}

}  // namespace

namespace {

using Int4LayerKernel = void (*)(Int4LayerArgs);

// Clusters of the kernel that fit the device at once (cached per device), or
// -1 when the kernel cannot be configured.
int int4_layer_clusters() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (cached[dev]) return cached[dev];
    const Int4LayerKernel kernels[2] = {int4_layer_kernel<true>, int4_layer_kernel<false>};
    for (Int4LayerKernel k : kernels) {
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kIlSmem)) !=
            cudaSuccess) {
            cudaGetLastError();
            return cached[dev] = -1;
        }
    }
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(kIlCluster * ((sms + kIlCluster - 1) / kIlCluster));
    q.blockDim = dim3(kIlThreads);
    q.dynamicSmemBytes = kIlSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kIlCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    q.attrs = attr;
    q.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, int4_layer_kernel<true>, &q) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        return cached[dev] = -1;
    }
    return cached[dev] = clusters;
}

}  // namespace

bool int4_layer_supported(int64_t tokens, int top_k, const DramaB200Int4Bank& b, int x_dtype) {
    if (tokens != 1 || top_k != kIlK || x_dtype != DRAMA_B200_BF16 || b.hidden != kIlH || b.intermediate != kIlI)
        return false;
    if (b.scale_dtype != DRAMA_B200_BF16 && b.scale_dtype != DRAMA_B200_F16) return false;
    // the tensor maps: 16-byte row and slot strides; the vector loads of four
    // gate/up scales (8 bytes) and four zero words (16 bytes)
    if ((b.w13_row_stride * 4) % 16 || (b.w2_row_stride * 4) % 16 || (b.w13_slot_stride * 4) % 16 ||
        (b.w2_slot_stride * 4) % 16)
        return false;
    if (reinterpret_cast<uintptr_t>(b.w13_scale) % 8 || b.w13_scale_row_stride % 4 || b.w13_scale_slot_stride % 4)
        return false;
    if (b.w13_zeros && (reinterpret_cast<uintptr_t>(b.w13_zeros) % 16 || b.w13_zeros_row_stride % 4 ||
                        b.w13_zeros_slot_stride % 4))
        return false;
    return tensor_map_encoder() != nullptr && int4_layer_clusters() >= kIlUnits;
}

cudaError_t int4_layer_launch(const DramaB200Int4Bank& b, const void* x, const void* ids, int ids_dtype,
                              const void* weights, int weights_dtype, void* out, int out_dtype, float* pair_out,
                              float* part, int32_t* tickets, int32_t* status, cudaStream_t s) {
    const TensorMapEncode encode = tensor_map_encoder();
    if (!encode || int4_layer_clusters() < kIlUnits) return cudaErrorInvalidConfiguration;
    Int4LayerArgs a{};
    a.bank = b;
    a.x = static_cast<const __nv_bfloat16*>(x);
    a.ids = ids;
    a.ids_dtype = ids_dtype;
    a.weights = weights;
    a.weights_dtype = weights_dtype;
    a.out = out;
    a.out_dtype = out_dtype;
    a.pair_out = pair_out;
    a.part = part;
    a.tickets = tickets;
    a.status = status;
    // W13 [slot][gate|up][row][H/2 bytes] viewed as [slot][2][I][H/256][128]
    // bytes; one box = 16 rows of gate and up, this CTA's H/8 bytes of each.
    const uint64_t row13 = static_cast<uint64_t>(b.w13_row_stride) * 4, slot13 = static_cast<uint64_t>(b.w13_slot_stride) * 4;
    const cuuint64_t dims[5] = {128, static_cast<cuuint64_t>(kIlH / 256), static_cast<cuuint64_t>(kIlI), 2,
                                static_cast<cuuint64_t>(b.slots)};
    const cuuint64_t strides[4] = {128, row13, row13 * kIlI, slot13};
    const cuuint32_t box[5] = {128, static_cast<cuuint32_t>(kIlH / kIlCluster / 256), 16, 2, 1};
    const cuuint32_t unit_strides[5] = {1, 1, 1, 1, 1};
    if (encode(&a.w13_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<int32_t*>(b.w13), dims, strides, box,
               unit_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    // W2 [slot][row][I/2 bytes]; one box = the unit's 96 bytes x 256 rows.
    const cuuint64_t dims2[3] = {static_cast<cuuint64_t>(kIlI / 2), static_cast<cuuint64_t>(kIlH),
                                 static_cast<cuuint64_t>(b.slots)};
    const cuuint64_t strides2[2] = {static_cast<cuuint64_t>(b.w2_row_stride) * 4,
                                    static_cast<cuuint64_t>(b.w2_slot_stride) * 4};
    const cuuint32_t box2[3] = {static_cast<cuuint32_t>(kIlW2Row), static_cast<cuuint32_t>(kIlW2Box), 1};
    if (encode(&a.w2_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int32_t*>(b.w2), dims2, strides2, box2,
               unit_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = kIlCluster;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kIlCluster * kIlUnits);
    cfg.blockDim = dim3(kIlThreads);
    cfg.dynamicSmemBytes = kIlSmem;
    cfg.stream = s;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, b.scale_dtype == DRAMA_B200_BF16 ? int4_layer_kernel<true> : int4_layer_kernel<false>,
                              a);
}

}  // namespace drama
