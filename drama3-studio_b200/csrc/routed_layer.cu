// One decode MoE layer for a single hidden row in two launches, with no
// cross-CTA atomics and no grid-wide waits.
//
// The arithmetic is drama_b200_fp8_moe_layer's (RMSNorm and router GEMV in the
// fixed fp32 orders shared with the oracle, torch-order softmax / top-k, the
// K1 GEMV fragments, slot-ordered combine, bf16 residual); the schedule is
// built for one token, where a layer is ~38 MB of weights and every extra
// launch or global round trip is a visible fraction of it:
//
//   routed_up_kernel (thread-block clusters of kRuCluster CTAs)
//     before waiting for the previous layer, each CTA pulls gamma and its
//     router rows on chip; then every CTA normalises the row into shared
//     memory, the CTAs of a cluster split the router GEMV (CTA rank r computes
//     experts e = r mod cluster size) and store each logit into every CTA of
//     the cluster (distributed shared memory, hardware cluster barrier), and
//     every CTA routes the row itself (same logits, same result; top-k by a
//     CTA-wide rank pass). CTA c streams whole gate/up tiles c, c + grid, ...
//     of the routed experts through per-warp cp.async rings; a tile split
//     between warps is reduced in shared memory in warp (= K) order, and its
//     SiLU(gate) * up row goes to the workspace. Each CTA also pulls its share
//     of the routed experts' down-projection rows into L2.
//   routed_down_kernel (programmatic dependent launch)
//     CTA c owns hidden rows [16c, 16c + 16): two warps per route slot compute
//     those rows of the slot's down projection over the two halves of the K
//     range; the halves are added in order, the slots summed in slot order,
//     rounded, and added to the residual.
#include <cooperative_groups.h>

#include "common.cuh"
#include "decode_tiles.cuh"
#include "kernels.h"
#include "route.cuh"

namespace drama {

namespace {

namespace cg = cooperative_groups;

constexpr int kRuCluster = 4;                 // smallest cluster sharing one router GEMV
constexpr int kRuWarps = 8;
constexpr int kRuDepth = 5;                   // 8 warps x 5 stages x 4 KB = 160 KB of rings
constexpr int kRuThreads = kRuWarps * 32;
constexpr int kRuRingBytes = kRuWarps * kRuDepth * 8 * 512;
constexpr int kRuPartBytes = kRuWarps * 2 * 32 * 8 * 4;  // two split-tile partials per warp
constexpr int kRdWarps = 16;                  // two warps (K halves) per route slot
constexpr int kRdBlocks = 3;                  // K blocks staged per warp and pass: 16 x 3 x 4 KB = 192 KB
constexpr int kRdThreads = kRdWarps * 32;
constexpr int kRdSmemBytes = kRdWarps * kRdBlocks * 8 * 512;

__host__ __device__ constexpr size_t ru_smem_bytes(int hidden, int experts) {
    return static_cast<size_t>(kRuRingBytes) + kRuPartBytes + static_cast<size_t>(hidden) * 6 +
           static_cast<size_t>((experts + 3) / 4) * 16;
}

// The K1 helpers read the bank and the intermediate size from a DecodeArgs.
__device__ __forceinline__ DecodeArgs bank_args(const RoutedLayerArgs& a) {
    DecodeArgs la{};
    la.format = 0;
    la.fp8 = a.bank;
    la.hidden = a.H;
    la.intermediate = a.I;
    return la;
}

__global__ void __launch_bounds__(kRuThreads, 1) routed_up_kernel(RoutedLayerArgs a) {
    extern __shared__ __align__(16) uint4 smem_ru[];
    uint4* rings = smem_ru;
    float4* s_part = reinterpret_cast<float4*>(reinterpret_cast<char*>(smem_ru) + kRuRingBytes);
    float* s_norm = reinterpret_cast<float*>(reinterpret_cast<char*>(smem_ru) + kRuRingBytes + kRuPartBytes);
    uint4* s_x16 = reinterpret_cast<uint4*>(s_norm + a.H);
    float* s_logit = reinterpret_cast<float*>(s_x16 + a.H / 8);
    __shared__ float s_red[kRuWarps];
    __shared__ float s_xscale;
    __shared__ int s_ids[32], s_order[32];
    __shared__ float s_key[32];
    __shared__ int s_idx[32];
    __shared__ int s_cnt[33];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int H = a.H, I = a.I, E = a.E, k = a.k;
    const int KB = H / 128, TILES = I / 16;
    const DecodeWorkspace& ws = a.ws;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int csize = static_cast<int>(cluster.num_blocks());

    // Everything that does not depend on the previous layer is fetched before
    // waiting for it: gamma into registers, and this warp's router rows into
    // the (still idle) ring memory, row r of the warp at slot r * warps + warp.
    cluster.barrier_arrive();  // paired with barrier_wait before the first remote store
    const int per = H / 256;
    const int chunks = H / 256;
    float gam[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
        if (j < per) gam[j] = __ldg(a.gamma + tid * per + j);
    const int staged_rows = kRuRingBytes / (H * 2);
    {
        const uint32_t stage_base = smem_u32(rings);
        const uint64_t keep = policy_evict_last();  // rows re-read by every cluster
        int r = 0;
        for (int e = rank + csize * warp; e < E; e += csize * kRuWarps, ++r) {
            const int slot = r * kRuWarps + warp;
            if (slot >= staged_rows) break;
            const __nv_bfloat16* grow = a.gate + static_cast<int64_t>(e) * H;
            for (int i = 0; i < chunks; ++i)
                cp16(stage_base + slot * H * 2 + 512 * i + 16 * lane, grow + 256 * i + 8 * lane, keep);
        }
        cp_commit();
    }
    grid_launch_dependents();
    grid_dependency_wait();

    // RMSNorm: thread tid owns the H/256 consecutive elements from tid * H/256.
    {
        float v[16];
        if ((per & 7) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 8) {
                if (j < per) {
                    const uint4 q = __ldcg(reinterpret_cast<const uint4*>(a.hidden_in + tid * per + j));
                    const uint32_t wv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        v[j + 2 * u] = __uint_as_float(wv[u] << 16);
                        v[j + 2 * u + 1] = __uint_as_float(wv[u] & 0xffff0000u);
                    }
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < per) v[j] = __bfloat162float(__ldcg(a.hidden_in + tid * per + j));
        }
        float sq = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (j < per) sq = __fadd_rn(sq, __fmul_rn(v[j], v[j]));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, off));
        if (lane == 0) s_red[warp] = sq;
        __syncthreads();
        float total = 0.0f;
#pragma unroll
        for (int w8 = 0; w8 < kRuWarps; ++w8) total = __fadd_rn(total, s_red[w8]);
        const float mean = __fmul_rn(total, 1.0f / static_cast<float>(H));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (j < per) {
                const int i = tid * per + j;
                const __nv_bfloat16 y = __float2bfloat16_rn(__fmul_rn(__fmul_rn(v[j], inv), gam[j]));
                s_norm[i] = __bfloat162float(y);
                if (blockIdx.x == 0 && a.normed_out) a.normed_out[i] = y;
            }
        }
    }
    __syncthreads();
    // Router GEMV share of this cluster rank: experts e = rank (mod cluster
    // size), one warp per expert; lane l owns elements 256i + 8l + j, products
    // added in (i, j) order with separate multiply and add, lanes combined by
    // xor butterfly, logits rounded to bf16. Each logit is stored into every
    // CTA of the cluster.
    cp_wait<0>();
    cluster.barrier_wait();  // every CTA of the cluster is running
    {
        int r = 0;
        for (int e = rank + csize * warp; e < E; e += csize * kRuWarps, ++r) {
            const int slot = r * kRuWarps + warp;
            const __nv_bfloat16* grow = a.gate + static_cast<int64_t>(e) * H;
            const char* srow = reinterpret_cast<const char*>(rings) + static_cast<int64_t>(slot) * H * 2;
            uint4 gq[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < chunks)
                    gq[i] = slot < staged_rows ? *reinterpret_cast<const uint4*>(srow + 512 * i + 16 * lane)
                                               : __ldg(reinterpret_cast<const uint4*>(grow + 256 * i + 8 * lane));
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i < chunks) {
                    const __nv_bfloat16* gv = reinterpret_cast<const __nv_bfloat16*>(&gq[i]);
                    const float4 x0 = reinterpret_cast<const float4*>(s_norm + 256 * i + 8 * lane)[0];
                    const float4 x1 = reinterpret_cast<const float4*>(s_norm + 256 * i + 8 * lane)[1];
                    const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn(xv[j], __bfloat162float(gv[j])));
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
            const float logit = __bfloat162float(__float2bfloat16_rn(acc));
            if (lane < csize) *cluster.map_shared_rank(s_logit + e, lane) = logit;
        }
    }
    __syncwarp();
    cluster.sync();  // every logit of the row is in every CTA's shared memory; no remote access after this
    // Routing, redundantly in every CTA: softmax by warp 0 (in place), top-k
    // by rank over the CTA, sort and renormalisation by warp 0.
    if (warp == 0) {
        dispatch_experts(E, [&]<int LANES, int ITERS>() {
            route_softmax<LANES, ITERS>([&](int i) { return s_logit[i]; }, E, lane, s_logit);
        });
    }
    __syncthreads();
    route_select_cta(s_logit, E, k, s_key, s_idx, s_cnt);
    if (warp == 0) {
        int idx = 0;
        float wr = 0.0f;
        route_finish(k, true, lane, s_key, s_idx, idx, wr);
        const __nv_bfloat16 wb = __float2bfloat16_rn(wr);
        if (lane < k) {
            s_ids[lane] = idx;
            if (blockIdx.x == 0) {
                ws.order[lane] = idx;
                ws.wts[lane] = __bfloat162float(wb);
                if (a.ids_out) a.ids_out[lane] = idx;
                if (a.weights_out) a.weights_out[lane] = wb;
            }
        }
        __syncwarp();
        // route slots in ascending expert order (top-k IDs are distinct)
        if (lane < k) {
            int r = 0;
            for (int q = 0; q < k; ++q) r += s_ids[q] < s_ids[lane];
            s_order[r] = lane;
        }
        __syncwarp();
    }
    __syncthreads();

    // Gate/up stream. CTA tiles: blockIdx.x + i * grid (i < ntiles); their
    // cells (tile, 128-K block) in order are split evenly over the warps.
    const DecodeArgs la = bank_args(a);
    const int all_tiles = k * TILES;
    const int ntiles = static_cast<int>(blockIdx.x) < all_tiles
                           ? (all_tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                           : 0;
    const int ncells = ntiles * KB;
    const int qw = (ncells + kRuWarps - 1) / kRuWarps;
    const int c0 = min(ncells, warp * qw), c1 = min(ncells, c0 + qw);
    const int n = c1 - c0;
    const uint64_t pol = policy_evict_first();
    uint4* ring = rings + warp * kRuDepth * 8 * 32;
    const uint32_t ring_base = smem_u32(ring + lane);
    auto cell_of = [&](int lc) {
        const int tile = static_cast<int>(blockIdx.x) + (lc / KB) * static_cast<int>(gridDim.x);
        return CellIt{tile / TILES, tile % TILES, lc % KB};
    };
    // h rows g and g + 8 of tile `tile_local` from its full gate/up sums
    auto finalize = [&](int tile_local, const float (&acc)[8]) {
        if (t != 0) return;
        const int tile = static_cast<int>(blockIdx.x) + tile_local * static_cast<int>(gridDim.x);
        const int slot = s_order[tile / TILES], jt = tile % TILES;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float gate = __bfloat162float(__float2bfloat16_rn(acc[r * 2] * s_xscale));
            const float up = __bfloat162float(__float2bfloat16_rn(acc[4 + r * 2] * s_xscale));
            const float act = __bfloat162float(__float2bfloat16_rn(gate / (1.0f + expf(-gate))));
            reinterpret_cast<__nv_bfloat16*>(ws.h)[static_cast<int64_t>(slot) * I + jt * 16 + g + 8 * r] =
                __float2bfloat16_rn(act * up);
        }
    };
    const int first_tile = c0 / KB;
    // A tile this warp only partly covers is parked in shared memory (slot 0:
    // the warp's first tile, slot 1: its last); a fully covered one is final.
    auto close_tile = [&](int tile_local, float (&acc)[8]) {
        const bool whole = tile_local * KB >= c0 && (tile_local + 1) * KB <= c1;
        if (whole) {
            finalize(tile_local, acc);
        } else {
            float4* dst = s_part + ((warp * 2 + (tile_local == first_tile ? 0 : 1)) * 32 + lane) * 2;
            dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    };
#pragma unroll
    for (int s = 0; s < kRuDepth; ++s) {
        if (s < n) {
            const CellIt it = cell_of(c0 + s);
            up_issue<0>(ring_base + s * 8 * 512, la, s_ids[s_order[it.grp]], it, g, t, pol);
        }
        cp_commit();
    }
    // This CTA's share of the down-projection rows, into L2 for the next launch
    // (slab (slot, 16-row tile) i by CTA i mod grid), issued behind the stream.
    {
        const DramaB200Fp8Bank& b = a.bank;
        const int tiles = H / 16;
        for (int it = blockIdx.x + gridDim.x * tid; it < k * tiles; it += gridDim.x * kRuThreads) {
            const char* base = static_cast<const char*>(b.w2) + s_ids[it / tiles] * b.w2_slot_stride +
                               static_cast<int64_t>(it % tiles) * 16 * b.w2_row_stride;
            if (b.w2_row_stride == I) {
                prefetch_l2_bulk(base, static_cast<uint32_t>(16 * I));
            } else {
                for (int r = 0; r < 16; ++r) prefetch_l2_bulk(base + r * b.w2_row_stride, static_cast<uint32_t>(I));
            }
        }
    }
    // f16 copy of the normalised row scaled by 2^-e (B operand of the up GEMV),
    // made while the first cells are in flight.
    {
        float m = 0.0f;
        for (int i = tid; i < H; i += kRuThreads) m = fmaxf(m, fabsf(s_norm[i]));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        __syncwarp();
        if (lane == 0) s_red[warp] = m;
        __syncthreads();
        float amax = 0.0f;
#pragma unroll
        for (int w8 = 0; w8 < kRuWarps; ++w8) amax = fmaxf(amax, s_red[w8]);
        const int e = f16_exponent_for(amax);
        const float inv = ldexpf(1.0f, -e);
        if (tid == 0) s_xscale = ldexpf(1.0f, e);
        for (int c = tid; c < H / 8; c += kRuThreads) {
            const float4 p0 = reinterpret_cast<const float4*>(s_norm)[2 * c];
            const float4 p1 = reinterpret_cast<const float4*>(s_norm)[2 * c + 1];
            const float vv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
            s_x16[c] = pack8<0>(vv, inv);
        }
    }
    __syncthreads();
    // Block scales of the warp's cells, 16 cells per register: lane L < 16
    // holds the gate scale of cell 16c + L, lane 16 + L its up scale. Loaded
    // one chunk ahead, so no cell waits on a scale load.
    const DramaB200Fp8Bank& bk = a.bank;
    auto load_scales = [&](int chunk) -> float {
        const int ci = chunk * 16 + (lane & 15);
        if (ci >= n) return 0.0f;
        const CellIt it = cell_of(c0 + ci);
        const int row = (lane < 16 ? 0 : I) + it.jt * 16;
        return __ldg(bk.w13_scale + s_ids[s_order[it.grp]] * bk.w13_scale_slot_stride +
                     (row >> 7) * bk.w13_scale_row_stride + it.kb);
    };
    float sc_cur = load_scales(0), sc_nxt = load_scales(1);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < n; ++i) {
        const int lc = c0 + i;
        if (i > 0 && (i & 15) == 0) {
            sc_cur = sc_nxt;
            sc_nxt = load_scales((i >> 4) + 1);
        }
        cp_wait<kRuDepth - 1>();
        if (i > 0 && lc % KB == 0) close_tile(lc / KB - 1, acc);
        uint4 q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) q[v] = ring[((i % kRuDepth) * 8 + v) * 32 + lane];
        uint32_t xb[16];
        const CellIt it = cell_of(lc);
        if (g == 0) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                // lane t owns k = 16t.. and 64 + 16t.. of the block
                const uint4 x = s_x16[it.kb * 16 + 2 * t + (v & 1) + 8 * (v >> 1)];
                xb[4 * v] = x.x;
                xb[4 * v + 1] = x.y;
                xb[4 * v + 2] = x.z;
                xb[4 * v + 3] = x.w;
            }
        } else {
#pragma unroll
            for (int v = 0; v < 16; ++v) xb[v] = 0u;
        }
        __syncwarp();
        const float sg = __shfl_sync(0xffffffffu, sc_cur, i & 15);
        const float su = __shfl_sync(0xffffffffu, sc_cur, 16 + (i & 15));
        up_mma_fp8_scaled(q, sg, su, xb, acc);
        if (i + kRuDepth < n) {
            const CellIt nx = cell_of(lc + kRuDepth);
            up_issue<0>(ring_base + (i % kRuDepth) * 8 * 512, la, s_ids[s_order[nx.grp]], nx, g, t, pol);
        }
        cp_commit();
    }
    if (n > 0) close_tile((c1 - 1) / KB, acc);
    __syncwarp();
    __syncthreads();
    // Tiles split between warps: summed in warp order by one warp.
    for (int tl = warp; tl < ntiles; tl += kRuWarps) {
        const int w0 = (tl * KB) / qw, w1 = (tl * KB + KB - 1) / qw;
        if (w0 == w1) continue;
        float tot[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int v = w0; v <= w1; ++v) {
            const int slot = tl == (v * qw) / KB ? 0 : 1;
            const float4* src = s_part + ((v * 2 + slot) * 32 + lane) * 2;
            const float4 p0 = src[0], p1 = src[1];
            tot[0] += p0.x;
            tot[1] += p0.y;
            tot[2] += p0.z;
            tot[3] += p0.w;
            tot[4] += p1.x;
            tot[5] += p1.y;
            tot[6] += p1.z;
            tot[7] += p1.w;
        }
        finalize(tl, tot);
    }
}

__global__ void __launch_bounds__(kRdThreads, 1) routed_down_kernel(RoutedLayerArgs a) {
    extern __shared__ __align__(16) uint4 smem_rd[];
    __shared__ float s_half[kRoutedMaxTopK][2][16];
    __shared__ float s_w[kRoutedMaxTopK];
    __shared__ int s_ids[kRoutedMaxTopK];
    grid_launch_dependents();
    grid_dependency_wait();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int H = a.H, I = a.I, k = a.k, KB2 = I / 128, KBH = (KB2 + 1) / 2;
    const DecodeWorkspace& ws = a.ws;
    if (tid < k) {
        s_ids[tid] = __ldcg(ws.order + tid);
        s_w[tid] = __ldcg(ws.wts + tid);
    }
    __syncthreads();
    const DramaB200Fp8Bank& b = a.bank;
    const uint64_t pol = policy_evict_first();
    uint4* region = smem_rd + warp * kRdBlocks * 8 * 32;
    const uint32_t rbase = smem_u32(region + lane);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(ws.h);
    for (int nt = blockIdx.x; nt < H / 16; nt += gridDim.x) {
        // work item = (route slot j, K half): warp w takes items w, w + warps, ...
        for (int item = warp; item < 2 * k; item += kRdWarps) {
            const int j = item >> 1, half = item & 1;
            const int kb_begin = half ? KBH : 0, kb_end = half ? KB2 : KBH;
            const int expert = s_ids[j];
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            // lane (g, t): rows g and g + 8 of the tile, bytes 16t.. and
            // 64 + 16t.. of each 128-wide K block (the decode kernels' map)
            const uint8_t* wbase = static_cast<const uint8_t*>(b.w2) + expert * b.w2_slot_stride +
                                   static_cast<int64_t>(nt * 16 + g) * b.w2_row_stride + 16 * t;
            const int64_t r8 = 8 * b.w2_row_stride;
            const __nv_bfloat16* hrow = h + static_cast<int64_t>(j) * I;
            // lane kb holds the block scale of K block kb (KB2 <= 32)
            const float sreg = lane < KB2 ? __ldg(b.w2_scale + expert * b.w2_scale_slot_stride +
                                                  ((nt * 16) >> 7) * b.w2_scale_row_stride + lane)
                                          : 0.0f;
            for (int kb0 = kb_begin; kb0 < kb_end; kb0 += kRdBlocks) {
                const int nb = min(kRdBlocks, kb_end - kb0);
                for (int u = 0; u < nb; ++u) {
                    const uint32_t d = rbase + u * 8 * 512;
                    const uint8_t* p = wbase + (kb0 + u) * 128;
                    cp16(d + 0 * 512, p, pol);
                    cp16(d + 1 * 512, p + 64, pol);
                    cp16(d + 2 * 512, p + r8, pol);
                    cp16(d + 3 * 512, p + r8 + 64, pol);
                    if (g == 0) {
                        const __nv_bfloat16* hp = hrow + (kb0 + u) * 128;
                        cp16(d + 4 * 512, hp + 16 * t, pol);
                        cp16(d + 5 * 512, hp + 16 * t + 8, pol);
                        cp16(d + 6 * 512, hp + 64 + 16 * t, pol);
                        cp16(d + 7 * 512, hp + 64 + 16 * t + 8, pol);
                    }
                }
                cp_commit();
                cp_wait<0>();
                __syncwarp();
                for (int u = 0; u < nb; ++u) {
                    uint4 q[8];
#pragma unroll
                    for (int v = 0; v < 8; ++v)
                        q[v] = (v < 4 || g == 0) ? region[(u * 8 + v) * 32 + lane] : make_uint4(0u, 0u, 0u, 0u);
                    __syncwarp();
                    uint32_t hb[16];
                    const int e = dn_fragment<0, DRAMA_B200_BF16>(q + 4, hb);
                    float s0, s1;
                    column_scales(e, t, s0, s1);
                    const float sb = __shfl_sync(0xffffffffu, sreg, kb0 + u);
                    dn_mma_fp8_block2(q, sb, s0, s1, hb, acc);
                }
                __syncwarp();
            }
            if (t == 0) {
                s_half[j][half][g] = acc[0];
                s_half[j][half][g + 8] = acc[2];
            }
            __syncwarp();
        }
        __syncthreads();
        if (tid < 16) {
            // per slot: the two K halves in order, rounded, times the route
            // weight; slots summed in slot order
            float y = 0.0f;
            for (int j = 0; j < k; ++j)
                y += __bfloat162float(__float2bfloat16_rn(s_half[j][0][tid] + s_half[j][1][tid])) * s_w[j];
            const __nv_bfloat16 moe = __float2bfloat16_rn(y);
            const int row = nt * 16 + tid;
            if (a.moe_out) a.moe_out[row] = moe;
            a.hidden_out[row] =
                __float2bfloat16_rn(__bfloat162float(__ldcg(a.hidden_in + row)) + __bfloat162float(moe));
        }
        __syncwarp();
        __syncthreads();
    }
}

}  // namespace

bool routed_layer_supported(int64_t tokens, int top_k, int hidden, int intermediate, int experts) {
    return tokens == 1 && top_k >= 1 && top_k <= kRoutedMaxTopK && hidden % 256 == 0 && hidden <= 4096 &&
           intermediate % 128 == 0 && intermediate <= 4096 && experts >= 1 && experts <= 1024;
}

cudaError_t routed_layer_launch(const RoutedLayerArgs& a, int sm_count, cudaStream_t s) {
    constexpr int kSizes[3] = {16, 8, kRuCluster};
    static int ru_grid[64][3] = {};  // per device and cluster size: resident clusters x size (0: not usable)
    static bool ru_ready[64] = {};
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = 1;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    const size_t ru_max = ru_smem_bytes(4096, 1024);
    if (!ru_ready[dev]) {
        err = cudaFuncSetAttribute(routed_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(ru_max));
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(routed_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRdSmemBytes);
        if (err != cudaSuccess) return err;
        if (cudaFuncSetAttribute(routed_up_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
            cudaGetLastError();
        // For each cluster size: as many whole clusters as can be resident at
        // once (no second wave).
        for (int i = 0; i < 3; ++i) {
            const int size = kSizes[i];
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3(size * ((sm_count + size - 1) / size));
            q.blockDim = dim3(kRuThreads);
            q.dynamicSmemBytes = ru_max;
            attrs[0].val.clusterDim.x = size;
            q.attrs = attrs;
            q.numAttrs = 1;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, routed_up_kernel, &q) != cudaSuccess) {
                cudaGetLastError();
                clusters = 0;
            }
            ru_grid[dev][i] = clusters * size;
        }
        if (!ru_grid[dev][2]) return cudaErrorInvalidConfiguration;
        ru_ready[dev] = true;
    }
    // The cluster size with the fewest bytes per CTA before and during the
    // stream: its share of the router rows (E * H * 2 / size) plus its
    // gate/up tiles (ceil(tiles / grid) * 32 rows * H bytes); each SM pulls
    // its bytes at roughly an equal share of HBM bandwidth.
    const int all_tiles = a.k * (a.I / 16);
    int pick = -1;
    double best = 0.0;
    for (int i = 0; i < 3; ++i) {
        const int grid = ru_grid[dev][i];
        if (!grid) continue;
        const double bytes = static_cast<double>(a.E) * a.H * 2 / kSizes[i] +
                             static_cast<double>((all_tiles + grid - 1) / grid) * 32.0 * a.H;
        if (pick < 0 || bytes < best) {
            pick = i;
            best = bytes;
        }
    }
    attrs[0].val.clusterDim.x = kSizes[pick];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ru_grid[dev][pick]);
    cfg.blockDim = dim3(kRuThreads);
    cfg.dynamicSmemBytes = ru_smem_bytes(a.H, a.E);
    cfg.stream = s;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    err = cudaLaunchKernelEx(&cfg, routed_up_kernel, a);
    if (err != cudaSuccess) return err;
    const int tiles = a.H / 16;
    return launch_pdl(routed_down_kernel, dim3(tiles < sm_count ? tiles : sm_count), dim3(kRdThreads),
                      static_cast<size_t>(kRdSmemBytes), s, a);
}

}  // namespace drama
