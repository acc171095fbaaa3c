// One decode MoE layer for a single hidden row in ONE launch.
//
// The arithmetic is drama_b200_fp8_moe_layer's: RMSNorm and the router GEMV
// in the fixed fp32 orders shared with the oracle (or the caller's normalised
// row and bf16 logits), torch-order softmax / top-k / renormalisation, the K1
// FP8 fragments (exact E4M3 -> f16, block scales on fp32 block sums), gate/up
// rounded to bf16, SiLU(gate) * up in bf16, each expert's down projection
// rounded to bf16, times its route weight, summed over route slots in slot
// order, and the bf16 residual add.
//
// Schedule. The grid is one wave of 4-CTA thread-block clusters. Cluster u
// owns unit u = (route slot j, part p): a contiguous run of 16-wide tiles of
// the intermediate dimension of expert ids[j]. Its four CTAs split the hidden
// dimension H into quarters, so CTA r of the cluster
//   1. streams the unit's (gate tile, up tile) row pairs, bytes
//      [r H/4, (r+1) H/4) of each, into a ring of shared-memory stages: one
//      tiled TMA load per stage (a 5-D view of the bank, 128-byte swizzle, no
//      multicast) issued by a producer warp, mbarrier full/empty pairs; the
//      consumer warps multiply each 128-wide K block with the matching part
//      of the normalised row on mma.sync fragments;
//   2. adds its K-block partials per row and stores them into every CTA of
//      the cluster (distributed shared memory); after the cluster barrier each
//      CTA sums the four quarters in rank order and forms the unit's
//      SiLU(gate) * up values;
//   3. multiplies rows [r H/4, (r+1) H/4) of the down projection, restricted
//      to the unit's intermediate columns (loaded with cp.async while steps 1
//      and 2 run), with those values: a partial down projection;
//   4. stores the fp32 partial and takes an arrival ticket (one acquire-
//      release atomic per CTA); the last CTA of quarter r to arrive (no
//      waiting) copies every unit's partial of the quarter into shared memory
//      and sums, for every row, each slot's parts in part order, rounds,
//      weights, adds the slots in slot order and the residual, and resets the
//      ticket.
// Every expert weight byte is read once, by ~128 SMs at once, and the layer
// needs no second launch. Before waiting for the previous layer
// (programmatic dependent launch) each CTA pulls its share of the router rows
// into the still idle ring; RMSNorm, the router GEMV (split over the cluster,
// logits exchanged through distributed shared memory) and routing follow.
#include <cooperative_groups.h>

#include "common.cuh"
#include "decode_tiles.cuh"
#include "kernels.h"
#include "route.cuh"
#include "tma.cuh"

namespace drama {

namespace {

namespace cg = cooperative_groups;

constexpr int kDlCluster = 4;
constexpr int kDlWarps = 8;                      // consumer warps (RMSNorm / router: 256 threads)
constexpr int kDlThreads = (kDlWarps + 1) * 32;  // + one TMA producer warp
constexpr int kDlConsumers = kDlWarps * 32;
constexpr int kDlMaxTiles = 16;                  // intermediate tiles per unit
constexpr int kDlMaxSmem = 230400;               // dynamic shared memory per CTA (opt-in 232448 less static)
constexpr int kDlMaxHidden = 2048;

// Dynamic shared memory of one CTA, from a 1024-byte aligned base (the
// 128-byte swizzle of the TMA stages repeats every 1024 bytes). The ring and
// the down-projection buffer are one region; it holds the staged router rows
// until routing is done, and the partial rows for the combine at the end.
// With `overlay` every gate/up stage of the unit has its own slot (no ring
// reuse) and the down rows land over the first stages once they are consumed.
struct DlLayout {
    int hq, kbq, stage, stages, nkt, w2_cols, w2_rows, w2_boxes, w2_stages, overlay;
    uint32_t region, w2, hin, norm, x16, logit, cell, xch, h16, s2, full, empty, w2_bar, total;
};

__host__ __device__ inline DlLayout dl_layout(int H, int E, int nkt, int stages, int overlay) {
    DlLayout L{};
    L.hq = H / kDlCluster;
    L.kbq = L.hq / 128;
    L.stage = 32 * L.hq;  // 16 gate rows + 16 up rows, a multiple of 1024 bytes
    L.stages = stages;
    L.nkt = nkt;
    // down rows: boxes of 4 intermediate tiles (64 bytes) x up to 256 rows,
    // 64-byte swizzle; column boxes outer, row boxes inner
    L.w2_cols = (nkt + 3) / 4;
    L.w2_rows = L.hq < 256 ? L.hq : 256;
    L.w2_boxes = L.w2_cols * (L.hq / L.w2_rows);
    uint32_t off = 0;
    auto take = [&](uint32_t bytes) {
        const uint32_t p = off;
        off += (bytes + 127u) & ~127u;
        return p;
    };
    const uint32_t ring_bytes = static_cast<uint32_t>(stages) * L.stage;
    const uint32_t w2_bytes = static_cast<uint32_t>(L.w2_boxes) * L.w2_rows * 64;
    L.overlay = overlay;
    L.w2_stages = static_cast<int>((w2_bytes + L.stage - 1) / L.stage);
    L.region = overlay ? (ring_bytes > w2_bytes ? ring_bytes : w2_bytes) : ring_bytes + w2_bytes;
    take(L.region);
    L.w2 = overlay ? 0 : ring_bytes;
    L.hin = take(H * 2);
    L.norm = take(H * 2);
    L.x16 = take(L.hq * 2);
    L.logit = take((((E + 3) & ~3) + 4) * 4);
    L.cell = take(nkt * L.kbq * 32 * 4);
    L.xch = take(kDlCluster * nkt * 32 * 4);
    L.h16 = take(nkt * 16 * 2);
    L.s2 = take(4 * (L.hq / 128) * 4);
    L.full = take(stages * 8);
    L.empty = take(stages * 8);
    L.w2_bar = take(8);
    L.total = off + 1024;  // room to align the base
    return L;
}

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// The last arriver's sums for two adjacent rows (column pair c2 of the
// quarter): each slot's PP parts in part order (unit j PP + p at row
// (j PP + p) hq2 of `sp`, float2 columns), rounded to bf16, times the route
// weight, added in slot order. PP is a template argument so that a slot's
// loads issue together and the slot loop unrolls (runtime part counts make
// the loop several times slower); PP = 0 is the generic loop.
template <int PP>
__device__ __forceinline__ void dl_slot_sums(const float2* sp, int c2, int hq2, int k, int parts, const float* s_w,
                                             float& y0, float& y1) {
    if constexpr (PP > 0) {
#pragma unroll 4
        for (int j = 0; j < k; ++j) {
            float2 v[PP];
#pragma unroll
            for (int p = 0; p < PP; ++p) v[p] = sp[(j * PP + p) * hq2 + c2];
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int p = 0; p < PP; ++p) {
                s0 += v[p].x;
                s1 += v[p].y;
            }
            const float wj = s_w[j];
            y0 = __fadd_rn(y0, __fmul_rn(bf16_round(s0), wj));
            y1 = __fadd_rn(y1, __fmul_rn(bf16_round(s1), wj));
        }
    } else {
        for (int j = 0; j < k; ++j) {
            float s0 = 0.0f, s1 = 0.0f;
            for (int p = 0; p < parts; ++p) {
                const float2 v = sp[(j * parts + p) * hq2 + c2];
                s0 += v.x;
                s1 += v.y;
            }
            const float wj = s_w[j];
            y0 = __fadd_rn(y0, __fmul_rn(bf16_round(s0), wj));
            y1 = __fadd_rn(y1, __fmul_rn(bf16_round(s1), wj));
        }
    }
}

// LANES x ITERS lanes and values per lane of the softmax cover the expert
// count; one instantiation per expert-count class keeps a single softmax in
// the kernel's code. The kernel runs once per layer, straight through, so its
// code must fit the SM's instruction cache (about 128 KB on the B200) to stay
// resident from one layer's launch to the next.
//
// HC > 0 fixes the hidden size, NKTC > 0 the tiles of every unit (all stages
// resident), PC > 0 the units per route slot and EC > 0 the expert count:
// the shape-dependent loops
// then have compile-time trip counts and unroll, which makes the serial steps
// (the down projection and the combine above all) several times faster than
// with runtime bounds. The host picks such an instantiation only for a shape
// it was made for (decode_layer_kernel_fixed); the arithmetic and its order
// are the generic kernel's.
template <int LANES, int ITERS, int HC, int NKTC, int PC, int EC>
__global__ void __launch_bounds__(kDlThreads, 1) decode_layer_kernel(const __grid_constant__ DecodeLayerArgs a) {
    extern __shared__ __align__(1024) uint8_t dl_smem_raw[];
    __shared__ float s_red[kDlWarps];
    __shared__ float s_xscale, s_hscale;
    __shared__ int s_ids[32];
    __shared__ float s_w[32];
    __shared__ float s_key[32], s_rkey[32];
    __shared__ int s_idx[32], s_ridx[32];
    __shared__ int s_last;

    const RoutedLayerArgs& A = a.layer;
    const int H = HC > 0 ? HC : A.H, I = A.I, E = EC > 0 ? EC : A.E, k = A.k;
    const DlLayout L = NKTC > 0 ? dl_layout(H, E, NKTC, NKTC, 1) : dl_layout(H, E, a.nkt, a.stages, a.overlay);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    cg::cluster_group cluster = cg::this_cluster();
    const int r = static_cast<int>(cluster.block_rank());
    const int unit = static_cast<int>(blockIdx.x) / kDlCluster;
    const int units = static_cast<int>(gridDim.x) / kDlCluster;
    const int P = PC > 0 ? PC : a.parts, TPI = I / 16;
    const int slot_j = unit / P, part = unit % P;
    const int tile0 = TPI * part / P, nkt = NKTC > 0 ? NKTC : TPI * (part + 1) / P - tile0;
    const int HQ = L.hq, KBQ = L.kbq;
    const bool fused = a.logits_in == nullptr;
    int32_t* status = A.ws.status + 3;

    const uint32_t raw_u32 = smem_u32(dl_smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
    uint8_t* base = dl_smem_raw + (base_u32 - raw_u32);
    __nv_bfloat16* s_hin = reinterpret_cast<__nv_bfloat16*>(base + L.hin);
    __nv_bfloat16* s_norm = reinterpret_cast<__nv_bfloat16*>(base + L.norm);  // the bf16 normalised row
    uint4* s_x16 = reinterpret_cast<uint4*>(base + L.x16);
    float* s_logit = reinterpret_cast<float*>(base + L.logit);
    float* s_cell = reinterpret_cast<float*>(base + L.cell);
    float* s_xch = reinterpret_cast<float*>(base + L.xch);
    __half* s_h16 = reinterpret_cast<__half*>(base + L.h16);
    float* s_s2 = reinterpret_cast<float*>(base + L.s2);
    const uint32_t full0 = base_u32 + L.full, empty0 = base_u32 + L.empty;

    if (tid == 0) {
        for (int s = 0; s < L.stages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, KBQ < kDlWarps ? KBQ : kDlWarps);
        }
        mbar_init(base_u32 + L.w2_bar, 1);
        fence_mbar_init();
    }
    cluster.barrier_arrive();  // paired with barrier_wait before the first remote store

    // Before the previous layer is done: this CTA's router rows (experts
    // e = r mod 4, warp-interleaved: row q of warp w at slot 8q + w) into the
    // idle region, and gamma.
    const int per = H / 256;
    float gam[8];
    if (fused && warp < kDlWarps) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j < per) gam[j] = __ldg(A.gamma + tid * per + j);
        const uint64_t keep = policy_evict_last();
        int q = 0;
        for (int e = r + kDlCluster * warp; e < E; e += kDlCluster * kDlWarps, ++q) {
            const int slot = q * kDlWarps + warp;  // the plan keeps every row of this rank staged
            const __nv_bfloat16* grow = A.gate + static_cast<int64_t>(e) * H;
            for (int i = 0; i < H / 256; ++i)
                cp16(base_u32 + slot * H * 2 + 512 * i + 16 * lane, grow + 256 * i + 8 * lane, keep);
        }
    }
    cp_commit();
    grid_launch_dependents();
    grid_dependency_wait();

    // RMSNorm (threads 0..255, the oracle's order) or the caller's row; the
    // hidden row is kept in shared memory for the residual add.
    if (warp < kDlWarps) {
        if (fused) {
            float v[8];
            if ((per & 7) == 0) {
                const uint4 qv = __ldcg(reinterpret_cast<const uint4*>(A.hidden_in + tid * per));
                reinterpret_cast<uint4*>(s_hin + tid * per)[0] = qv;
                const uint32_t wv[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    v[2 * u] = __uint_as_float(wv[u] << 16);
                    v[2 * u + 1] = __uint_as_float(wv[u] & 0xffff0000u);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (j < per) {
                        const __nv_bfloat16 hv = __ldcg(A.hidden_in + tid * per + j);
                        s_hin[tid * per + j] = hv;
                        v[j] = __bfloat162float(hv);
                    }
                }
            }
            float sq = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < per) sq = __fadd_rn(sq, __fmul_rn(v[j], v[j]));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, off));
            if (lane == 0) s_red[warp] = sq;
            named_barrier(1, kDlConsumers);
            float total = 0.0f;
#pragma unroll
            for (int w8 = 0; w8 < kDlWarps; ++w8) total = __fadd_rn(total, s_red[w8]);
            const float mean = __fmul_rn(total, 1.0f / static_cast<float>(H));
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, A.eps)));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (j < per) {
                    const int i = tid * per + j;
                    const __nv_bfloat16 y = __float2bfloat16_rn(__fmul_rn(__fmul_rn(v[j], inv), gam[j]));
                    s_norm[i] = y;
                    if (blockIdx.x == 0 && A.normed_out) A.normed_out[i] = y;
                }
            }
        } else {
            for (int i = tid; i < H; i += kDlConsumers) {
                const __nv_bfloat16 y = __ldcg(a.normed_in + i);
                s_norm[i] = y;
                s_hin[i] = __ldcg(A.hidden_in + i);
                if (blockIdx.x == 0 && A.normed_out) A.normed_out[i] = y;
            }
            for (int e = tid; e < E; e += kDlConsumers) s_logit[e] = __bfloat162float(__ldcg(a.logits_in + e));
        }
    }
    __syncthreads();
    cp_wait<0>();
    cluster.barrier_wait();  // every CTA of the cluster is running
    if (fused && warp < kDlWarps) {
        // Router GEMV share of this rank: rows e = r (mod 4), four per pass
        // of a warp; lane l owns elements 256i + 8l + j of every row, products
        // added in (i, j) order with separate multiply and add, lanes combined
        // by a xor butterfly, each logit rounded to bf16 and stored into every
        // CTA of the cluster.
        for (int q0 = 0;; q0 += 4) {
            if (r + kDlCluster * (warp + kDlWarps * q0) >= E) break;
            // rows q0..q0+3 of this warp; a row past E reads row q0 and is dropped
            const uint8_t* rows[4];
            bool live[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                live[u] = r + kDlCluster * (warp + kDlWarps * (q0 + u)) < E;
                rows[u] = base + static_cast<size_t>((live[u] ? q0 + u : q0) * kDlWarps + warp) * H * 2 + 16 * lane;
            }
            uint64_t acc01 = 0ull, acc23 = 0ull;  // {row 0, row 1}, {row 2, row 3}
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (i < H / 256) {
                    const uint4 xq = lds128(s_norm + 256 * i + 8 * lane);
                    const uint4 g0 = lds128(rows[0] + 512 * i), g1 = lds128(rows[1] + 512 * i);
                    const uint4 g2 = lds128(rows[2] + 512 * i), g3 = lds128(rows[3] + 512 * i);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float xj = bf16_at(xq, j);
                        const uint64_t xx = pack_f32x2(xj, xj);
                        acc01 = add_f32x2(acc01, mul_f32x2(xx, pack_f32x2(bf16_at(g0, j), bf16_at(g1, j))));
                        acc23 = add_f32x2(acc23, mul_f32x2(xx, pack_f32x2(bf16_at(g2, j), bf16_at(g3, j))));
                    }
                }
            }
            float acc[4];
            unpack_f32x2(acc01, acc[0], acc[1]);
            unpack_f32x2(acc23, acc[2], acc[3]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int u = 0; u < 4; ++u) acc[u] = __fadd_rn(acc[u], __shfl_xor_sync(0xffffffffu, acc[u], off));
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = r + kDlCluster * (warp + kDlWarps * (q0 + u));
                if (live[u] && lane < kDlCluster) *cluster.map_shared_rank(s_logit + e, lane) = bf16_round(acc[u]);
            }
        }
    }
    __syncwarp();
    cluster.sync();             // all logits in every CTA; no remote access until the next cluster barrier
    fence_proxy_async_smem();   // the router rows' bytes are rewritten by TMA below

    // Routing (softmax -> top-k -> renormalise, torch's order): warp 0 takes
    // the softmax; the consumer threads rank every probability (2 threads per
    // expert, each counting over half the row); warp 0 takes the k winners in
    // rank order when no two of them are equal, else puts them in the order
    // of torch's gatherTopK and sorts them with torch's network, while warps
    // 1..7 make the f16 copy of this quarter of the normalised row, scaled by
    // 2^-e with e from the whole row.
    const int E4 = (E + 3) & ~3;
    if (warp == 0) {
        route_softmax<LANES, ITERS>([&](int i) { return s_logit[i]; }, E, lane, s_logit);
    } else if (warp == 1 && lane < E4 - E) {
        s_logit[E + lane] = -1.0f;
    } else if (warp == 2) {
        // valid ids in every rank and order slot: with NaN probabilities no
        // expert claims some ranks, and their slots keep these
        s_rkey[lane] = 0.0f;
        s_ridx[lane] = lane < E ? lane : 0;
        s_key[lane] = 0.0f;
        s_idx[lane] = lane < E ? lane : 0;
    }
    __syncthreads();
    if (warp < kDlWarps) {
        const float4* p4 = reinterpret_cast<const float4*>(s_logit);
        const int n4 = E4 / 4, h4 = (n4 + 1) / 2;
        for (int e0 = 0; e0 < E; e0 += kDlConsumers / 2) {
            const int e = e0 + (tid >> 1), half = tid & 1;
            const float pe = e < E ? s_logit[e] : 0.0f;
            int rk = 0;
            if (e < E) {
                const int j4_end = half ? n4 : h4;
#pragma unroll 4
                for (int j4 = half ? h4 : 0; j4 < j4_end; ++j4) {
                    const float4 qv = p4[j4];
                    const int j = 4 * j4;
                    rk += (qv.x > pe) || (qv.x == pe && j < e);
                    rk += (qv.y > pe) || (qv.y == pe && j + 1 < e);
                    rk += (qv.z > pe) || (qv.z == pe && j + 2 < e);
                    rk += (qv.w > pe) || (qv.w == pe && j + 3 < e);
                }
            }
            rk += __shfl_xor_sync(0xffffffffu, rk, 1);
            if (e < E && half == 0 && rk < k) {
                s_rkey[rk] = pe;
                s_ridx[rk] = e;
            }
        }
    }
    __syncthreads();
    if (warp == 0) {
        const float v = lane < k ? s_rkey[lane] : -1.0f;
        const int ix = lane < k ? s_ridx[lane] : 0x7fffffff;
        int idx = 0;
        float wr = 0.0f;
        // With no two of the k winners equal, torch's sorted order is their
        // rank order (value descending) and the network below is the identity.
        const unsigned kmask = k < 32 ? (1u << k) - 1u : 0xffffffffu;
        const unsigned same = __match_any_sync(0xffffffffu, __float_as_uint(v)) & kmask & ~(1u << lane);
        if (!__any_sync(0xffffffffu, lane < k && same != 0u)) {
            idx = ix;
            wr = route_weight(k, true, lane, v, lane < k);
        } else {
            // gatherTopK order: values above the k-th in index order, then the
            // ones equal to it in index order; then torch's sorting network
            const float kth = s_rkey[k - 1];
            const bool gt = lane < k && v > kth;
            const unsigned gmask = __ballot_sync(0xffffffffu, gt);
            int before = 0;
            for (int m = 0; m < k; ++m) {
                const int im = __shfl_sync(0xffffffffu, ix, m);
                before += (((gmask >> m) & 1u) == static_cast<unsigned>(gt)) && im < ix;
            }
            if (lane < k) {
                const int pos = gt ? before : __popc(gmask) + before;
                s_key[pos] = v;
                s_idx[pos] = ix;
            }
            __syncwarp();
            route_finish(k, true, lane, s_key, s_idx, idx, wr);
        }
        idx = static_cast<unsigned>(idx) < static_cast<unsigned>(E) ? idx : 0;  // only NaN rows can miss
        const __nv_bfloat16 wb = __float2bfloat16_rn(wr);
        if (lane < k) {
            s_ids[lane] = idx;
            s_w[lane] = __bfloat162float(wb);
            if (blockIdx.x == 0) {
                if (A.ids_out) A.ids_out[lane] = idx;
                if (A.weights_out) A.weights_out[lane] = wb;
            }
        }
    } else if (warp < kDlWarps) {
        const int tw = tid - 32;
        float m = 0.0f;
        for (int i = tw; i < H; i += kDlConsumers - 32) m = fmaxf(m, fabsf(__bfloat162float(s_norm[i])));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (lane == 0) s_red[warp] = m;
        named_barrier(2, kDlConsumers - 32);
        float amax = 0.0f;
#pragma unroll
        for (int w8 = 1; w8 < kDlWarps; ++w8) amax = fmaxf(amax, s_red[w8]);
        const int e = f16_exponent_for(amax);
        const float inv = ldexpf(1.0f, -e);
        if (tw == 0) s_xscale = ldexpf(1.0f, e);
        for (int c = tw; c < HQ / 8; c += kDlConsumers - 32) {
            const uint4 q = lds128(s_norm + r * HQ + 8 * c);
            float vv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) vv[j] = bf16_at(q, j);
            s_x16[c] = pack8<0>(vv, inv);
        }
    }
    __syncthreads();

    const int expert = s_ids[slot_j];
    const int blk0 = tile0 >> 3;  // first 128-wide scale block of the unit's intermediate columns
    const DramaB200Fp8Bank& b = A.bank;
    if (warp == kDlWarps) {
        // Producer: stage s = the unit's tile tile0 + s, one 5-D box
        // {128 B, KBQ blocks, 16 rows, gate|up, 1 slot} per stage.
        if (lane == 0 && L.overlay) {
            // Every gate/up stage of the unit at once; the down rows to L2
            // now, and into the first stages once those are consumed.
            const uint64_t pol = policy_evict_first();
            for (int s = 0; s < nkt; ++s) {
                mbar_arrive_expect_tx(full0 + 8 * s, static_cast<uint32_t>(L.stage));
                tma_load_5d(base_u32 + s * L.stage, &a.w13_map, 0, r * KBQ, (tile0 + s) * 16, 0, expert,
                            full0 + 8 * s, pol);
            }
            const int rboxes = HQ / L.w2_rows;
            for (int bx = 0; bx < L.w2_boxes; ++bx) {
                const int cb = bx / rboxes, rb = bx - cb * rboxes;
                tma_prefetch_3d(&a.w2_map, (tile0 + 4 * cb) * 16, r * HQ + rb * L.w2_rows, expert);
            }
            for (int s = 0; s < L.w2_stages; ++s) mbar_wait(empty0 + 8 * s, 0, status);
            const uint32_t w2b = base_u32 + L.w2_bar;
            mbar_arrive_expect_tx(w2b, static_cast<uint32_t>(L.w2_boxes) * L.w2_rows * 64u);
            for (int bx = 0; bx < L.w2_boxes; ++bx) {
                const int cb = bx / rboxes, rb = bx - cb * rboxes;
                tma_load_3d(base_u32 + L.w2 + bx * L.w2_rows * 64, &a.w2_map, (tile0 + 4 * cb) * 16,
                            r * HQ + rb * L.w2_rows, expert, w2b, pol);
            }
        } else if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            const int first = nkt < L.stages ? nkt : L.stages;
            for (int s = 0; s < nkt; ++s) {
                const int st = s % L.stages;
                if (s >= L.stages) mbar_wait(empty0 + 8 * st, ((s / L.stages) - 1) & 1, status);
                mbar_arrive_expect_tx(full0 + 8 * st, static_cast<uint32_t>(L.stage));
                tma_load_5d(base_u32 + st * L.stage, &a.w13_map, 0, r * KBQ, (tile0 + s) * 16, 0, expert,
                            full0 + 8 * st, pol);
                if (s + 1 == first) {
                    // the down rows, behind the first ring of gate/up stages
                    const uint32_t w2b = base_u32 + L.w2_bar;
                    mbar_arrive_expect_tx(w2b, static_cast<uint32_t>(L.w2_boxes) * L.w2_rows * 64u);
                    const int rboxes = HQ / L.w2_rows;
                    for (int bx = 0; bx < L.w2_boxes; ++bx) {
                        const int cb = bx / rboxes, rb = bx - cb * rboxes;
                        tma_load_3d(base_u32 + L.w2 + bx * L.w2_rows * 64, &a.w2_map, (tile0 + 4 * cb) * 16,
                                    r * HQ + rb * L.w2_rows, expert, w2b, pol);
                    }
                }
            }
        }
        __syncwarp();
    } else {
        const uint64_t pol = policy_evict_first();
        // Block scales of the unit's down-projection columns for rows
        // [r HQ, (r+1) HQ) (the rows themselves come by TMA).
        const int nblk = ((tile0 + nkt - 1) >> 3) - blk0 + 1;
        {
            for (int item = tid; item < nblk * (HQ / 128); item += kDlConsumers) {
                const int c = item / (HQ / 128), nb = item - c * (HQ / 128);
                cp4(base_u32 + L.s2 + 4 * item, b.w2_scale + expert * b.w2_scale_slot_stride +
                                                    ((r * HQ) / 128 + nb) * b.w2_scale_row_stride + blk0 + c);
            }
            cp_commit();
        }
        // Block scales of this warp's cells (cell c = warp + 8i is K block
        // c % KBQ of stage c / KBQ): lane i < 16 holds cell i's gate scale,
        // lane 16 + i its up scale.
        const int cells = nkt * KBQ;
        float sc = 0.0f;
        {
            const int i = lane & 15, c = warp + kDlWarps * i;
            if (c < cells) {
                const int s = c / KBQ, kb = c - s * KBQ;
                const int row = (lane < 16 ? 0 : I) + (tile0 + s) * 16;
                sc = __ldg(b.w13_scale + expert * b.w13_scale_slot_stride + (row >> 7) * b.w13_scale_row_stride +
                           r * KBQ + kb);
            }
        }
        // Swizzled stage reads: 16-byte chunk c of 128-byte line l sits at
        // chunk c ^ (l & 7); rows g, g + 8, 16 + g, 24 + g of K block kb are
        // lines (row * KBQ + kb), all with the same l & 7. With fewer than 4
        // K blocks per line group, odd rows read their second chunk first so
        // that the lanes of one load hit distinct banks.
        const bool swap = KBQ < 4 && (g & 1);
        for (int i = 0;; ++i) {
            const int c = warp + kDlWarps * i;
            if (c >= cells) break;
            const int s = c / KBQ, kb = c - s * KBQ, st = s % L.stages;
            const uint32_t x = static_cast<uint32_t>((g * KBQ + kb) & 7);
            const uint32_t ca = (static_cast<uint32_t>(swap ? t + 4 : t) ^ x) << 4;
            const uint32_t cb = (static_cast<uint32_t>(swap ? t : t + 4) ^ x) << 4;
            const uint8_t* sb = base + st * L.stage + kb * 128;
            const uint8_t* r0 = sb + g * KBQ * 128;
            const uint8_t* r1 = sb + (g + 8) * KBQ * 128;
            const uint8_t* r2 = sb + (g + 16) * KBQ * 128;
            const uint8_t* r3 = sb + (g + 24) * KBQ * 128;
            mbar_wait(full0 + 8 * st, (s / L.stages) & 1, status);
            uint4 qa[4], qb[4];
            qa[0] = lds128(r0 + ca);
            qa[1] = lds128(r1 + ca);
            qa[2] = lds128(r2 + ca);
            qa[3] = lds128(r3 + ca);
            qb[0] = lds128(r0 + cb);
            qb[1] = lds128(r1 + cb);
            qb[2] = lds128(r2 + cb);
            qb[3] = lds128(r3 + cb);
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * st);
            uint4 q[8];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                q[2 * v] = swap ? qb[v] : qa[v];
                q[2 * v + 1] = swap ? qa[v] : qb[v];
            }
            uint32_t xb[16];
            if (g == 0) {
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    // lane t owns k = 16t.. and 64 + 16t.. of the block
                    const uint4 xv = s_x16[kb * 16 + 2 * t + (v & 1) + 8 * (v >> 1)];
                    xb[4 * v] = xv.x;
                    xb[4 * v + 1] = xv.y;
                    xb[4 * v + 2] = xv.z;
                    xb[4 * v + 3] = xv.w;
                }
            } else {
#pragma unroll
                for (int v = 0; v < 16; ++v) xb[v] = 0u;
            }
            const float sg = __shfl_sync(0xffffffffu, sc, i & 15);
            const float su = __shfl_sync(0xffffffffu, sc, 16 + (i & 15));
            float tot[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            up_mma_fp8_scaled(q, sg, su, xb, tot);
            if (t == 0) {
                float* dst = s_cell + (s * KBQ + kb) * 32;
                dst[g] = tot[0];
                dst[g + 8] = tot[2];
                dst[16 + g] = tot[4];
                dst[24 + g] = tot[6];
            }
        }
        named_barrier(1, kDlConsumers);
        // This CTA's quarter of every gate/up row sum (K blocks in order),
        // into slot r of every cluster CTA's exchange area.
        for (int idx = tid; idx < nkt * 32; idx += kDlConsumers) {
            const int s = idx >> 5, row = idx & 31;
            float v = 0.0f;
            for (int kb = 0; kb < KBQ; ++kb) v += s_cell[(s * KBQ + kb) * 32 + row];
            float* dst = s_xch + (r * L.nkt + s) * 32 + row;
#pragma unroll
            for (int d = 0; d < kDlCluster; ++d) *cluster.map_shared_rank(dst, d) = v;
        }
    }
    cluster.sync();  // every quarter of every row sum is in every CTA

    if (warp < kDlWarps) {
        // SiLU(gate) * up of the unit's tiles, quarters summed in rank order;
        // stored as f16 scaled by one power of two for the unit (exact for
        // bf16 values down to 2^-28 of the largest).
        {
            const int s = tid >> 4, j = tid & 15;
            float h = 0.0f;
            if (s < nkt) {
                float gsum = 0.0f, usum = 0.0f;
#pragma unroll
                for (int d = 0; d < kDlCluster; ++d) {
                    gsum += s_xch[(d * L.nkt + s) * 32 + j];
                    usum += s_xch[(d * L.nkt + s) * 32 + 16 + j];
                }
                const float gate = bf16_round(gsum * s_xscale);
                const float up = bf16_round(usum * s_xscale);
                const float act = bf16_round(gate / (1.0f + expf(-gate)));
                h = bf16_round(act * up);
            }
            float m = fabsf(h);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
            if (lane == 0) s_red[warp] = m;
            named_barrier(1, kDlConsumers);
            float amax = 0.0f;
#pragma unroll
            for (int w8 = 0; w8 < kDlWarps; ++w8) amax = fmaxf(amax, s_red[w8]);
            const int e = f16_exponent_for(amax);
            if (s < nkt) s_h16[s * 16 + j] = __float2half_rn(h * ldexpf(1.0f, -e));
            if (tid == 0) s_hscale = ldexpf(1.0f, e);
        }
        cp_wait<0>();
        mbar_wait(base_u32 + L.w2_bar, 0, status);
        named_barrier(1, kDlConsumers);  // h, the down rows and their scales in shared memory
        // Partial down projection: warp w takes 16-row tiles w, w + 8, ... of
        // the quarter, up to four at once; lane (g, t) reads word t of each
        // 16-byte chunk of rows g and g + 8 (physical k = 4t.. of the tile)
        // and the h fragment in the same order. A TMA box holds 64-byte rows
        // with 16-byte chunk c of row n at chunk c ^ ((n >> 1) & 3). Chunks of
        // one 128-wide scale block accumulate in the MMA; each block is scaled
        // once.
        const uint8_t* w2s = base + L.w2;
        const uint8_t* h16s = reinterpret_cast<const uint8_t*>(s_h16);
        const float hscale = s_hscale;
        float* part = a.part + static_cast<int64_t>(unit) * H + r * HQ;
        if constexpr (NKTC > 0) {
            // Fixed shape: warp w takes row tiles w + 8u of the quarter; the
            // unit's tiles span at most two scale blocks, the first cb tiles
            // in block blk0 (the host checks NKTC - cb <= 8).
            constexpr int kU = HC / kDlCluster / 16 / kDlWarps;
            const int cb = 8 - (tile0 & 7);
            const uint8_t* rowb[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) rowb[u] = w2s + ((warp + kDlWarps * u) * 16 + g) * 64 + 4 * t;
            float dA[kU][4], dB[kU][4];
#pragma unroll
            for (int u = 0; u < kU; ++u)
#pragma unroll
                for (int e = 0; e < 4; ++e) dA[u][e] = dB[u][e] = 0.0f;
#pragma unroll
            for (int c = 0; c < NKTC; ++c) {
                const uint2 hb = lds64(h16s + c * 32 + 8 * t);
                const uint32_t off = static_cast<uint32_t>((c >> 2) * (HC / kDlCluster) * 64) +
                                     (static_cast<uint32_t>((c & 3) ^ ((g >> 1) & 3)) << 4);
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    uint32_t Af[4];
                    e4m3x4_to_f16x2x2(lds32(rowb[u] + off), Af[0], Af[2]);
                    e4m3x4_to_f16x2x2(lds32(rowb[u] + off + 8 * 64), Af[1], Af[3]);
                    if (c < cb)
                        mma_f16_16816(dA[u], Af, hb.x, hb.y);
                    else
                        mma_f16_16816(dB[u], Af, hb.x, hb.y);
                }
            }
            if (t == 0) {
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int nt = warp + kDlWarps * u;
                    const float sa = s_s2[(nt * 16) >> 7] * hscale;
                    float a0 = fmaf(dA[u][0], sa, 0.0f), a1 = fmaf(dA[u][2], sa, 0.0f);
                    if (NKTC > cb) {
                        const float sb = s_s2[(HC / kDlCluster / 128) + ((nt * 16) >> 7)] * hscale;
                        a0 = fmaf(dB[u][0], sb, a0);
                        a1 = fmaf(dB[u][2], sb, a1);
                    }
                    __stcg(part + nt * 16 + g, a0);
                    __stcg(part + nt * 16 + g + 8, a1);
                }
            }
        } else {
            const int NT = HQ / 16;
            for (int i0 = 0; warp + kDlWarps * i0 < NT; i0 += 4) {
                int nt[4];
                bool ok[4];
                float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
    #pragma unroll
                for (int u = 0; u < 4; ++u) {
                    nt[u] = warp + kDlWarps * (i0 + u);
                    ok[u] = nt[u] < NT;
                }
                // row n of a column box at (n / rows_box) * rows_box * 64 + (n % rows_box) * 64
                const uint8_t* rowb[4];
    #pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int n = (ok[u] ? nt[u] : warp) * 16 + g;
                    rowb[u] = w2s + n * 64 + 4 * t;
                }
                for (int c = 0; c < nkt;) {
                    const int blk = (tile0 + c) >> 3;
                    const int cend = min(nkt, (blk + 1) * 8 - tile0);
                    float d[4][4];
    #pragma unroll
                    for (int u = 0; u < 4; ++u) d[u][0] = d[u][1] = d[u][2] = d[u][3] = 0.0f;
                    for (; c < cend; ++c) {
                        const uint2 hb = lds64(h16s + c * 32 + 8 * t);
                        const uint32_t off = static_cast<uint32_t>((c >> 2) * HQ * 64) +
                                             (static_cast<uint32_t>((c & 3) ^ ((g >> 1) & 3)) << 4);
    #pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            if (ok[u]) {
                                uint32_t Af[4];
                                e4m3x4_to_f16x2x2(lds32(rowb[u] + off), Af[0], Af[2]);
                                e4m3x4_to_f16x2x2(lds32(rowb[u] + off + 8 * 64), Af[1], Af[3]);
                                mma_f16_16816(d[u], Af, hb.x, hb.y);
                            }
                        }
                    }
    #pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        if (ok[u]) {
                            const float scale = s_s2[(blk - blk0) * (HQ / 128) + ((nt[u] * 16) >> 7)] * hscale;
                            acc0[u] = fmaf(d[u][0], scale, acc0[u]);
                            acc1[u] = fmaf(d[u][2], scale, acc1[u]);
                        }
                    }
                }
                if (t == 0) {
    #pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        if (ok[u]) {
                            __stcg(part + nt[u] * 16 + g, acc0[u]);
                            __stcg(part + nt[u] * 16 + g + 8, acc1[u]);
                        }
                    }
                }
            }
        }
        // Ticket: the CTA barrier orders every thread's partial stores before
        // thread 0's release, and its acquire orders the last arriver's reads
        // of the other units' partials (after the next barrier).
        named_barrier(1, kDlConsumers);
        if (tid == 0) s_last = atomic_add_acq_rel_gpu(a.tickets + r, 1) == units - 1;
        named_barrier(1, kDlConsumers);
        if (s_last) {
            // Last CTA of quarter r: every unit's partial of the quarter into
            // shared memory (unit u = j P + p at u HQ), then for each row each
            // slot's parts in part order, rounded, weighted, slots added in
            // slot order, and the residual; a thread owns two adjacent rows.
            if (tid == 0) a.tickets[r] = 0;
            for (int item = tid; item < units * (HQ / 4); item += kDlConsumers) {
                const int u = item / (HQ / 4), c = item - u * (HQ / 4);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(base_u32 + (u * HQ + 4 * c) * 4),
                             "l"(a.part + static_cast<int64_t>(u) * H + r * HQ + 4 * c)
                             : "memory");
            }
            cp_commit();
            cp_wait<0>();
            named_barrier(1, kDlConsumers);
            const float2* sp = reinterpret_cast<const float2*>(base);
            for (int c2 = tid; c2 < HQ / 2; c2 += kDlConsumers) {
                float y0 = 0.0f, y1 = 0.0f;
                dl_slot_sums<PC>(sp, c2, HQ / 2, k, P, s_w, y0, y1);
                const int row = r * HQ + 2 * c2;
                const uint32_t hin = *reinterpret_cast<const uint32_t*>(s_hin + row);
                const __nv_bfloat16 m0 = __float2bfloat16_rn(y0), m1 = __float2bfloat16_rn(y1);
                const __nv_bfloat16 o0 = __float2bfloat16_rn(__uint_as_float(hin << 16) + __bfloat162float(m0));
                const __nv_bfloat16 o1 =
                    __float2bfloat16_rn(__uint_as_float(hin & 0xffff0000u) + __bfloat162float(m1));
                if (A.moe_out) *reinterpret_cast<__nv_bfloat162*>(A.moe_out + row) = __halves2bfloat162(m0, m1);
                *reinterpret_cast<__nv_bfloat162*>(A.hidden_out + row) = __halves2bfloat162(o0, o1);
            }
        }
    }
}

struct DlPlan {
    int parts, nkt, stages;
    DlLayout layout;
};

// Units per expert, tiles per unit and ring depth for a shape, or parts = 0
// when the shape is outside this kernel's envelope.
DlPlan dl_plan(int H, int I, int E, int k, int clusters) {
    DlPlan p{};
    if (H % (128 * kDlCluster) || H > kDlMaxHidden || I % 16 || I < 16 || E < 1 || E > 256 || k < 1 || k > 16)
        return p;
    const int tpi = I / 16;
    int parts = clusters / k;
    if (parts > tpi) parts = tpi;
    if (parts < 1) return p;
    const int nkt = (tpi + parts - 1) / parts;
    if (nkt > kDlMaxTiles) return p;
    // Every stage of the unit resident (the down rows over the first ones)
    // when shared memory allows, else a ring of up to 8 stages beside them.
    DlLayout L = dl_layout(H, E, nkt, nkt, 1);
    int use = nkt;
    if (L.total > static_cast<uint32_t>(kDlMaxSmem) || nkt < L.w2_stages) {
        const DlLayout base = dl_layout(H, E, nkt, 0, 0);
        const int stages = static_cast<int>((kDlMaxSmem - static_cast<int>(base.total)) / base.stage);
        if (stages < 2) return p;
        use = stages > 8 ? 8 : stages;
        L = dl_layout(H, E, nkt, use, 0);
        if (L.total > static_cast<uint32_t>(kDlMaxSmem)) return p;
    }
    // every router row of a rank staged in the region before routing, and
    // every unit's partial rows of a quarter in it for the combine
    if (static_cast<uint32_t>((E + kDlCluster - 1) / kDlCluster) * H * 2 > L.region ||
        static_cast<size_t>(k) * parts * L.hq * 4 > L.region)
        return p;
    p.parts = parts;
    p.nkt = nkt;
    p.stages = use;
    p.layout = L;
    return p;
}

}  // namespace

TensorMapEncode tensor_map_encoder() {
    static TensorMapEncode fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult found{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &found) == cudaSuccess &&
            found == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<TensorMapEncode>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

using DecodeLayerKernel = void (*)(DecodeLayerArgs);

// The instantiation for `experts` (up to 256 experts), or null.
DecodeLayerKernel decode_layer_kernel_for(int experts) {
    int p2 = 1;
    while (p2 < experts) p2 <<= 1;
    switch (p2) {
        case 1: return decode_layer_kernel<1, 1, 0, 0, 0, 0>;
        case 2: return decode_layer_kernel<2, 1, 0, 0, 0, 0>;
        case 4: return decode_layer_kernel<4, 1, 0, 0, 0, 0>;
        case 8: return decode_layer_kernel<8, 1, 0, 0, 0, 0>;
        case 16: return decode_layer_kernel<16, 1, 0, 0, 0, 0>;
        case 32: return decode_layer_kernel<32, 1, 0, 0, 0, 0>;
        case 64: return decode_layer_kernel<32, 2, 0, 0, 0, 0>;
        case 128: return decode_layer_kernel<32, 4, 0, 0, 0, 0>;
        case 256: return decode_layer_kernel<32, 8, 0, 0, 0, 0>;
        default: return nullptr;
    }
}

// The shape-specialised instantiation for a plan, or nullptr: hidden 2048
// with 128 experts (the reference's configuration: intermediate 768, top-8),
// four units per route slot of exactly 12 tiles each with all stages
// resident, and every unit's tiles within two 128-wide scale blocks.
DecodeLayerKernel decode_layer_kernel_fixed(int H, int I, int E, int parts, int nkt, int stages, int overlay) {
    constexpr int kH = 2048, kNkt = 12, kParts = 4, kE = 128;
    if (H != kH || E != kE || parts != kParts || nkt != kNkt || stages != kNkt || !overlay) return nullptr;
    const int tpi = I / 16;
    if (tpi != kParts * kNkt) return nullptr;
    for (int p = 0; p < parts; ++p)
        if (kNkt - (8 - ((tpi * p / parts) & 7)) > 8) return nullptr;
    return decode_layer_kernel<32, 4, kH, kNkt, kParts, kE>;
}

int decode_layer_clusters() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cached[dev]) return cached[dev];
    for (int e = 1; e <= 512; e <<= 1) {
        DecodeLayerKernel kern = e <= 256 ? decode_layer_kernel_for(e) : decode_layer_kernel<32, 4, 2048, 12, 4, 128>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDlMaxSmem) != cudaSuccess) {
            cudaGetLastError();
            return cached[dev] = -1;
        }
    }
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(kDlCluster * ((sms + kDlCluster - 1) / kDlCluster));
    q.blockDim = dim3(kDlThreads);
    q.dynamicSmemBytes = kDlMaxSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kDlCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    q.attrs = attr;
    q.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, decode_layer_kernel<32, 4, 0, 0, 0, 0>, &q) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        return cached[dev] = -1;
    }
    return cached[dev] = clusters;
}

bool decode_layer_supported(int64_t tokens, int top_k, int hidden, int intermediate, int experts) {
    if (tokens != 1 || !tensor_map_encoder() || !decode_layer_kernel_for(experts)) return false;
    const int clusters = decode_layer_clusters();
    return clusters > 0 && dl_plan(hidden, intermediate, experts, top_k, clusters).parts > 0;
}

cudaError_t decode_layer_launch(DecodeLayerArgs a, cudaStream_t s) {
    const int clusters = decode_layer_clusters();
    if (clusters <= 0) return cudaErrorInvalidConfiguration;
    const RoutedLayerArgs& A = a.layer;
    const DlPlan p = dl_plan(A.H, A.I, A.E, A.k, clusters);
    const TensorMapEncode encode = tensor_map_encoder();
    if (!p.parts || !encode) return cudaErrorInvalidConfiguration;
    a.parts = p.parts;
    a.nkt = p.nkt;
    a.stages = p.stages;
    a.overlay = p.layout.overlay;
    // W13 [slot][gate|up][row][H] viewed as [slot][2][I][H/128][128] bytes;
    // one box = 16 rows of gate and up, this CTA's H/4 bytes of each.
    const DramaB200Fp8Bank& b = A.bank;
    const cuuint64_t dims[5] = {128, static_cast<cuuint64_t>(A.H / 128), static_cast<cuuint64_t>(A.I), 2,
                                static_cast<cuuint64_t>(b.slots)};
    const cuuint64_t strides[4] = {128, static_cast<cuuint64_t>(b.w13_row_stride),
                                   static_cast<cuuint64_t>(b.w13_row_stride) * A.I,
                                   static_cast<cuuint64_t>(b.w13_slot_stride)};
    const cuuint32_t box[5] = {128, static_cast<cuuint32_t>(A.H / kDlCluster / 128), 16, 2, 1};
    const cuuint32_t unit_strides[5] = {1, 1, 1, 1, 1};
    if (encode(&a.w13_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<void*>(b.w13), dims, strides, box,
               unit_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    // W2 [slot][row][I] bytes; one box = 64 bytes (4 tiles) x up to 256 rows.
    const cuuint64_t dims2[3] = {static_cast<cuuint64_t>(A.I), static_cast<cuuint64_t>(A.H),
                                 static_cast<cuuint64_t>(b.slots)};
    const cuuint64_t strides2[2] = {static_cast<cuuint64_t>(b.w2_row_stride), static_cast<cuuint64_t>(b.w2_slot_stride)};
    const cuuint32_t box2[3] = {64, static_cast<cuuint32_t>(p.layout.w2_rows), 1};
    if (encode(&a.w2_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(b.w2), dims2, strides2, box2,
               unit_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = kDlCluster;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kDlCluster * A.k * p.parts);
    cfg.blockDim = dim3(kDlThreads);
    cfg.dynamicSmemBytes = p.layout.total;
    cfg.stream = s;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    DecodeLayerKernel kern = decode_layer_kernel_fixed(A.H, A.I, A.E, p.parts, p.nkt, p.stages, p.layout.overlay);
    return cudaLaunchKernelEx(&cfg, kern ? kern : decode_layer_kernel_for(A.E), a);
}

}  // namespace drama
