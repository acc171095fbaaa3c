// K1: decode-regime dequantising SwiGLU expert FFN (FP8 block-scaled / INT4).
//
// Semantics follow the reference's PyTorch dequant path, TorchExpertBackend
// (src/drama_low_vram/offload.py:199-244), and QuantizedExpertBackend(0)
// (src/drama_low_vram/quantized_kernels.py:217-248): gate/up projections are
// rounded to x's dtype, silu(gate) and silu(gate)*up are rounded to x's dtype,
// the down projection is rounded to x's dtype, multiplied by the route weight
// in fp32, and route slots are summed in slot order in fp32.
//
// Structure (launches chained with programmatic dependent launch):
//   prep : stable bucket of route slots into expert groups of <= 8 tokens,
//          f16 copy of x scaled by a power of two per token (exact for bf16).
//          (The fused MoE layer's router kernel does this job in the stack.)
//   up   : weight-streaming GEMV over cells = (group, 16-row gate/up tile,
//          128-K block). Every warp of a persistent grid (one CTA per SM) owns
//          q consecutive cells and streams them through a private ring of
//          shared-memory stages with 16-byte cp.async copies (no registers held
//          while loads are in flight; at batch 1 a warp's whole range is in
//          flight before its first MMA). Weights are converted in registers (E4M3x2 -> f16x2 in one instruction;
//          INT4 nibbles with one LOP3 + one f16x2 subtract per two values) and
//          fed to m16n8k16 MMAs whose N dimension holds the group's tokens, so
//          weight bytes are read once per group. Block scales are applied per
//          128-K block in fp32. Tiles split between warps are reduced in K order
//          by the last arriving warp, which applies SiLU*mul. The kernel also
//          bulk-prefetches the selected experts' down-projection slabs to L2.
//   down : same scheme over (group, 16-row tile of H, 128-K block); the last
//          arriving warp of a tile rounds, applies the route weight and, once
//          every group of that row tile is done, sums the route slots.
#include "common.cuh"
#include "kernels.h"
#include "bucket.cuh"
#include "decode_tiles.cuh"

namespace drama {

namespace {
// ---------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------
template <int FMT>
__global__ void __launch_bounds__(1024) decode_prep_kernel(DecodeArgs a) {
    extern __shared__ int smem_prep[];
    int* smem = smem_prep;
    __shared__ int dropped;
    __shared__ int warp_tot[32];
    grid_dependency_wait();
    grid_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t P = a.tokens * a.top_k;
    const int S = a.slots;
    const DecodeWorkspace& ws = a.ws;
    if (tid == 0) dropped = 0;
    __syncthreads();
    stable_bucket(a.ids, a.ids_dtype, P, S, smem, nullptr, ws.order, &dropped);
    // groups of <= 8 pairs per slot, in slot order.
    const int* counts = smem;
    const int* ends = smem + S;
    int ng = 0;
    if (tid < S) ng = (counts[tid] + kGroupTokens - 1) / kGroupTokens;
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
            int pairs[kGroupTokens];
            const int cnt = min(kGroupTokens, c - j * kGroupTokens);
            for (int q = 0; q < cnt; ++q) pairs[q] = ws.order[start + j * kGroupTokens + q];
            write_group(ws, gbase + j, tid, start + j * kGroupTokens, cnt, pairs);
        }
    }
    const int groups = warp_tot[31];
    if (tid == 0) {
        ws.num_groups[0] = groups;
        ws.status[0] = dropped;
    }
    zero_split_counters(ws, groups, a.hidden, a.intermediate, tid, blockDim.x);
    for (int64_t p = tid; p < P; p += blockDim.x) ws.wts[p] = load_any(a.weights, a.weights_dtype, p);
    if (dropped) {
        // Pairs with an out-of-range slot contribute zero (and are counted).
        float* po = a.pair_out ? a.pair_out : ws.pair_out;
        for (int64_t p = 0; p < P; ++p) {
            const int64_t id = load_index(a.ids, a.ids_dtype, p);
            if (id < 0 || id >= S)
                for (int n = tid; n < a.hidden; n += blockDim.x) po[p * a.hidden + n] = 0.0f;
        }
    }
    // f16 copy of every token row scaled by 2^-e: all threads on 8-element
    // chunks of all rows; per-row amax via an order-free atomicMax.
    const int H = a.hidden;
    unsigned* s_amax = reinterpret_cast<unsigned*>(smem + 34 * S);
    for (int64_t t = tid; t < a.tokens; t += blockDim.x) s_amax[t] = 0u;
    __syncthreads();
    const int64_t chunks = a.tokens * (H / 8);
    for (int64_t c = tid; c < chunks; c += blockDim.x) {
        float v[8];
        load8(a.x, a.x_dtype, c * 8, v);
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
        atomicMax(s_amax + c / (H / 8), __float_as_uint(m));
    }
    __syncthreads();
    for (int64_t t = tid; t < a.tokens; t += blockDim.x)
        ws.xscale[t] = ldexpf(1.0f, f16_exponent_for(__uint_as_float(s_amax[t])));
    for (int64_t c = tid; c < chunks; c += blockDim.x) {
        float v[8];
        load8(a.x, a.x_dtype, c * 8, v);
        const float inv = ldexpf(1.0f, -f16_exponent_for(__uint_as_float(s_amax[c / (H / 8)])));
        reinterpret_cast<uint4*>(ws.x16)[c] = pack8<FMT>(v, inv);
    }
}

template <int FMT, int XDT>
__global__ void __launch_bounds__(UpShape<FMT>::WARPS * 32, 1) decode_up_kernel(DecodeArgs a) {
    constexpr int NCH = UpShape<FMT>::NCH, DEPTH = UpShape<FMT>::DEPTH, WARPS = UpShape<FMT>::WARPS;
    extern __shared__ __align__(16) uint4 smem_up[];
    uint4* smem = smem_up;
    grid_dependency_wait();
    grid_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int KB = a.hidden / 128, TILES = a.intermediate / 16;
    const int w = blockIdx.x * WARPS + warp;
    GroupRec ig{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
    const Work wk = plan_work(a, TILES, KB, gridDim.x * WARPS, KB / UpShape<FMT>::UNIT_DIV, w, ig);
    const uint64_t pol = policy_evict_first();
    uint4* ring = smem + warp * DEPTH * NCH * 32;
    const uint32_t ring_base = smem_u32(ring + lane);
    uint4* s_x = smem + WARPS * DEPTH * NCH * 32;

    // Prologue: every cell of a short range is in flight before any compute.
    const int n = wk.c1 - wk.c0;
    CellIt iss = cell_at(wk.c0, KB, TILES);
#pragma unroll
    for (int s = 0; s < DEPTH; ++s) {
        if (s < n) {
            load_group(ig, iss.grp, a.ws);
            up_issue<FMT>(ring_base + s * NCH * 512, a, ig.slot, iss, g, t, pol);
            advance(iss, KB, TILES);
        }
        cp_commit();
    }
    // Stage the f16 activation rows in shared memory when they fit.
    const int rowv = a.hidden / 8 + 1;
    const bool staged = static_cast<int64_t>(a.tokens) * rowv * 16 <= kXReserve;
    if (staged) {
        const uint4* src = reinterpret_cast<const uint4*>(a.ws.x16);
        const int per = a.hidden / 8;
        const int total = static_cast<int>(a.tokens) * per;
        for (int i = threadIdx.x; i < total; i += blockDim.x) s_x[(i / per) * rowv + i % per] = __ldcg(src + i);
    }
    prefetch_down_slabs(a, wk.groups);
    __syncthreads();
    if (n == 0) return;

    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    CellIt cur = cell_at(wk.c0, KB, TILES);
    int cur_tile = cur.grp * TILES + cur.jt;
    GroupRec cg{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
    int xtok = -1;
    for (int i = 0; i < n; ++i) {
        const int stage = i % DEPTH;
        cp_wait<DEPTH - 1>();
        const int tile = cur.grp * TILES + cur.jt;
        if (tile != cur_tile) {
            if (tile_flush<8>(acc, cur_tile, KB, wk.pt, w, a.ws.up_part, a.ws.up_cnt, lane)) {
                GroupRec fg{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
                load_group(fg, cur_tile / TILES, a.ws);
                up_finalize<XDT>(a, fg, cur_tile % TILES, acc, g, t);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
            cur_tile = tile;
        }
        if (cg.id != cur.grp) {
            load_group(cg, cur.grp, a.ws);
            xtok = g < cg.count ? rec_pair(cg, g) / a.top_k : -1;
        }
        uint4 q[NCH];
#pragma unroll
        for (int v = 0; v < NCH; ++v) q[v] = ring[(stage * NCH + v) * 32 + lane];
        uint32_t xb[16];
        if (xtok >= 0) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                // FP8: k = 16t.. and 64+16t.. (8 halves per uint4); INT4: k = 32t..
                const int off = FMT == 0 ? cur.kb * 16 + 2 * t + (v & 1) + 8 * (v >> 1) : cur.kb * 16 + 4 * t + v;
                const uint4 x = staged ? s_x[xtok * rowv + off]
                                       : __ldcg(reinterpret_cast<const uint4*>(a.ws.x16) +
                                                static_cast<int64_t>(xtok) * (a.hidden / 8) + off);
                xb[4 * v] = x.x;
                xb[4 * v + 1] = x.y;
                xb[4 * v + 2] = x.z;
                xb[4 * v + 3] = x.w;
            }
        } else {
#pragma unroll
            for (int v = 0; v < 16; ++v) xb[v] = 0u;
        }
        up_mma<FMT>(q, a, cg.slot, cur, g, xb, acc);
        // The stage's data is in registers (consumed above): refill it.
        if (i + DEPTH < n) {
            load_group(ig, iss.grp, a.ws);
            up_issue<FMT>(ring_base + stage * NCH * 512, a, ig.slot, iss, g, t, pol);
            advance(iss, KB, TILES);
        }
        cp_commit();
        advance(cur, KB, TILES);
    }
    if (tile_flush<8>(acc, cur_tile, KB, wk.pt, w, a.ws.up_part, a.ws.up_cnt, lane)) {
        GroupRec fg{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
        load_group(fg, cur_tile / TILES, a.ws);
        up_finalize<XDT>(a, fg, cur_tile % TILES, acc, g, t);
    }
}

template <int FMT, int XDT>
__global__ void __launch_bounds__(DnShape<FMT, XDT>::WARPS * 32, 1) decode_down_kernel(DecodeArgs a) {
    using S = DnShape<FMT, XDT>;
    constexpr int NCH = S::NCH, DEPTH = S::DEPTH, WARPS = S::WARPS;
    extern __shared__ __align__(16) uint4 smem_dn[];
    uint4* smem = smem_dn;
    grid_dependency_wait();
    grid_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int KB = a.intermediate / 128, TILES = a.hidden / 16;
    const int w = blockIdx.x * WARPS + warp;
    GroupRec ig{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
    const Work wk = plan_work(a, TILES, KB, gridDim.x * WARPS, KB / S::UNIT_DIV, w, ig);
    if (wk.groups == 0) {
        // Every pair was dropped: the combined output is zero (plus residual).
        if (a.out && blockIdx.x == 0) {
            using T = typename Scalar<XDT>::T;
            for (int64_t i = threadIdx.x; i < a.tokens * a.hidden; i += blockDim.x) {
                float v = 0.0f;
                if (a.residual) v = Scalar<XDT>::round(Scalar<XDT>::load(static_cast<const T*>(a.residual) + i));
                static_cast<T*>(a.out)[i] = Scalar<XDT>::from(v);
            }
        }
        return;
    }
    const uint64_t pol = policy_evict_first();
    float* pair_out = a.pair_out ? a.pair_out : a.ws.pair_out;
    uint4* ring = smem + warp * DEPTH * NCH * 32;
    const uint32_t ring_base = smem_u32(ring + lane);
    const int n = wk.c1 - wk.c0;
    if (n == 0) return;

    CellIt iss = cell_at(wk.c0, KB, TILES);
#pragma unroll
    for (int s = 0; s < DEPTH; ++s) {
        if (s < n) {
            load_group(ig, iss.grp, a.ws);
            dn_issue<FMT, XDT>(ring_base + s * NCH * 512, a, ig, iss, g, t, pol);
            advance(iss, KB, TILES);
        }
        cp_commit();
    }

    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    CellIt cur = cell_at(wk.c0, KB, TILES);
    int cur_tile = cur.grp * TILES + cur.jt;
    GroupRec cg{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
    for (int i = 0; i < n; ++i) {
        const int stage = i % DEPTH;
        cp_wait<DEPTH - 1>();
        const int tile = cur.grp * TILES + cur.jt;
        if (tile != cur_tile) {
            if (tile_flush<4>(acc, cur_tile, KB, wk.pt, w, a.ws.dn_part, a.ws.dn_cnt, lane)) {
                GroupRec fg{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
                load_group(fg, cur_tile / TILES, a.ws);
                dn_finalize<XDT>(a, fg, cur_tile % TILES, acc, g, t, lane, wk.groups, pair_out);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j] = 0.0f;
            cur_tile = tile;
        }
        if (cg.id != cur.grp) load_group(cg, cur.grp, a.ws);
        uint4 q[NCH];
#pragma unroll
        for (int v = 0; v < NCH; ++v) q[v] = ring[(stage * NCH + v) * 32 + lane];
        uint32_t hb[16];
        const int e = dn_fragment<FMT, XDT>(q + S::NW, hb);
        dn_mma<FMT>(q, a, cg.slot, cur, g, t, hb, e, acc);
        if (i + DEPTH < n) {
            load_group(ig, iss.grp, a.ws);
            dn_issue<FMT, XDT>(ring_base + stage * NCH * 512, a, ig, iss, g, t, pol);
            advance(iss, KB, TILES);
        }
        cp_commit();
        advance(cur, KB, TILES);
    }
    if (tile_flush<4>(acc, cur_tile, KB, wk.pt, w, a.ws.dn_part, a.ws.dn_cnt, lane)) {
        GroupRec fg{-1, 0, 0, 0, {0u, 0u, 0u, 0u}};
        load_group(fg, cur_tile / TILES, a.ws);
        dn_finalize<XDT>(a, fg, cur_tile % TILES, acc, g, t, lane, wk.groups, pair_out);
    }
}

template <int FMT>
constexpr size_t up_smem_bytes() {
    return static_cast<size_t>(UpShape<FMT>::WARPS) * UpShape<FMT>::DEPTH * UpShape<FMT>::NCH * 512 + kXReserve;
}
template <int FMT, int XDT>
constexpr size_t dn_smem_bytes() {
    using S = DnShape<FMT, XDT>;
    return static_cast<size_t>(S::WARPS) * S::DEPTH * S::NCH * 512;
}

template <int FMT, int XDT>
cudaError_t launch_experts(const DecodeArgs& a, cudaStream_t s) {
    static bool configured = false;  // benign race: identical values
    if (!configured) {
        cudaError_t err = cudaFuncSetAttribute(decode_up_kernel<FMT, XDT>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(up_smem_bytes<FMT>()));
        if (err != cudaSuccess) return err;
        err = cudaFuncSetAttribute(decode_down_kernel<FMT, XDT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(dn_smem_bytes<FMT, XDT>()));
        if (err != cudaSuccess) return err;
        configured = true;
    }
    cudaError_t err = launch_pdl(decode_up_kernel<FMT, XDT>, dim3(a.ctas), dim3(UpShape<FMT>::WARPS * 32),
                                 up_smem_bytes<FMT>(), s, a);
    if (err != cudaSuccess) return err;
    return launch_pdl(decode_down_kernel<FMT, XDT>, dim3(a.ctas), dim3(DnShape<FMT, XDT>::WARPS * 32),
                      dn_smem_bytes<FMT, XDT>(), s, a);
}

template <int FMT, int XDT>
cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t s) {
    const size_t smem = bucket_smem_bytes(a.slots) + a.tokens * sizeof(unsigned);
    static bool configured = false;
    if (!configured) {
        const cudaError_t err =
            cudaFuncSetAttribute(decode_prep_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(bucket_smem_bytes(kMaxSlots) + kMaxDecodePairs * sizeof(unsigned)));
        if (err != cudaSuccess) return err;
        configured = true;
    }
    const cudaError_t err = launch_pdl(decode_prep_kernel<FMT>, dim3(1), dim3(1024), smem, s, a);
    if (err != cudaSuccess) return err;
    return launch_experts<FMT, XDT>(a, s);
}

}  // namespace

size_t decode_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, int sm_count, int experts,
                               char* base, DecodeWorkspace* ws) {
    const int64_t P = tokens * top_k;
    const int64_t W = static_cast<int64_t>(sm_count) * kDecodeCtasPerSm * kDecodeMaxWarps;
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return p;
    };
    DecodeWorkspace w{};
    w.status = reinterpret_cast<int32_t*>(take(16));
    w.num_groups = reinterpret_cast<int32_t*>(take(4));
    w.order = reinterpret_cast<int32_t*>(take(P * 4));
    w.g_rec = reinterpret_cast<int4*>(take(P * 32));
    w.xscale = reinterpret_cast<float*>(take(tokens * 4));
    w.x16 = reinterpret_cast<uint16_t*>(take(tokens * hidden * 2));
    w.wts = reinterpret_cast<float*>(take(P * 4));
    w.h = take(P * intermediate * 4);
    w.pair_out = reinterpret_cast<float*>(take(P * hidden * 4));
    w.up_part = reinterpret_cast<float*>(take(W * 2 * 32 * 8 * 4));
    w.up_cnt = reinterpret_cast<int32_t*>(take(P * (intermediate / 16) * 4));
    w.dn_part = reinterpret_cast<float*>(take(W * 2 * 32 * 4 * 4));
    w.dn_cnt = reinterpret_cast<int32_t*>(take(P * (hidden / 16) * 4));
    w.cmb_cnt = reinterpret_cast<int32_t*>(take((hidden / 16) * 4));
    if (experts > 0) {
        w.logits = reinterpret_cast<float*>(take(tokens * experts * 4));
        w.router_cnt = reinterpret_cast<int32_t*>(take(4));
        w.layer_part = reinterpret_cast<float*>(take(static_cast<size_t>(sm_count) * hidden * 4));
        w.layer_tickets = reinterpret_cast<int32_t*>(take(64));
    }
    if (ws) *ws = w;
    return off;
}

cudaError_t decode_experts_launch(const DecodeArgs& a, cudaStream_t s) {
    switch (a.format * 8 + a.x_dtype) {
        case 0 * 8 + DRAMA_B200_BF16: return launch_experts<0, DRAMA_B200_BF16>(a, s);
        case 0 * 8 + DRAMA_B200_F16: return launch_experts<0, DRAMA_B200_F16>(a, s);
        case 0 * 8 + DRAMA_B200_F32: return launch_experts<0, DRAMA_B200_F32>(a, s);
        case 1 * 8 + DRAMA_B200_BF16: return launch_experts<1, DRAMA_B200_BF16>(a, s);
        case 1 * 8 + DRAMA_B200_F16: return launch_experts<1, DRAMA_B200_F16>(a, s);
        default: return launch_experts<1, DRAMA_B200_F32>(a, s);
    }
}

cudaError_t decode_launch(const DecodeArgs& a, cudaStream_t s) {
    switch (a.format * 8 + a.x_dtype) {
        case 0 * 8 + DRAMA_B200_BF16: return launch_decode<0, DRAMA_B200_BF16>(a, s);
        case 0 * 8 + DRAMA_B200_F16: return launch_decode<0, DRAMA_B200_F16>(a, s);
        case 0 * 8 + DRAMA_B200_F32: return launch_decode<0, DRAMA_B200_F32>(a, s);
        case 1 * 8 + DRAMA_B200_BF16: return launch_decode<1, DRAMA_B200_BF16>(a, s);
        case 1 * 8 + DRAMA_B200_F16: return launch_decode<1, DRAMA_B200_F16>(a, s);
        default: return launch_decode<1, DRAMA_B200_F32>(a, s);
    }
}

}  // namespace drama
