// Shared expert + sigmoid gate, fused with the routed combine and the residual
// (src/drama_low_vram/backbone_graph.py:327-337):
//   shared = sigmoid(x @ g^T) * shared_expert(x)          (_shared_impl)
//   out    = after_mixer + (routed + shared)               (_post_impl)
// with the rounding points of the reference's bf16 torch modules:
//   gate, up = bf16(x @ Wg^T), bf16(x @ Wu^T);  h = bf16(bf16(silu(gate)) * up)
//   d = bf16(h @ Wd^T);  s = bf16(sigmoid(bf16(x @ g^T)));  shared = bf16(s * d)
//   t = bf16(routed + shared);  out = bf16(after_mixer + t)
// (routed and after_mixer are optional; without them out = shared or t.)
//
// One bfloat16 row at hidden 2048, intermediate 768 runs as one launch
// (shared_layer.cu). Otherwise:
// Launches (chained by programmatic dependent launch): the gate/up GEMV, whose
// epilogue forms the SwiGLU rows and (one extra cell per token group) the
// sigmoid gate scalars, then the down GEMV, whose epilogue applies the gate,
// the routed sum and the residual. The GEMVs stream
// the dense bf16 weights once per group of <= 8 tokens through
// mma.m16n8k16 bf16 fragments (tokens as N). When the tiles alone would leave
// the GPU idle (batch 1) a CTA of up to 16 warps shares one tile, each warp a
// part of K, and warp 0 adds the fp32 parts in warp order from shared memory,
// so results do not depend on timing.
#include "common.cuh"
#include "grouped.cuh"
#include "kernels.h"

namespace drama {
namespace {

constexpr int kShThreads = 128;
constexpr int kShTarget = 4736;  // 148 SMs x 32 warps: the split-K target
constexpr int kShTok = 8;        // tokens per MMA N tile

struct ShGemvArgs {
    const __nv_bfloat16* w0;  // gate_proj [I][H] (up) or down_proj [H][I] (down)
    const __nv_bfloat16* w1;  // up_proj [I][H] (up) or NULL
    const __nv_bfloat16* gate_weight;  // up: the [H] shared_expert_gate row
    int64_t w0_row, w1_row;   // elements
    int n, k;                 // output rows (I for up: SwiGLU rows; H for down), contraction length
    const __nv_bfloat16* act; // [T][k]
    int64_t tokens;
    int ksplit;               // warps per CTA sharing one cell (K parts), 1: one cell per warp
    // epilogue
    __nv_bfloat16* h;         // up: [T][I] SwiGLU rows
    float* gate_s;            // up writes, down reads: [T] bf16-rounded sigmoid gate
    const __nv_bfloat16* routed;    // down: [T][H] or NULL
    const __nv_bfloat16* residual;  // down: [T][H] or NULL
    __nv_bfloat16* out;       // down: [T][H]
};

// Up (GLU): a cell's 16 MMA rows are gate rows 8j..8j+7 and up rows 8j..8j+7,
// so a thread holds gate and up of the same row and the epilogue forms
// bf16(bf16(silu(gate)) * up) itself; one extra cell per token group (tile
// I/8) multiplies the gate vector and writes the sigmoid gate scalars.
// Down: a cell is one 16-row tile of H; its epilogue applies the gate, the
// routed sum and the residual.
template <bool DOWN>
__global__ void __launch_bounds__(512) shared_gemv_kernel(ShGemvArgs a) {
    constexpr bool GLU = !DOWN;
    grid_launch_dependents();  // programmatic dependent launch
    grid_dependency_wait();
    __shared__ float4 s_part[16][32];
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, warp = threadIdx.x >> 5;
    const int tiles = GLU ? a.n / 8 + 1 : a.n / 16;
    const int tgroups = static_cast<int>((a.tokens + kShTok - 1) / kShTok);
    const int spans_per = a.k / 32 / a.ksplit;  // 32-column spans
    const uint64_t pol = policy_evict_first();
    // a.ksplit > 1: the CTA's a.ksplit warps share one cell (warp = K part) and add their fp32 sums in warp
    // order through shared memory; a.ksplit == 1: every warp owns whole cells
    const bool team = a.ksplit > 1;
    const int first = team ? blockIdx.x : blockIdx.x * (blockDim.x >> 5) + warp;
    const int step = team ? gridDim.x : gridDim.x * (blockDim.x >> 5);
    for (int cell = first; cell < tgroups * tiles; cell += step) {
        const int kpart = team ? warp : 0;
        const int tg = cell / tiles, tile = cell - tg * tiles;
        const bool gate_cell = GLU && tile == a.n / 8;
        const int64_t tok = static_cast<int64_t>(tg) * kShTok + g;
        const __nv_bfloat16* xrow = tok < a.tokens ? a.act + tok * a.k : nullptr;
        // MMA rows g and g + 8 of this thread
        const int row = GLU ? tile * 8 + g : tile * 16 + g;
        const __nv_bfloat16* w0 = gate_cell ? a.gate_weight : a.w0 + row * a.w0_row;
        const __nv_bfloat16* w1 = gate_cell ? a.gate_weight : GLU ? a.w1 + row * a.w1_row : a.w0 + (row + 8) * a.w0_row;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int sp0 = kpart * spans_per;
        for (int sp = sp0; sp < sp0 + spans_per; sp += 4) {
            uint4 q0[4], q1[4], xb[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int col = (sp + u) * 32 + 8 * t;
                q0[u] = ld_stream_v4(w0 + col, pol);
                q1[u] = ld_stream_v4(w1 + col, pol);
                xb[u] = xrow ? __ldg(reinterpret_cast<const uint4*>(xrow + col)) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                // columns 8t..8t+7 of the span: (0,1)+(2,3) feed the first k16 MMA, (4,5)+(6,7) the second
                const uint32_t a1[4] = {q0[u].x, q1[u].x, q0[u].y, q1[u].y};
                const uint32_t a2[4] = {q0[u].z, q1[u].z, q0[u].w, q1[u].w};
                mma_bf16_16816(acc, a1, xb[u].x, xb[u].y);
                mma_bf16_16816(acc, a2, xb[u].z, xb[u].w);
            }
        }
        if (team) {
            s_part[warp][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            __syncthreads();
            if (warp == 0) {
                acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
                for (int q = 0; q < a.ksplit; ++q) {  // warp (= K) order: the sum does not depend on timing
                    const float4 v = s_part[q][lane];
                    acc[0] += v.x;
                    acc[1] += v.y;
                    acc[2] += v.z;
                    acc[3] += v.w;
                }
            }
        }
        if (!team || warp == 0) {
            // acc[0..1]: MMA row g, tokens 2t, 2t+1 of the group; acc[2..3]: MMA row g + 8
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int64_t tk = static_cast<int64_t>(tg) * kShTok + 2 * t + c;
                if (tk >= a.tokens) continue;
                const float v0 = __bfloat162float(__float2bfloat16_rn(acc[c]));      // F.linear in bf16
                const float v1 = __bfloat162float(__float2bfloat16_rn(acc[2 + c]));
                if constexpr (GLU) {
                    if (gate_cell) {  // every MMA row holds x . g; row 0 writes the gate scalars
                        if (g == 0) a.gate_s[tk] = __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-v0))));
                    } else {          // gate row `row` and up row `row`
                        const float act = __bfloat162float(__float2bfloat16_rn(v0 / (1.0f + expf(-v0))));
                        a.h[tk * a.n + row] = __float2bfloat16_rn(act * v1);
                    }
                } else {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int64_t o = tk * a.n + row + 8 * hh;
                        float y = __bfloat162float(__float2bfloat16_rn(a.gate_s[tk] * (hh ? v1 : v0)));
                        if (a.routed) y = __bfloat162float(__float2bfloat16_rn(__bfloat162float(a.routed[o]) + y));
                        if (a.residual) y = __bfloat162float(a.residual[o]) + y;
                        a.out[o] = __float2bfloat16_rn(y);
                    }
                }
            }
        }
        if (team) __syncthreads();  // s_part is reused by the next cell
    }
}

// K parts per tile: as many as keep the warps within the target, each part a
// whole number of 4-span load batches (one round trip per batch).
int sh_split(int64_t cells, int spans) {
    for (int ks = spans / 4 < 16 ? spans / 4 : 16; ks > 1; --ks)
        if (cells * ks <= kShTarget && spans % (ks * 4) == 0) return ks;
    return 1;
}

}  // namespace

size_t shared_expert_workspace_layout(int64_t tokens, int hidden, int inter, char* base, SharedWorkspace* ws) {
    size_t off = 0;
    auto take = [&](size_t bytes) -> char* {
        char* p = base ? base + off : nullptr;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return p;
    };
    SharedWorkspace w{};
    // The control words come first for every token count, so that no other
    // layout of the same buffer ever writes over the zeroed tickets.
    char* control = take(256);
    w.tickets = reinterpret_cast<int32_t*>(control);
    w.status = control ? reinterpret_cast<int32_t*>(control + 64) : nullptr;  // after up to 16 tickets
    w.h = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(tokens) * inter * 2));
    w.gate_s = reinterpret_cast<float*>(take(tokens * 4));
    if (tokens == 1) w.part = reinterpret_cast<float*>(take(static_cast<size_t>(inter / 32) * hidden * 4));
    if (ws) *ws = w;
    return off;
}

cudaError_t shared_expert_launch(const DramaB200SharedExpert& m, const void* x, int64_t tokens, const void* routed,
                                 const void* residual, void* out, const SharedWorkspace& ws, int sm_count,
                                 cudaStream_t s) {
    if (ws.part && shared_layer_supported(m, tokens))  // one row of the reference's shape: one launch
        return shared_layer_launch(m, x, routed, residual, out, ws.part, ws.tickets, ws.status, s);
    const int H = m.hidden, I = m.intermediate;
    const int64_t tg = (tokens + kShTok - 1) / kShTok;
    // split tiles: one CTA of ks warps per cell; otherwise four single-warp cells per CTA
    auto cta_threads = [](int ks) { return ks > 1 ? 32 * ks : kShThreads; };
    auto grid_cells = [&](int64_t cells, int ks) {
        const int per_cta = ks > 1 ? 1 : kShThreads / 32;
        const int64_t ctas = (cells + per_cta - 1) / per_cta;
        const int64_t cap = static_cast<int64_t>(sm_count) * (ks > 1 ? (32 + ks - 1) / ks : 16);
        return static_cast<unsigned>(ctas < 1 ? 1 : (ctas > cap ? cap : ctas));
    };
    ShGemvArgs up{};
    up.w0 = static_cast<const __nv_bfloat16*>(m.gate_proj);
    up.w1 = static_cast<const __nv_bfloat16*>(m.up_proj);
    up.gate_weight = static_cast<const __nv_bfloat16*>(m.gate_weight);
    up.w0_row = m.gate_row_stride;
    up.w1_row = m.up_row_stride;
    up.n = I;
    up.k = H;
    up.act = static_cast<const __nv_bfloat16*>(x);
    up.tokens = tokens;
    const int64_t up_cells = tg * (I / 8 + 1);  // + the gate-scalar cell of each token group
    up.ksplit = sh_split(up_cells, H / 32);
    up.h = ws.h;
    up.gate_s = ws.gate_s;
    cudaError_t err = launch_pdl(shared_gemv_kernel<false>, dim3(grid_cells(up_cells, up.ksplit)),
                                 dim3(cta_threads(up.ksplit)), 0, s, up);
    if (err != cudaSuccess) return err;
    ShGemvArgs dn{};
    dn.w0 = static_cast<const __nv_bfloat16*>(m.down_proj);
    dn.w1 = nullptr;
    dn.w0_row = m.down_row_stride;
    dn.n = H;
    dn.k = I;
    dn.act = ws.h;
    dn.tokens = tokens;
    dn.ksplit = sh_split(tg * (H / 16), I / 32);
    dn.gate_s = ws.gate_s;
    dn.routed = static_cast<const __nv_bfloat16*>(routed);
    dn.residual = static_cast<const __nv_bfloat16*>(residual);
    dn.out = static_cast<__nv_bfloat16*>(out);
    return launch_pdl(shared_gemv_kernel<true>, dim3(grid_cells(tg * (H / 16), dn.ksplit)),
                      dim3(cta_threads(dn.ksplit)), 0, s, dn);
}

}  // namespace drama
