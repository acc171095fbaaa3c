// Internal kernel entry points and argument blocks (host side of the ABI).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "drama_b200.h"

namespace drama {

// Launch with programmatic stream serialisation: the kernel may start while
// its predecessor drains and calls griddepcontrol.wait before reading inputs.
template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

struct RouteArgs {
    const void* logits;
    int logits_dtype;
    int64_t tokens;
    int experts;
    int top_k;
    int renormalize;
    void* ids;
    int ids_dtype;
    void* weights;
    int weights_dtype;
};
cudaError_t route_topk(const RouteArgs& a, cudaStream_t s);

struct PermuteArgs {
    const void* ids;
    int ids_dtype;
    int64_t pairs;
    int experts;
    int64_t* order;
    int64_t* counts;
    int64_t* offsets;
    int32_t* status;
};
cudaError_t permute_routes(const PermuteArgs& a, cudaStream_t s);
size_t bucket_smem_bytes(int experts);
// The same permutation over many CTAs (experts <= 1024), for many pairs:
// chunk_counts is scratch of permute_wide_scratch_bytes; position[p] (when
// given) receives pair p's sorted position, -1 for a dropped pair.
size_t permute_wide_scratch_bytes(int64_t pairs, int experts);
cudaError_t permute_routes_wide(const PermuteArgs& a, int* chunk_counts, int64_t* position, cudaStream_t s);

// ---------------------------------------------------------------------------
// Decode (K1) workspace carved out of one caller buffer.
// ---------------------------------------------------------------------------
constexpr int kDecodeMaxWarps = 16;      // upper bound on warps per CTA of the GEMV kernels
constexpr int kDecodeCtasPerSm = 1;      // resident CTAs per SM
constexpr int kGroupTokens = 8;          // tokens per expert group (one n8 MMA)
constexpr int kMaxDecodePairs = 4096;
constexpr int64_t kMaxPrefillPairs = int64_t(1) << 24;  // sorted-row coordinates stay in int32
constexpr int kStageTokens = 8;          // token rows staged in shared memory by the up kernel
constexpr int kStageGroups = 4;          // expert groups staged in shared memory by the down kernel
constexpr int kMaxSlots = 1024;

struct DecodeWorkspace {
    int32_t* status;      // [4]
    int32_t* num_groups;  // [1]
    int32_t* order;       // [P]   pairs sorted by slot (stable)
    int4* g_rec;          // [P][2] group records: {slot, start, count, 0}, 8 x u16 pair indices
    float* xscale;        // [T]   2^e per token row
    uint16_t* x16;        // [T][H] f16 copy of x * 2^-e (layout per format)
    float* wts;           // [P]   route weights as fp32
    void* h;              // [P][I] SwiGLU activations in x's dtype
    float* pair_out;      // [P][H] weighted fp32 partials (when the caller gives none)
    float* up_part;       // [Wu][2][32][8]
    int32_t* up_cnt;      // [P * I/16]
    float* dn_part;       // [Wd][2][32][4]
    int32_t* dn_cnt;      // [P * H/16]
    int32_t* cmb_cnt;     // [H/16]
    float* logits;        // [T][E] router logits (MoE layer entry point only)
    int32_t* router_cnt;  // [1]
    float* layer_part;    // [SMs][H] partial down projections of the one-launch layer (MoE layer only)
    int32_t* layer_tickets;  // [16] its arrival tickets, reset by the last arriver
};

// The split-K and combine counters of one call: zeroed by whichever kernel
// builds the expert groups, before the expert kernels run.
#ifdef __CUDACC__
// Group record g: rec[2g] = {slot, first sorted position, pair count, 0};
// rec[2g+1] = pair index (token * top_k + route slot) of each of the (<= 8)
// pairs, two u16 per word.
__device__ __forceinline__ void write_group(const DecodeWorkspace& ws, int g, int slot, int start, int count,
                                            const int* pairs) {
    uint32_t t[4] = {0u, 0u, 0u, 0u};
    for (int c = 0; c < count; ++c) t[c >> 1] |= static_cast<uint32_t>(pairs[c] & 0xffff) << (16 * (c & 1));
    ws.g_rec[2 * g] = make_int4(slot, start, count, 0);
    ws.g_rec[2 * g + 1] = make_int4(static_cast<int>(t[0]), static_cast<int>(t[1]), static_cast<int>(t[2]),
                                    static_cast<int>(t[3]));
}
__device__ __forceinline__ void zero_split_counters(const DecodeWorkspace& ws, int groups, int hidden,
                                                    int intermediate, int tid, int threads) {
    const int up = groups * (intermediate / 16), dn = groups * (hidden / 16);
    for (int i = tid; i < up; i += threads) ws.up_cnt[i] = 0;
    for (int i = tid; i < dn; i += threads) ws.dn_cnt[i] = 0;
    for (int i = tid; i < hidden / 16; i += threads) ws.cmb_cnt[i] = 0;
}
#endif

// experts > 0 adds the router scratch used by the fused MoE layer.
size_t decode_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate,
                               int sm_count, int experts, char* base, DecodeWorkspace* ws);

struct DecodeArgs {
    int format;  // 0 = FP8 block-scaled, 1 = INT4 group-128
    DramaB200Fp8Bank fp8;
    DramaB200Int4Bank int4;
    const void* x;
    int x_dtype;
    int64_t tokens;
    int top_k;
    const void* ids;
    int ids_dtype;
    const void* weights;
    int weights_dtype;
    void* out;
    float* pair_out;
    const void* residual;  // optional [T][H] added before the final rounding
    void* moe_out;         // optional [T][H] combined expert output before the residual
    DecodeWorkspace ws;
    int hidden, intermediate, slots;
    int ctas;  // one CTA per SM
};

cudaError_t decode_launch(const DecodeArgs& a, cudaStream_t s);          // prep + up + down
cudaError_t decode_experts_launch(const DecodeArgs& a, cudaStream_t s);  // up + down

constexpr int kMaxLayerPairs = 256;
constexpr int kRouterCtas = 16;

struct MoeLayerArgs {
    const __nv_bfloat16* hidden_in;
    __nv_bfloat16* hidden_out;
    const float* gamma;
    const __nv_bfloat16* gate;
    const __nv_bfloat16* next_gate;
    float eps;
    int64_t tokens;
    int experts, top_k, hidden, intermediate;
    DecodeWorkspace ws;
    int64_t* ids_out;
    __nv_bfloat16* weights_out;
    __nv_bfloat16* normed_out;
    int router_ctas;
};
cudaError_t moe_router_launch(const MoeLayerArgs& m, cudaStream_t s);

// ---------------------------------------------------------------------------
// Prefill (K2, prefill_gemm.cu): permute + grouped tensor-core GEMMs + combine.
// ---------------------------------------------------------------------------
struct PrefillWorkspace {
    int32_t* status;          // [4]: [0] pairs dropped for an out-of-range id
    int64_t* order;           // [P] pairs sorted by expert (stable)
    int64_t* counts;          // [E]
    int64_t* offsets;         // [E + 1]
    __nv_bfloat16* h;         // [P][I] SwiGLU activations in sorted order
    __nv_bfloat16* down;      // [P][H] bf16 down projections by pair
};
// Per-row bf16 down projections on the swap-AB grouped GEMMs (expert_rows.cu).
struct RowsWorkspace {
    int32_t* status;          // [4]: [0] rows dropped for an out-of-range id
    int64_t* order;           // [rows] sorted by expert (stable)
    int64_t* counts;          // [E]
    int64_t* offsets;         // [E + 1]
    __half* xh;               // [rows][H] f16 copies scaled per 64 columns
    float* xs;                // [rows][H / 64] their scales (powers of two)
    __half* h;                // [rows][I] SwiGLU activations, sorted, f16 scaled per 64 columns
    float* hs;                // [rows][I / 64]
    int32_t* ids;             // [rows] expert ids taken from tagged rows
};
size_t expert_rows_workspace_layout(int64_t rows, int hidden, int intermediate, int experts, char* base,
                                    RowsWorkspace* ws);
// GEMM 1 rows written to other ranks: received row r (from rank r / cap) goes
// to dst[r / cap] + (rank * cap + r % cap) * H.
// After the last CTA of GEMM 1: signals[d][2 * ranks + rank] = *epoch for every d.
struct RowsScatter {
    int ranks = 0;            // 0: no scatter
    int rank = 0;
    int64_t cap = 0;
    __nv_bfloat16* dst[8] = {};
    int32_t* signals[8] = {};
    int32_t* done = nullptr;
    const int32_t* epoch = nullptr;
};
// Rows written by other ranks into blocks of `cap`: wait for signals[0, ranks)
// == *epoch; rows of block s past signals[ranks + s] get id `unused`.
struct RowsReceive {
    const int32_t* signals = nullptr;  // null: plain rows
    const int32_t* epoch = nullptr;
    int ranks = 0;
    int64_t cap = 0;
    int unused = 0;
    int32_t* status = nullptr;
    int64_t wait_ns = 0;               // limit of the flag wait; 0: the default (2 s)
};
cudaError_t expert_rows_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t x_stride, int64_t rows,
                               const void* ids, int ids_dtype, void* out, const RowsWorkspace& ws, int sm_count,
                               cudaStream_t s, const RowsScatter* scatter = nullptr,
                               const RowsReceive* receive = nullptr);

// Expert-parallel exchange (expert_parallel.cu).
constexpr int kMaxEpRanks = 8;
cudaError_t ep_dispatch_launch(const void* hidden, int64_t tokens, int H, const void* ids, int ids_dtype, int top_k,
                               int experts, int ranks, const int32_t* placement, int64_t cap, void* send_rows,
                               int64_t row_stride, int32_t* send_ids, int32_t* pair_rows, int32_t* status,
                               int sm_count, cudaStream_t s);
cudaError_t ep_combine_launch(const void* rows, int64_t row_count, const int32_t* pair_rows, const void* weights,
                              int weights_dtype, int64_t tokens, int top_k, int H, const void* residual, void* out,
                              int sm_count, cudaStream_t s, const int32_t* wait_flags = nullptr,
                              const int32_t* wait_epoch = nullptr, int wait_ranks = 0, int32_t* status = nullptr,
                              int64_t wait_ns = 0);

// Expert-parallel exchange over peer memory (ep_p2p.cu).
constexpr int kP2pMaxPairs = 4096;  // (token, slot) pairs per rank and layer of the fused peer dispatch
cudaError_t ep_p2p_dispatch_launch(const DramaB200EpPeers& peers, const void* hidden, int64_t tokens,
                                   const void* ids, int ids_dtype, int top_k, const int32_t* placement,
                                   int32_t* pair_rows, int32_t* status, int sm_count, cudaStream_t s);

// W8A8 modes 1-3 (w8a8_decode.cu): ConvRot-rotated INT8 activations times
// INT8 / 6-bit / 4-bit-codebook weights on int8 tensor cores.
struct W8a8Workspace {
    int32_t* status;          // [4]: [0] pairs dropped for an out-of-range slot
    int32_t* num_groups;      // [1]
    int32_t* order;           // [P] pairs sorted by slot (stable)
    int4* g_rec;              // [P][2] group records (write_group layout)
    int8_t* xq;               // [T][H] rotated, quantised token rows
    float* xs;                // [T]
    __nv_bfloat16* up;        // [P][I] SwiGLU rows (bf16); INT4 decode: [P][2I] gate/up
    int8_t* hq;               // [P][I] rotated, quantised SwiGLU rows
    float* hs;                // [P]
    float* wts;               // [P] route weights as fp32
    float* pair_out;          // [P][H] weighted fp32 partials
    int32_t* cmb_cnt;         // [H/16] finished down cells per row tile (zeroed by prep)
    float* layer_part;        // one row (tokens == 1): [kMaxLayerUnits][H] partial down projections
    int32_t* layer_tickets;   // one row: [4] arrivals per quarter of H, zero between calls (in the status chunk)
};
size_t w8a8_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, char* base,
                             W8a8Workspace* ws);
// Units (route slot, part of the intermediate dimension) of a one-launch layer.
constexpr int kMaxLayerUnits = 32;
// GPTQ W4A16 for one bf16 decode row in one launch (int4_layer.cu): the
// reference's shape (hidden 2048, intermediate 768, top-8) when the device
// fits its 32 clusters of 4 CTAs; scratch: layer_part and layer_tickets.
bool int4_layer_supported(int64_t tokens, int top_k, const DramaB200Int4Bank& b, int x_dtype);
cudaError_t int4_layer_launch(const DramaB200Int4Bank& b, const void* x, const void* ids, int ids_dtype,
                              const void* weights, int weights_dtype, void* out, int out_dtype, float* pair_out,
                              float* part, int32_t* tickets, int32_t* status, cudaStream_t s);
// GPTQ W4A16 on the same schedule (bf16 hidden rows; scratch from w8a8_workspace_layout).
cudaError_t int4_rows_launch(const DramaB200Int4Bank& bank, const void* x, int64_t tokens, int top_k,
                             const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                             int out_dtype, float* pair_out, const W8a8Workspace& ws, int sm_count, cudaStream_t s);
cudaError_t w8a8_decode_launch(const DramaB200W8a8Bank& bank, const void* x, int64_t tokens, int top_k,
                               const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                               int out_dtype, float* pair_out, const W8a8Workspace& ws, int sm_count,
                               cudaStream_t s);

// The official FP8 W8A8 contract (fp8_w8a8.cu): 1x128 E4M3 activations,
// E4M3 tensor-core block dots, bf16 gate/up, requantised SwiGLU rows.
struct Fp8W8a8Workspace {
    int32_t* status;    // [4]: [0] pairs with an out-of-range id
    uint8_t* xq;        // [T][H] E4M3 token rows
    float* xs;          // [T][H/128]
    float* h;           // [P][I] SwiGLU rows (fp32)
    uint8_t* hq;        // [P][I] E4M3
    float* hs;          // [P][I/128]
    float* pair_out;    // [P][H] weighted fp32 partials
};
size_t fp8_w8a8_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, char* base,
                                 Fp8W8a8Workspace* ws);

// The driver's cuTensorMapEncodeTiled (null when the driver lacks it).
using TensorMapEncode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
TensorMapEncode tensor_map_encoder();

// The FP8 W8A8 contract for many rows on tcgen05 tensor cores
// (fp8_prefill_tc.cu): permute, sorted-row quantisation, gate/up and down
// grouped GEMMs, slot combine.
struct Fp8PrefillWorkspace {
    int32_t* status;    // [4]: [0] pairs with an out-of-range id, [1] a GEMM wait timed out
    int64_t* order;     // [P] pairs sorted by expert
    int64_t* counts;    // [E]
    int64_t* offsets;   // [E + 1]
    int64_t* position;  // [P] sorted position of each pair (-1: dropped)
    float* sorted_w;    // [P] each pair's route weight (fp32) at its sorted position
    int* chunk_counts;  // permutation scratch
    uint8_t* xq;        // [P + 128][H] E4M3 token rows in sorted order
    float* xs;          // [P + 128][H/128]
    uint8_t* hq;        // [P + 128][I] E4M3 SwiGLU rows in sorted order
    float* hs;          // [P + 128][I/128]
    float* pair_out;    // [P][H] weighted fp32 partials
};
bool fp8_prefill_tc_supported(int hidden, int intermediate, int experts);
size_t fp8_prefill_tc_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, int experts,
                                       char* base, Fp8PrefillWorkspace* ws);
cudaError_t fp8_prefill_tc_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t tokens, int top_k,
                                  const void* ids, int ids_dtype, const void* weights, int weights_dtype, void* out,
                                  float* pair_out, const Fp8PrefillWorkspace& ws, int sm_count, cudaStream_t s);
cudaError_t fp8_w8a8_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t tokens, int top_k, const void* ids,
                            int ids_dtype, const void* weights, int weights_dtype, void* out, float* pair_out,
                            const Fp8W8a8Workspace& ws, cudaStream_t s);

// Shared expert + gate fused with the routed combine (shared_expert.cu).
constexpr int kMaxSharedTokens = 4096;
struct SharedWorkspace {
    int32_t* tickets;         // [<= 16] the one-launch layer's arrivals per row share (zero between calls)
    int32_t* status;          // [4] [1] waits that ran out
    __nv_bfloat16* h;         // [T][I] SwiGLU rows
    float* gate_s;            // [T] bf16-rounded sigmoid gate
    float* part;              // T == 1: [I / 32][H] the one-launch layer's partial down projections
};
size_t shared_expert_workspace_layout(int64_t tokens, int hidden, int inter, char* base, SharedWorkspace* ws);
// One bfloat16 row at hidden 2048, intermediate 768: the whole shared expert
// and its combine in one launch (shared_layer.cu).
bool shared_layer_supported(const DramaB200SharedExpert& m, int64_t tokens);
cudaError_t shared_layer_launch(const DramaB200SharedExpert& m, const void* x, const void* routed,
                                const void* residual, void* out, float* part, int32_t* tickets, int32_t* status,
                                cudaStream_t s);
cudaError_t shared_expert_launch(const DramaB200SharedExpert& m, const void* x, int64_t tokens, const void* routed,
                                 const void* residual, void* out, const SharedWorkspace& ws, int sm_count,
                                 cudaStream_t s);

size_t prefill_workspace_layout(int64_t tokens, int top_k, int hidden, int intermediate, int experts, char* base,
                                PrefillWorkspace* ws);
cudaError_t prefill_launch(const DramaB200Fp8Bank& bank, const void* x, int64_t tokens, int top_k, const void* ids,
                           int ids_dtype, const void* weights, int weights_dtype, void* out,
                           const PrefillWorkspace& ws, int sm_count, cudaStream_t s);

// ---------------------------------------------------------------------------
// Single-row MoE layer in two launches (routed_layer.cu): router + gate/up in
// thread-block clusters, then down + combine + residual per hidden tile.
// ---------------------------------------------------------------------------
constexpr int kRoutedMaxTopK = 16;

struct RoutedLayerArgs {
    DramaB200Fp8Bank bank;
    const __nv_bfloat16* hidden_in;
    __nv_bfloat16* hidden_out;
    const float* gamma;
    const __nv_bfloat16* gate;
    float eps;
    int E, k, H, I;
    DecodeWorkspace ws;  // uses order[0..k) (expert ids), wts[0..k), h
    int64_t* ids_out;
    __nv_bfloat16* weights_out;
    __nv_bfloat16* normed_out;
    __nv_bfloat16* moe_out;
};
bool routed_layer_supported(int64_t tokens, int top_k, int hidden, int intermediate, int experts);
cudaError_t routed_layer_launch(const RoutedLayerArgs& a, int sm_count, cudaStream_t s);

// ---------------------------------------------------------------------------
// Single-row MoE layer in ONE launch (decode_layer.cu): 4-CTA clusters, each
// owning a run of one routed expert's intermediate tiles; gate/up rows by
// bulk copies into a shared-memory ring, the down projection per run, and
// the slot-ordered combine by the last CTA to arrive.
// ---------------------------------------------------------------------------
struct DecodeLayerArgs {
    CUtensorMap w13_map;                 // the bank's gate/up rows as [slot][gate|up][row][K block][128 B]
    CUtensorMap w2_map;                  // the bank's down rows as [slot][row][I bytes]
    RoutedLayerArgs layer;               // uses ws.status[3] (a bounded wait timed out)
    const __nv_bfloat16* normed_in;      // with logits_in: the caller's normalised row, bf16 [H]
    const __nv_bfloat16* logits_in;      // null: RMSNorm and router GEMV inside the kernel
    float* part;                         // [units][H] fp32 partial down projections
    int32_t* tickets;                    // [4] arrival tickets, reset by the last arriver
    int parts, nkt, stages, overlay;     // set by decode_layer_launch (with w13_map)
};
bool decode_layer_supported(int64_t tokens, int top_k, int hidden, int intermediate, int experts);
cudaError_t decode_layer_launch(DecodeLayerArgs a, cudaStream_t s);

}  // namespace drama
