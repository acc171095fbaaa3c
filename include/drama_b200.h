/* drama_b200 — B200 (sm_100a) routed-expert hot path behind a plain C ABI.
 *
 * Conventions (mirroring the reference's native ABI v1,
 * native/include/drama_native.h:1-90 and native/src/runtime.cpp:278-290):
 *   - every entry point returns 0 on success, -1 on failure; the failure text
 *     is available from drama_b200_error() on the same host thread;
 *   - all validation happens before any launch or write;
 *   - buffers are borrowed device pointers (plain pointers, sizes, strides in
 *     elements); nothing is retained after return;
 *   - work is enqueued on the caller's CUDA stream (a cudaStream_t passed as
 *     void*); no entry point allocates, synchronises or blocks, so every call
 *     can be captured in a CUDA graph;
 *   - kernels that need scratch take a caller-owned device workspace sized by
 *     the matching *_workspace_bytes() query. The workspace must be zero-filled
 *     once before its first use; every call leaves it reusable. Calls that
 *     share one workspace must be ordered on the GPU (same stream or events).
 */
#ifndef DRAMA_B200_H
#define DRAMA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DRAMA_B200_API __attribute__((visibility("default")))
#else
#define DRAMA_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DRAMA_B200_ABI_VERSION 1

/* Element type codes used by every dtype argument. */
enum {
    DRAMA_B200_F32 = 0,
    DRAMA_B200_F16 = 1,
    DRAMA_B200_BF16 = 2,
    DRAMA_B200_I32 = 3,
    DRAMA_B200_I64 = 4
};

/* ABI version (DRAMA_B200_ABI_VERSION). Replaces drama_native_abi
 * (native/include/drama_native.h:15). */
DRAMA_B200_API int drama_b200_abi(void);

/* Thread-local text of the last failure. Replaces drama_native_error
 * (native/include/drama_native.h:18). */
DRAMA_B200_API const char* drama_b200_error(void);

/* 0 when `device` is an sm_100 GPU this library was built for; -1 otherwise.
 * Replaces the capability gate of nvidia_policy.policy_for
 * (src/drama_low_vram/nvidia_policy.py:21-33). */
DRAMA_B200_API int drama_b200_device_check(int device, int* sm_count);

/* ---------------------------------------------------------------------------
 * K3 router: softmax -> top-k -> optional renormalisation -> cast.
 * Replaces BackboneDecodeGraph._route_impl's routing lines
 * (src/drama_low_vram/backbone_graph.py:319-323):
 *   probs = softmax(logits.float()); w, ids = probs.topk(k);
 *   if renormalize: w /= w.sum(-1); w = w.to(weights_dtype)
 * logits: [tokens, experts] (F32/F16/BF16), experts <= 1024, 1 <= top_k <= 32.
 * ids: [tokens, top_k] (I32/I64); weights: [tokens, top_k] (F32/F16/BF16).
 * Indices and their order reproduce torch's CUDA topk, ties included.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API int drama_b200_route_topk(const void* logits, int logits_dtype, int64_t tokens,
                                         int experts, int top_k, int renormalize, void* ids,
                                         int ids_dtype, void* weights, int weights_dtype,
                                         void* stream);

/* K3 gather/permute: stable argsort of flat route IDs, per-expert counts and
 * start offsets. Replaces ExpertOffloadManager._forward_partitioned's host
 * routing (src/drama_low_vram/offload.py:1206-1211):
 *   order = argsort(flat_ids, stable=True); counts = bincount(flat_ids, E)
 * ids: [pairs] (I32/I64) in [0, experts); experts <= 1024; pairs <= 2^24.
 * order: [pairs] int64; counts: [experts] int64; offsets: [experts+1] int64.
 * An ID outside [0, experts) makes the call fail before any launch only when
 * it is detectable on the host; on the device such pairs are dropped from the
 * order and counted in status[0] (int32, may be NULL). */
DRAMA_B200_API int drama_b200_permute_routes(const void* ids, int ids_dtype, int64_t pairs,
                                             int experts, int64_t* order, int64_t* counts,
                                             int64_t* offsets, int32_t* status, void* stream);

/* The same permutation over many CTAs, for many pairs (the single-CTA form
 * above serves decode-sized calls): the same order, counts and offsets, and
 * position[p] = the sorted position of pair p (-1 for a dropped pair; may be
 * NULL). scratch: drama_b200_permute_routes_wide_scratch_bytes bytes of
 * device memory, 16-byte aligned. status[0] is written (not accumulated). */
DRAMA_B200_API size_t drama_b200_permute_routes_wide_scratch_bytes(int64_t pairs, int experts);

DRAMA_B200_API int drama_b200_permute_routes_wide(const void* ids, int ids_dtype, int64_t pairs, int experts,
                                                  int64_t* order, int64_t* counts, int64_t* offsets,
                                                  int64_t* position, void* scratch, size_t scratch_bytes,
                                                  int32_t* status, void* stream);

/* ---------------------------------------------------------------------------
 * Expert banks. Layouts are the reference's staged views: ExpertStore /
 * StagedExperts (src/drama_low_vram/offload.py:101-184) for FP8 and
 * QuantizedStore mode 0 (src/drama_low_vram/quantized_model.py:26-68) for
 * INT4. Strides are in elements; the innermost dimension is contiguous; every
 * weight row starts on a 16-byte boundary.
 * ------------------------------------------------------------------------- */
typedef struct DramaB200Fp8Bank {
    const void* w13;          /* E4M3 [slots, 2I, H]: gate rows then up rows */
    const float* w13_scale;   /* fp32 [slots, 2I/128, H/128] */
    const void* w2;           /* E4M3 [slots, H, I] */
    const float* w2_scale;    /* fp32 [slots, H/128, I/128] */
    int64_t w13_slot_stride, w13_row_stride;
    int64_t w13_scale_slot_stride, w13_scale_row_stride;
    int64_t w2_slot_stride, w2_row_stride;
    int64_t w2_scale_slot_stride, w2_scale_row_stride;
    int32_t slots, hidden, intermediate, reserved;
} DramaB200Fp8Bank;

typedef struct DramaB200Int4Bank {
    const int32_t* w13;        /* [slots, 2I, H/8]; nibble k%8 at bit 4*(k%8) */
    const void* w13_scale;     /* BF16 or F16 [slots, 2I, H/128] */
    const int32_t* w13_zeros;  /* [slots, 2I/8, H/128], nibble n%8 at bit 4*(n%8); NULL = 8 */
    const int32_t* w2;         /* [slots, H, I/8] */
    const void* w2_scale;      /* BF16 or F16 [slots, H, I/128] */
    const int32_t* w2_zeros;   /* [slots, H/8, I/128]; NULL = 8 */
    int64_t w13_slot_stride, w13_row_stride;
    int64_t w13_scale_slot_stride, w13_scale_row_stride;
    int64_t w13_zeros_slot_stride, w13_zeros_row_stride;
    int64_t w2_slot_stride, w2_row_stride;
    int64_t w2_scale_slot_stride, w2_scale_row_stride;
    int64_t w2_zeros_slot_stride, w2_zeros_row_stride;
    int32_t scale_dtype;       /* DRAMA_B200_BF16 or DRAMA_B200_F16 */
    int32_t slots, hidden, intermediate;
} DramaB200Int4Bank;

/* ---------------------------------------------------------------------------
 * K1 decode: dequantising SwiGLU expert FFN with the weighted combine fused.
 * Replaces ExpertBackend.forward / forward_pairs
 * (src/drama_low_vram/offload.py:187-196) as TorchExpertBackend computes them
 * (offload.py:199-244; the FP8 W16A16 dequant path) and
 * QuantizedExpertBackend(0) (src/drama_low_vram/quantized_kernels.py:217-248):
 *   gate, up = x @ W13^T (rounded to x's dtype); h = silu(gate) * up;
 *   partial[p] = (h @ W2^T rounded to x's dtype) * weight[p]   (fp32)
 *   out[t] = sum over route slots, in slot order, of partial[t*top_k + s]
 * x: [tokens, H] (F32/F16/BF16); ids/weights: [tokens, top_k] local slots and
 * route weights. When top_k == 1 and out == NULL the call is forward_pairs:
 * pair_out [tokens, H] fp32 receives the weighted partials. Either output may
 * be NULL but not both. Weight bytes are read once per (slot, <=8 tokens).
 * pairs = tokens*top_k <= 4096, slots <= 1024.
 * drama_b200_int4_decode with bfloat16 rows and H, I multiples of 256 runs the
 * grouped schedule of the W8A8 entry below, with the weights dequantised per
 * element to bf16 as the reference's kernel does (quantized_kernels.py:139-147:
 * bf16((code - zp) * scale)) and bf16 MMAs; other rows take the f16 path with
 * exact levels and per-block scales.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API size_t drama_b200_decode_workspace_bytes(int64_t tokens, int top_k, int hidden,
                                                        int intermediate);

DRAMA_B200_API int drama_b200_fp8_decode(const DramaB200Fp8Bank* bank, const void* x,
                                         int x_dtype, int64_t tokens, int top_k,
                                         const void* ids, int ids_dtype, const void* weights,
                                         int weights_dtype, void* out, float* pair_out,
                                         void* workspace, size_t workspace_bytes,
                                         void* stream);

/* ---------------------------------------------------------------------------
 * The official FP8 W8A8 decode contract of the reference's production GPU
 * backend (TritonExpertBackend / fp8_decode.forward and quantized_pairs,
 * src/drama_low_vram/fp8_decode.py:114-147, decode_gemm 24-58; CPU statement
 * native/src/runtime.cpp:162-237, fp8_cpu_reference.py:14-52) on the same
 * FP8 bank as drama_b200_fp8_decode:
 *   x -> 1x128 E4M3 blocks, scale = max(amax, 1e-10) * (1/448);
 *   gu = sum over blocks of fma(dot(W13, q) * scale, block scale, acc);
 *   h = (bf16(gate) / (1 + exp(-bf16(gate)))) * bf16(up) -> 1x128 E4M3;
 *   down likewise; partial = down * weight (fp32); out = bf16(slot-order sum).
 * x: bf16 [tokens, H]; out (bf16 [tokens, H]) and/or pair_out (fp32
 * [tokens*top_k, H], forward_pairs) ; x_fp8_out (uint8 [tokens, H]) and
 * x_scale_out (fp32 [tokens, H/128]), when given, receive the quantised token
 * rows. Ids outside [0, slots) contribute zero and are counted in workspace
 * status word 0. H, I multiples of 128; pairs <= 4096.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API size_t drama_b200_fp8_w8a8_workspace_bytes(int64_t tokens, int top_k, int hidden,
                                                          int intermediate);

DRAMA_B200_API int drama_b200_fp8_w8a8_decode(const DramaB200Fp8Bank* bank, const void* x, int64_t tokens,
                                              int top_k, const void* ids, int ids_dtype, const void* weights,
                                              int weights_dtype, void* out, float* pair_out, void* x_fp8_out,
                                              float* x_scale_out, void* workspace, size_t workspace_bytes,
                                              void* stream);

/* ---------------------------------------------------------------------------
 * The same FP8 W8A8 contract for many rows on tcgen05 tensor cores (the
 * prefill regime of TritonExpertBackend.forward / forward_pairs,
 * src/drama_low_vram/offload.py:279-341, whose grouped FP8 GEMM it replaces):
 * pairs bucketed by expert, sorted rows quantised 1x128, gate/up and down
 * grouped GEMMs with 128x128 weight block scales promoted per 128-wide K block,
 * then the slot-ordered combine. Outputs as drama_b200_fp8_w8a8_decode
 * (out and/or pair_out; a pair with an out-of-range id contributes zero and
 * its pair_out row is zero; pair_out 32-byte aligned). hidden a multiple of 256 and <= 2048,
 * intermediate a multiple of 128 and <= 2048, at most 512 experts
 * (drama_b200_fp8_w8a8_prefill_supported); at most 2^24 pairs; bf16 rows; workspace 256-byte
 * aligned, drama_b200_fp8_w8a8_prefill_workspace_bytes bytes.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API int drama_b200_fp8_w8a8_prefill_supported(int hidden, int intermediate, int experts);

DRAMA_B200_API size_t drama_b200_fp8_w8a8_prefill_workspace_bytes(int64_t tokens, int top_k, int hidden,
                                                                  int intermediate, int experts);

DRAMA_B200_API int drama_b200_fp8_w8a8_prefill(const DramaB200Fp8Bank* bank, const void* x, int64_t tokens,
                                               int top_k, const void* ids, int ids_dtype, const void* weights,
                                               int weights_dtype, void* out, float* pair_out, void* workspace,
                                               size_t workspace_bytes, void* stream);

DRAMA_B200_API int drama_b200_int4_decode(const DramaB200Int4Bank* bank, const void* x,
                                          int x_dtype, int64_t tokens, int top_k,
                                          const void* ids, int ids_dtype, const void* weights,
                                          int weights_dtype, void* out, float* pair_out,
                                          void* workspace, size_t workspace_bytes,
                                          void* stream);

/* ---------------------------------------------------------------------------
 * W8A8 expert banks, modes 1-3 of QuantizedExpertBackend(mode)
 * (src/drama_low_vram/quantized_kernels.py:115-189 _quant_gemm, 217-248 the
 * backend; layouts of quantized_model.py:45-68, 114-151):
 *   mode 1 INT8-ConvRot: w [slots, N, K] int8, scale [slots, N, 1] fp32.
 *   mode 2 W6A8: w [slots, N, 3K/4]: K/2 bytes of low nibbles (column 2j in
 *          the low nibble of byte j) then K/4 bytes of top-two bits (column
 *          4j+i at bits 2i of byte j), level = code - 32; scale [slots, N,
 *          K/16 + 4] uint8: an FP8 E4M3 relative scale per 16 columns, then the
 *          fp32 channel scale.
 *   mode 3 W4A8: w [slots, N, K/2] 4-bit codes, level = codebook[code];
 *          scale [slots, N, K/16 + 8]: as mode 2 plus one fp32 codebook entry
 *          in bytes K/16+4..K/16+8 of rows 0..15.
 * Weight grid (modes 2/3) = clamp(rint(level * relative), +-127) in fp32.
 * Strides are in BYTES. W13 rows: N = 2I, K = H; W2 rows: N = H, K = I.
 * ------------------------------------------------------------------------- */
typedef struct DramaB200W8a8Bank {
    int32_t mode;              /* 1, 2 or 3 */
    const void* w13;
    const void* w13_scale;
    const void* w2;
    const void* w2_scale;
    int64_t w13_slot_stride, w13_row_stride;
    int64_t w13_scale_slot_stride, w13_scale_row_stride;
    int64_t w2_slot_stride, w2_row_stride;
    int64_t w2_scale_slot_stride, w2_scale_row_stride;
    int32_t slots, hidden, intermediate;
} DramaB200W8a8Bank;

/* The W8A8 expert FFN, QuantizedExpertBackend(mode).forward / forward_pairs:
 *   r = bf16(x_row @ kron(H4,H4,H4,H4)/16 per 256 columns)   (ConvRot)
 *   q = clamp(rint(r / s), +-127), s = max(amax(r), 1e-12) / 127  (per row)
 *   proj = bf16((float(int32 sum q * grid) * s) * channel)
 *   gate, up = proj(x, W13); h = bf16(bf16(silu(gate)) * up)
 *   partial[p] = float(proj(h, W2)) * weight[p]   (fp32)
 *   out[t] = sum over route slots, in slot order, of partial[t*top_k + s]
 * x: [tokens, H] bfloat16 (the reference's compute dtype on sm_80+); out the
 * same; ids/weights [tokens, top_k]; pair_out as in drama_b200_fp8_decode.
 * The rotation is computed as four radix-4 stages in float64 and rounded once;
 * the integer sums are exact. H and I must be multiples of 256;
 * pairs <= 4096, slots <= 1024. Ids outside [0, slots) contribute zero and are
 * counted in the workspace status word. */
DRAMA_B200_API size_t drama_b200_w8a8_workspace_bytes(int64_t tokens, int top_k, int hidden, int intermediate);

DRAMA_B200_API int drama_b200_w8a8_decode(const DramaB200W8a8Bank* bank, const void* x, int x_dtype,
                                          int64_t tokens, int top_k, const void* ids, int ids_dtype,
                                          const void* weights, int weights_dtype, void* out, float* pair_out,
                                          void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Shared expert + sigmoid gate fused with the routed combine and the residual:
 * BackboneDecodeGraph._shared_impl and _post_impl
 * (src/drama_low_vram/backbone_graph.py:327-337) with the rounding points of
 * the bf16 torch modules they call:
 *   gate, up = bf16(x @ gate_proj^T), bf16(x @ up_proj^T)
 *   h = bf16(bf16(silu(gate)) * up);  d = bf16(h @ down_proj^T)
 *   s = bf16(sigmoid(bf16(x . gate_weight)));  shared = bf16(s * d)
 *   t = routed ? bf16(routed + shared) : shared
 *   out = residual ? bf16(residual + t) : t
 * x, routed, residual, out: [tokens, H] bfloat16 (row stride H); weights bf16
 * row-major with row strides in elements (multiples of 8, 16-byte aligned).
 * H and I multiples of 128, tokens <= 4096. out may alias routed or residual
 * (each element is read before it is written, by the same thread).
 * One row at H 2048, I 768 runs as a single launch that starts reading the
 * weights before the launch it follows on the stream has finished (only x,
 * routed and residual wait for it): the weights must not be written by that
 * launch.
 * ------------------------------------------------------------------------- */
typedef struct DramaB200SharedExpert {
    const void* gate_proj;     /* [I, H] */
    const void* up_proj;       /* [I, H] */
    const void* down_proj;     /* [H, I] */
    const void* gate_weight;   /* [H]: shared_expert_gate (a Linear to one output, no bias) */
    int64_t gate_row_stride, up_row_stride, down_row_stride;
    int32_t hidden, intermediate;
} DramaB200SharedExpert;

DRAMA_B200_API size_t drama_b200_shared_expert_workspace_bytes(int64_t tokens, int hidden, int intermediate);

DRAMA_B200_API int drama_b200_shared_expert(const DramaB200SharedExpert* mlp, const void* x, int64_t tokens,
                                            const void* routed, const void* residual, void* out, void* workspace,
                                            size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * One decode MoE layer, fully on the device (graph-capturable):
 *   normed = bf16(x * 1/sqrt(mean(x^2) + eps) * gamma)      (fixed fp32 order)
 *   logits = bf16(normed @ gate^T)                           (fixed fp32 order)
 *   w, ids = route_topk(logits, top_k, renormalize=1) ; w -> bf16
 *   hidden_out = bf16(hidden_in + experts(normed, ids, w))   (K1 arithmetic)
 * This is one layer of BackboneDecodeGraph (src/drama_low_vram/
 * backbone_graph.py:306-337: router pre-graph, expert call, residual post-
 * graph) with no mixer or shared expert and with the expert call on the
 * device instead of ExpertOffloadManager's host routing (offload.py:1016-1063).
 * hidden_in/hidden_out: bf16 [tokens, H] (must not overlap); gate: bf16
 * [experts, H]; gamma: fp32 [H]; next_gate (optional) is prefetched into L2
 * for the following layer. ids_out (int64 [tokens, top_k]), weights_out
 * (bf16), normed_out (bf16 [tokens, H]) and moe_out (bf16 [tokens, H], the
 * combined expert output before the residual add) are optional traces.
 * hidden_in, hidden_out, normed_out and moe_out start on 16-byte boundaries.
 * tokens * top_k <= 256, H % 256 == 0, experts = bank->slots <= 1024.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API size_t drama_b200_moe_layer_workspace_bytes(int64_t tokens, int top_k, int hidden,
                                                           int intermediate, int experts);

DRAMA_B200_API int drama_b200_fp8_moe_layer(const DramaB200Fp8Bank* bank, const void* gate,
                                            const void* next_gate, const float* gamma, float eps,
                                            const void* hidden_in, void* hidden_out,
                                            int64_t tokens, int top_k, int64_t* ids_out,
                                            void* weights_out, void* normed_out, void* moe_out,
                                            void* workspace, size_t workspace_bytes, void* stream);

/* Kernel launches one drama_b200_fp8_moe_layer call makes for these sizes on
 * the current device (1: the one-launch single-row layer; 2: the two-launch
 * single-row layer; 3: router, gate/up and down launches for several rows). */
DRAMA_B200_API int drama_b200_moe_layer_launches(int64_t tokens, int top_k, int hidden, int intermediate,
                                                 int experts);

/* The same decode layer driven by the caller's router inputs: `normed` is the
 * bf16 [H] row after the RMSNorm and `logits` the bf16 [experts] router
 * logits, both as the reference's decode graph computes them
 * (BackboneDecodeGraph._route_impl, src/drama_low_vram/backbone_graph.py:
 * 316-319: post_attention_layernorm, then moe.gate as a bf16 F.linear). The
 * layer applies softmax(logits.float()) -> topk -> renormalise -> bf16 (lines
 * 320-323, torch's order), the experts on `normed`, and the residual
 * (hidden_out = bf16(hidden_in + experts)), so its routes are the reference's
 * bit for bit whatever RMSNorm and GEMV order produced the inputs.
 * tokens == 1; hidden % 512 == 0 up to 2048; intermediate % 16 == 0;
 * top_k <= 16; normed, logits, hidden_in, hidden_out and moe_out start on
 * 16-byte boundaries. Workspace: drama_b200_moe_layer_workspace_bytes. */
DRAMA_B200_API int drama_b200_fp8_moe_layer_logits(const DramaB200Fp8Bank* bank, const void* normed,
                                                   const void* logits, const void* hidden_in, void* hidden_out,
                                                   int64_t tokens, int top_k, int64_t* ids_out,
                                                   void* weights_out, void* moe_out, void* workspace,
                                                   size_t workspace_bytes, void* stream);

/* The two halves of drama_b200_fp8_moe_layer, for callers that time or
 * interleave them: the router (RMSNorm, router GEMV, top-k, expert groups,
 * written into the workspace) and the expert GEMVs with combine + residual
 * (reading the groups the router left in the same workspace). Issue them on
 * one stream, router first, with the same bank/tokens/top_k/workspace. */
DRAMA_B200_API int drama_b200_fp8_moe_router(const DramaB200Fp8Bank* bank, const void* gate,
                                             const void* next_gate, const float* gamma, float eps,
                                             const void* hidden_in, int64_t tokens, int top_k,
                                             int64_t* ids_out, void* weights_out, void* normed_out,
                                             void* workspace, size_t workspace_bytes, void* stream);

DRAMA_B200_API int drama_b200_fp8_moe_experts(const DramaB200Fp8Bank* bank, const void* hidden_in,
                                              void* hidden_out, int64_t tokens, int top_k,
                                              void* moe_out, void* workspace, size_t workspace_bytes,
                                              void* stream);

/* Device status words of the last decode call on this workspace:
 * [0] = pairs dropped for an out-of-range slot id. Copy them to the host
 * with drama_b200_decode_status_offset() bytes into the workspace. */
DRAMA_B200_API size_t drama_b200_decode_status_offset(void);

/* ---------------------------------------------------------------------------
 * K2 prefill: the same layer math as drama_b200_fp8_decode for many tokens,
 * as grouped tensor-core GEMMs over experts. Replaces ExpertBackend.forward
 * (src/drama_low_vram/offload.py:187-196) as TorchExpertBackend computes it
 * (offload.py:199-244): W = bf16(fp8 * block scale) (offload.py:44-56),
 *   gu = bf16(x @ W13^T); h = bf16(bf16(silu(gate)) * up);
 *   down = bf16(h @ W2^T); out[t] = bf16(sum over slots, in slot order, of
 *   down[t*k+s] * weight[t*k+s])   (fp32 sum).
 * x, out: bf16 [tokens, H] (must not overlap); ids: [tokens, top_k] I32/I64
 * local slots; weights: [tokens, top_k] F32/F16/BF16. H % 256 == 0,
 * I % 128 == 0, slots <= 1024, pairs <= 2^24. A pair whose id is outside
 * [0, slots) contributes zero and is counted in status word 0
 * (drama_b200_prefill_status_offset() bytes into the workspace).
 * ------------------------------------------------------------------------- */
DRAMA_B200_API size_t drama_b200_prefill_workspace_bytes(int64_t tokens, int top_k, int hidden,
                                                         int intermediate, int experts);

DRAMA_B200_API size_t drama_b200_prefill_status_offset(void);

DRAMA_B200_API int drama_b200_fp8_prefill(const DramaB200Fp8Bank* bank, const void* x, int64_t tokens,
                                          int top_k, const void* ids, int ids_dtype,
                                          const void* weights, int weights_dtype, void* out,
                                          void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * FP8 decode without a workspace, for callers that cannot allocate device
 * memory: a host binding with no device allocator of its own, or a process
 * whose memory manager has reserved the device and permits no further
 * allocation (cudaMalloc would also synchronise the device). This entry point
 * has no counterpart in the reference; the reference always allocates its
 * outputs and scratch through PyTorch.
 *
 * Same arguments and results as drama_b200_fp8_decode minus the workspace.
 * Its scratch is a static device array of drama_b200_static_scratch_bytes()
 * (16 MiB) inside the library, held on every GPU that loads the library until
 * the process exits. A call whose scratch need, drama_b200_decode_workspace_
 * bytes() for the same sizes, exceeds that fails with a message naming both
 * sizes; on a 148-SM B200 at top-8 that is above 94 tokens at hidden 2048 /
 * intermediate 768 and above 43 tokens at hidden 4096 / intermediate 2048.
 * The call allocates nothing.
 *
 * The first call in each device context (with that device current) looks up
 * the array's device address with cudaGetSymbolAddress and keeps it for that
 * context; make that first call before any stream capture. The array needs
 * no clearing: every call rewrites its status words and zeroes its counters
 * before the expert kernels read them, and keeps the last call's other
 * contents. Every call, from any thread, shares the one array, so calls that
 * can overlap on the GPU (different streams without ordering between them)
 * race; order them.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API size_t drama_b200_static_scratch_bytes(void);

DRAMA_B200_API int drama_b200_fp8_decode_static(const DramaB200Fp8Bank* bank, const void* x,
                                                int x_dtype, int64_t tokens, int top_k,
                                                const void* ids, int ids_dtype,
                                                const void* weights, int weights_dtype,
                                                void* out, float* pair_out, void* stream);

/* ---------------------------------------------------------------------------
 * Per-row expert projections for few rows per expert (decode batches, the
 * rows an expert-parallel rank receives, staged offload). Replaces
 * TorchExpertBackend.forward_pairs (src/drama_low_vram/offload.py:215-244)
 * before its route weighting: row r of out [rows, hidden] (bf16) =
 * bf16(bf16(bf16(silu(g)) * u) @ W2^T) with g, u = bf16(x[r] @ W13^T), for the
 * expert ids[r] (I32/I64), computed as the decode kernels compute it: exact
 * f16 expansion of the E4M3 weights, block scales applied to fp32 partial
 * sums, activations as f16 with a power-of-two scale per 64 values. Rows whose id
 * is outside [0, slots) are not written (status[0] counts them, at
 * drama_b200_prefill_status_offset() in the workspace). x: rows of hidden
 * bf16 values, row r at x + r * x_row_stride (elements, a multiple of 8);
 * with ids == NULL each row is tagged: its expert id is the int32 at element
 * `hidden` of the row (x_row_stride >= hidden + 8), as drama_b200_ep_dispatch
 * writes them. hidden and intermediate multiples of 128; rows <= 2^24. Each
 * row's result is independent of the other rows in the call.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API size_t drama_b200_expert_rows_workspace_bytes(int64_t rows, int hidden, int intermediate,
                                                             int experts);

DRAMA_B200_API int drama_b200_fp8_expert_rows(const DramaB200Fp8Bank* bank, const void* x, int64_t x_row_stride,
                                              int64_t rows, const void* ids, int ids_dtype, void* out,
                                              void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Expert parallelism over G ranks (E/G experts per rank). The reference is single-GPU, so the exchange has no counterpart in
 * it; the two entries split the reference's partitioned expert call
 * (src/drama_low_vram/offload.py:1206-1276: group the (token, slot) pairs by
 * expert, run each expert on its rows, sum fp32 weighted rows in slot order at
 * 1242-1244) across the ranks.
 *
 * drama_b200_ep_dispatch: for the local hidden rows [tokens, hidden_size]
 * (bf16) and their routes ids [tokens, top_k] (global expert ids), writes
 * the following. placement (int32 [experts], may be NULL) gives each expert's
 * rank-major position, a permutation of [0, experts): expert e lives on rank
 * placement[e] / (experts / ranks) as local id placement[e] % (experts /
 * ranks); NULL means placement[e] = e (contiguous blocks).
 *   send_rows [ranks, capacity] rows of send_row_stride bf16 elements (a
 *     multiple of 8, >= hidden_size): the hidden row of every pair in the
 *     block of the rank owning its expert, pairs in order;
 *   the receiver-local expert id of each row, or E/G for an unused row: in
 *     send_ids [ranks, capacity] int32, or when send_ids is NULL as the int32
 *     at element hidden_size of the row itself (send_row_stride >=
 *     hidden_size + 8), so that one all-to-all carries rows and ids;
 *   pair_rows [tokens * top_k] int32: the row of each pair in send_rows, -1
 *     for a pair whose id is outside [0, experts) or that did not fit;
 *   status[0] (int32, may be NULL) = pairs with an out-of-range id, status[1]
 *     = pairs beyond a destination's capacity (capacity = tokens * top_k
 *     never overflows).
 * After an all-to-all of the tagged send rows, drama_b200_fp8_expert_rows
 * (ids NULL) on the received rows gives each row's bf16 down projection
 * (unused rows are dropped by their id); a second all-to-all brings them back
 * in the same positions.
 *
 * drama_b200_ep_combine: out[t] = bf16(residual[t] + bf16(sum over slots s in
 * order of rows[pair_rows[t*k+s]] * weights[t*k+s])), fp32 products and sums
 * (offload.py:212, 1244), over rows [row_count, hidden_size] bf16; a pair whose
 * row is -1 or outside [0, row_count) contributes zero. residual may be NULL,
 * or equal to out.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API int drama_b200_ep_dispatch(const void* hidden, int64_t tokens, int hidden_size, const void* ids,
                                          int ids_dtype, int top_k, int experts, int ranks,
                                          const int32_t* placement, int64_t capacity, void* send_rows,
                                          int64_t send_row_stride, int32_t* send_ids, int32_t* pair_rows,
                                          int32_t* status, void* stream);

DRAMA_B200_API int drama_b200_ep_combine(const void* rows, int64_t row_count, const int32_t* pair_rows,
                                         const void* weights, int weights_dtype, int64_t tokens, int top_k,
                                         int hidden_size, const void* residual, void* out, void* stream);

/* ---------------------------------------------------------------------------
 * Expert-parallel exchange over NVLink peer memory (no counterpart in the
 * reference; an alternative to the all-to-alls around drama_b200_ep_dispatch).
 * Each rank allocates three buffers with drama_b200_ep_buffers_alloc, shares
 * them with drama_b200_ipc_handle / drama_b200_ipc_open, and fills a
 * DramaB200EpPeers with every rank's pointers (its own for its own rank):
 *   recv    [ranks][capacity][hidden + 8] bf16: block s written by rank s;
 *           row = hidden values, then the receiver-local expert id (int32);
 *   back    [ranks][capacity][hidden] bf16: block d written by rank d;
 *   signals [3 * ranks] int32 (zeroed): dispatch flags, row counts, return
 *           flags; epoch and done are this rank's own counters (zeroed).
 * A layer is, in stream order on every rank:
 *   drama_b200_ep_p2p_dispatch     (rows into the owners' recv, then flags)
 *   drama_b200_fp8_expert_rows_p2p (waits for every source; results into
 *                                   the sources' back, then return flags)
 *   drama_b200_ep_p2p_combine      (waits for every expert rank; slot sum)
 * Every rank must issue the same sequence of layers. Waits give up after
 * wait_ns nanoseconds of global time (0: 2 s; at most 60 s) and set status[2]
 * (bit 1: the row prep's wait for a source, bit 2: the combine's wait for an
 * expert rank); the result of that step is then invalid. The counters block
 * (epoch, dispatch and GEMM arrival counts) is 256 zeroed bytes.
 * ------------------------------------------------------------------------- */
typedef struct DramaB200EpPeers {
    int32_t ranks, rank;
    int64_t capacity;           /* rows per (source, destination) block: tokens * top_k */
    int32_t hidden, experts;
    void* recv[8];
    void* back[8];
    int32_t* signals[8];
    int32_t* epoch;             /* this rank's step counter */
    int32_t* done;              /* this rank's arrival counters (32 int32, zeroed) */
    int64_t wait_ns;            /* limit of every peer wait; 0: 2 s */
} DramaB200EpPeers;

DRAMA_B200_API int drama_b200_ep_buffers_alloc(int ranks, int64_t capacity, int hidden, void** recv, void** back,
                                               int32_t** signals, int32_t** counters);

DRAMA_B200_API int drama_b200_ep_buffers_free(void* recv, void* back, int32_t* signals, int32_t* counters);

/* CUDA IPC of a buffer from drama_b200_ep_buffers_alloc (64-byte handles). */
DRAMA_B200_API int drama_b200_ipc_handle(const void* device_ptr, void* handle_out);

DRAMA_B200_API int drama_b200_ipc_open(const void* handle, void** device_ptr);

DRAMA_B200_API int drama_b200_ipc_close(void* device_ptr);

/* pair_rows as drama_b200_ep_dispatch; tokens * top_k <= 4096. */
DRAMA_B200_API int drama_b200_ep_p2p_dispatch(const DramaB200EpPeers* peers, const void* hidden, int64_t tokens,
                                              const void* ids, int ids_dtype, int top_k,
                                              const int32_t* placement, int32_t* pair_rows, int32_t* status,
                                              void* stream);

/* workspace: drama_b200_expert_rows_workspace_bytes(ranks * capacity, ...). */
DRAMA_B200_API int drama_b200_fp8_expert_rows_p2p(const DramaB200Fp8Bank* bank, const DramaB200EpPeers* peers,
                                                  void* workspace, size_t workspace_bytes, int32_t* status,
                                                  void* stream);

DRAMA_B200_API int drama_b200_ep_p2p_combine(const DramaB200EpPeers* peers, const int32_t* pair_rows,
                                             const void* weights, int weights_dtype, int64_t tokens, int top_k,
                                             const void* residual, void* out, int32_t* status, void* stream);

/* ---------------------------------------------------------------------------
 * K4 staging: host -> HBM expert copies on a copy stream. Replaces the
 * transfer half of _StagingPool.stage (src/drama_low_vram/offload.py:543-651:
 * the host gather at 561-594 and the H2D copy_ on the compute stream at
 * 596-636) and its _copy_done event (offload.py:637-645).
 *
 * Copy i moves bytes[i] from host_src[i] to dev_dst[i]. Sources must be
 * page-locked host memory (cudaHostAlloc or cudaHostRegister); a pageable
 * source is rejected because cudaMemcpyAsync would silently run it
 * synchronously. Destinations must be device memory on one device. Copies
 * that continue one another in both address spaces are issued as one
 * cudaMemcpyAsync. Before the first copy copy_stream waits on wait_event
 * (may be NULL: e.g. the compute event after the last reader of these slots);
 * after the last copy done_event is recorded on copy_stream (may be NULL).
 * Both events must already exist (cudaEventCreate). All pointers are checked
 * before anything is enqueued. count 0 only waits and records.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API int drama_b200_stage_copies(const void* const* host_src, void* const* dev_dst,
                                           const uint64_t* bytes, int count, void* copy_stream,
                                           void* wait_event, void* done_event);

/* ---------------------------------------------------------------------------
 * Host byte sources for staging: page-lock an existing host range, e.g. a
 * private mmap of an expert cache file (experts.bin, manifest format
 * "drama3-official-fp8-experts" v1, src/drama_low_vram/expert_cache_file.py:
 * 28-33, 112-153, 526-556), so that drama_b200_stage_copies can DMA expert
 * rows straight out of the mapping. The reference instead gathers those rows
 * into a pinned bounce buffer on the host (offload.py:561-594, native
 * drama_gather_rows, native/include/drama_native.h:28) before each copy.
 *
 * [host_ptr, host_ptr + bytes) is widened to whole pages and registered with
 * cudaHostRegisterPortable, plus cudaHostRegisterReadOnly when read_only is
 * non-zero (refused when the device cannot do it). Read-only registration of a
 * MAP_PRIVATE file mapping pins the page-cache pages themselves, with no
 * copy-on-write copies; the driver refuses PROT_READ-only file mappings and
 * shared writable mappings of disk files, with or without the flag.
 * The widened range is returned in registered_base/registered_bytes;
 * pass registered_base to drama_b200_host_unregister. Ranges that share a page
 * cannot both be registered.
 * ------------------------------------------------------------------------- */
DRAMA_B200_API int drama_b200_host_register(void* host_ptr, uint64_t bytes, int read_only,
                                            void** registered_base, uint64_t* registered_bytes);

DRAMA_B200_API int drama_b200_host_unregister(void* registered_base);

/* *locked = 1 when the first and the last byte of [host_ptr, host_ptr + bytes)
 * are page-locked host memory, else 0. Unlike torch's Tensor.is_pinned, which
 * looks at the start of the whole storage, this looks at the range itself: a
 * view into a partly registered mapping reads as locked only where it is. */
DRAMA_B200_API int drama_b200_host_locked(const void* host_ptr, uint64_t bytes, int* locked);

#ifdef __cplusplus
}
#endif

#endif /* DRAMA_B200_H */
