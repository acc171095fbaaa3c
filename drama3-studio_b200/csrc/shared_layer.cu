// The shared expert + sigmoid gate, fused with the routed sum and the
// residual, for ONE bfloat16 row in ONE launch (hidden 2048, intermediate
// 768): BackboneDecodeGraph._shared_impl + _post_impl
// (src/drama_low_vram/backbone_graph.py:327-337) with the bf16 modules'
// rounding points, as shared_expert.cu:
//   gate, up = bf16(x . gate_proj[j]), bf16(x . up_proj[j])
//   h = bf16(bf16(silu(gate)) * up);  d = bf16(h . down_proj[n])
//   s = bf16(sigmoid(bf16(x . gate_weight)));  y = bf16(s * d)
//   y = bf16(routed + y) (with routed);  out = bf16(residual + y) (with residual)
//
// Schedule: 24 clusters of 4 CTAs. Cluster u owns unit u, intermediate
// columns [32u, 32u + 32) (two 16-wide tiles), and CTA r of the cluster holds
// quarter r of K for gate/up and quarter r of the output rows for the down
// projection. The weights are constants, so each CTA issues its tensor-map
// loads (64 KB of gate/up rows, 32 KB of down columns, no multicast) BEFORE
// the programmatic dependency wait: they stream while the previous launch
// finishes. After the wait each CTA
//   1. forms its quarter of every gate/up row sum and of x . gate_weight on the
//      CUDA cores (fixed order: 16 products per lane, then a lane butterfly),
//      and stores them into every CTA of the cluster (distributed shared
//      memory); after the cluster barrier each CTA adds the quarters in rank
//      order and forms the unit's 32 values of h and the gate scalar s;
//   2. multiplies its 512 down rows by those 32 values (four lanes per row,
//      8 products each, a two-step butterfly): a partial down projection,
//      stored in fp32;
//   3. takes an arrival ticket (one acquire-release atomic per CTA); the last
//      CTA of quarter r adds, for each of its rows, the 24 units' partials in
//      unit order and applies the rounding chain above.
// Other shapes and batches keep the two-launch schedule of shared_expert.cu.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace drama {

namespace {

namespace cg = cooperative_groups;

constexpr int kSlH = 2048;
constexpr int kSlI = 768;
constexpr int kSlCluster = 4;
constexpr int kSlWarps = 8;                        // consumer warps
constexpr int kSlThreads = (kSlWarps + 1) * 32;    // + one TMA producer warp
constexpr int kSlConsumers = kSlWarps * 32;
constexpr int kSlCols = 32;                        // intermediate columns per unit (two 16-wide tiles)
constexpr int kSlUnits = kSlI / kSlCols;           // 24
constexpr int kSlHq = kSlH / kSlCluster;           // this CTA's quarter of K and of the output rows (512)
constexpr int kSlRows = 2 * kSlCols;               // gate and up rows of a unit (64)
constexpr uint32_t kSlBox = 16 * kSlHq * 2;        // one gate or up box: 16 rows x a quarter of K, bf16 (16 KB)
constexpr uint32_t kSlW2Box = 256 * kSlCols * 2;   // 256 down rows x the unit's 32 columns (16 KB)
constexpr int kSlXch = kSlRows + 4;                // exchange slots per rank: 64 row sums, x . gate_weight, pad
static_assert(kSlRows % kSlWarps == 0 && kSlHq == 2 * kSlConsumers, "rows per warp, rows per combine thread");

// Shared memory from a 1024-byte aligned base. Each offset is the previous one
// plus the region named beside it.
constexpr uint32_t kOffGU = 0;
constexpr uint32_t kOffW2 = kOffGU + 4 * kSlBox;                     // gate/up: boxes [tile 0 gate, up, tile 1 gate, up]
constexpr uint32_t kOffX = kOffW2 + 2 * kSlW2Box;                    // down: [512 rows][32 columns] bf16
constexpr uint32_t kOffXch = kOffX + kSlHq * 2;                      // x: this CTA's quarter of the row
constexpr uint32_t kOffCell = kOffXch + kSlCluster * kSlXch * 4;     // xch: [rank][kSlXch] quarters
constexpr uint32_t kOffH = kOffCell + kSlXch * 4;                    // cell: this CTA's quarters
constexpr uint32_t kOffBar = kOffH + kSlCols * 4;                    // h: the unit's 32 values (fp32 of bf16)
constexpr uint32_t kSlUsed = kOffBar + 8 * 8 + 1024;                 // barriers, + room to align the base
// One CTA per SM: a CTA that shared an SM would halve both CTAs' share of it.
constexpr uint32_t kSlSmem = kSlUsed > 116 * 1024 ? kSlUsed : 116 * 1024;
static_assert(kSlSmem <= 227 * 1024, "shared memory per CTA");

struct SharedLayerArgs {
    const __nv_bfloat16* x;         // [H]
    const __nv_bfloat16* gate_weight;  // [H]
    const __nv_bfloat16* routed;    // [H] or NULL
    const __nv_bfloat16* residual;  // [H] or NULL
    __nv_bfloat16* out;             // [H]
    float* part;                    // [units][H] fp32 partial down projections
    int32_t* tickets;               // [4] arrivals per quarter, zero between calls
    int32_t* status;                // [4] [1] waits that ran out
    CUtensorMap gate_map;           // gate_proj viewed as [I][H/64][64] bf16
    CUtensorMap up_map;             // up_proj, the same view
    CUtensorMap down_map;           // down_proj viewed as [1][H][I] bf16
};

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ uint32_t sl_smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

}  // namespace

namespace {

__global__ void __launch_bounds__(kSlThreads, 1) shared_layer_kernel(const __grid_constant__ SharedLayerArgs a) {
    extern __shared__ __align__(1024) uint8_t sl_smem_raw[];
    __shared__ float s_gdot[2];
    __shared__ float s_gs;
    __shared__ int s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    cg::cluster_group cluster = cg::this_cluster();
    const int r = static_cast<int>(cluster.block_rank());
    const int unit = static_cast<int>(blockIdx.x) / kSlCluster;
    const uint32_t raw_u32 = sl_smem_u32(sl_smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
    uint8_t* base = sl_smem_raw + (base_u32 - raw_u32);
    __nv_bfloat16* s_x = reinterpret_cast<__nv_bfloat16*>(base + kOffX);
    float* s_xch = reinterpret_cast<float*>(base + kOffXch);
    float* s_cell = reinterpret_cast<float*>(base + kOffCell);
    float* s_h = reinterpret_cast<float*>(base + kOffH);
    const uint32_t full0 = base_u32 + kOffBar, w2_bar = full0 + 8 * 4;
    int32_t* status = a.status;

    if (tid == 0) {
        for (int b = 0; b < 4; ++b) mbar_init(full0 + 8 * b, 1);
        mbar_init(w2_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    cluster.barrier_arrive();  // paired with the wait before the first remote store

    // The weights do not depend on the previous launch: their loads and the
    // gate vector go out before the dependency wait.
    uint4 gw = make_uint4(0u, 0u, 0u, 0u);
    if (warp == kSlWarps) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            for (int b = 0; b < 4; ++b) {  // box b: tile b / 2, gate (even) or up (odd) rows
                mbar_arrive_expect_tx(full0 + 8 * b, kSlBox);
                tma_load_3d(base_u32 + kOffGU + b * kSlBox, (b & 1) ? &a.up_map : &a.gate_map, 0, r * (kSlHq / 64),
                            unit * kSlCols + (b >> 1) * 16, full0 + 8 * b, pol);
            }
            mbar_arrive_expect_tx(w2_bar, 2 * kSlW2Box);
            for (int bx = 0; bx < 2; ++bx)
                tma_load_3d(base_u32 + kOffW2 + bx * kSlW2Box, &a.down_map, unit * kSlCols, r * kSlHq + bx * 256, 0,
                            w2_bar, pol);
        }
        __syncwarp();
    } else if (tid < kSlHq / 8) {
        gw = __ldg(reinterpret_cast<const uint4*>(a.gate_weight + r * kSlHq) + tid);
    }
    grid_launch_dependents();
    grid_dependency_wait();  // x, routed and residual may come from the previous launch

    if (warp < kSlWarps) {
        // This CTA's quarter of x, and its quarter of x . gate_weight (warps
        // 0 and 1: 8 products per lane, a lane butterfly, the two warps added).
        if (tid < kSlHq / 8) {
            const uint4 xv = __ldcg(reinterpret_cast<const uint4*>(a.x + r * kSlHq) + tid);
            reinterpret_cast<uint4*>(s_x)[tid] = xv;
            float p = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) p = fmaf(bf16_at(xv, e), bf16_at(gw, e), p);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) p += __shfl_xor_sync(0xffffffffu, p, off);
            if (lane == 0) s_gdot[warp] = p;
        }
        named_barrier(1, kSlConsumers);
        if (tid == 0) s_cell[kSlRows] = s_gdot[0] + s_gdot[1];

        // Gate/up rows: warp w takes unit rows 8w..8w+7 of box w / 2. A row of
        // a box is 8 lines of 128 bytes (64 K values each), 16-byte unit u of
        // line L stored at u ^ (L % 8); lane (c, u) = (lane / 8, lane % 8)
        // reads unit u of lines c and c + 4.
        const int c0 = lane >> 3, u = lane & 7;
        const uint4 xa = lds128(s_x + c0 * 64 + u * 8);
        const uint4 xb = lds128(s_x + (c0 + 4) * 64 + u * 8);
        const int box = warp >> 1;
        const uint8_t* bx = base + kOffGU + box * kSlBox;
        mbar_wait(full0 + 8 * box, 0, status ? status + 1 : nullptr);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = 8 * (warp & 1) + i;  // row of the box
            const uint4 wa = lds128(bx + (row * 8 + c0) * 128 + ((u ^ c0) << 4));
            const uint4 wb = lds128(bx + (row * 8 + c0 + 4) * 128 + ((u ^ (c0 + 4)) << 4));
            float acc = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = fmaf(bf16_at(wa, e), bf16_at(xa, e), acc);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = fmaf(bf16_at(wb, e), bf16_at(xb, e), acc);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
            if (lane == 0) s_cell[8 * warp + i] = acc;  // unit row 16 box + row
        }
        named_barrier(1, kSlConsumers);
        // The quarters into slot r of every cluster CTA's exchange area.
        cluster.barrier_wait();  // every CTA of the cluster is running
        if (tid <= kSlRows) {
            const float v = s_cell[tid];
            float* dst = s_xch + r * kSlXch + tid;
#pragma unroll
            for (int d = 0; d < kSlCluster; ++d) *cluster.map_shared_rank(dst, d) = v;
        }
    }
    if (warp == kSlWarps) cluster.barrier_wait();
    cluster.sync();  // every quarter is in every CTA

    if (warp < kSlWarps) {
        // h of the unit's 32 columns and the gate scalar, quarters in rank
        // order, with the bf16 modules' rounding points. Column c is row c % 16
        // of tile c / 16: gate unit row 32 (c / 16) + c % 16, up row + 16.
        if (tid < kSlCols) {
            const int gr = 32 * (tid >> 4) + (tid & 15);
            float gsum = 0.0f, usum = 0.0f;
#pragma unroll
            for (int d = 0; d < kSlCluster; ++d) {
                gsum += s_xch[d * kSlXch + gr];
                usum += s_xch[d * kSlXch + gr + 16];
            }
            const float gate = bf16r(gsum), up = bf16r(usum);
            const float act = bf16r(gate / (1.0f + expf(-gate)));
            s_h[tid] = bf16r(act * up);
        } else if (tid == kSlCols) {
            float dot = 0.0f;
#pragma unroll
            for (int d = 0; d < kSlCluster; ++d) dot += s_xch[d * kSlXch + kSlRows];
            s_gs = bf16r(1.0f / (1.0f + expf(-bf16r(dot))));
        }
        mbar_wait(w2_bar, 0, status ? status + 1 : nullptr);
        named_barrier(1, kSlConsumers);  // h, the gate scalar and the down columns in shared memory

        // Partial down projection: warp w takes rows 64w..64w+63 of the
        // quarter, 8 per pass; lane (row, q) = (lane / 4, lane % 4) multiplies
        // columns 8q..8q+7 and four lanes add their sums by a butterfly.
        const int q = lane & 3;
        float hv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) hv[e] = s_h[8 * q + e];
        const uint8_t* w2s = base + kOffW2;
        float* pr = a.part + static_cast<int64_t>(unit) * kSlH + r * kSlHq;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            const int row = 64 * warp + 8 * p + (lane >> 2);
            const uint4 wv = lds128(w2s + row * (kSlCols * 2) + 16 * q);
            float acc = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = fmaf(bf16_at(wv, e), hv[e], acc);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (q == 0) __stcg(pr + row, acc);
        }
        // Ticket: the CTA barrier orders every thread's partial stores before
        // thread 0's release; its acquire orders the last arriver's reads.
        named_barrier(1, kSlConsumers);
        if (tid == 0) s_last = atomic_add_acq_rel_gpu(a.tickets + r, 1) == kSlUnits - 1;
        named_barrier(1, kSlConsumers);
        if (s_last) {
            // Last CTA of quarter r: rows 2 tid and 2 tid + 1 of every unit's
            // partial, all loads in flight before the first store, added in
            // unit order; then the rounding chain.
            if (tid == 0) a.tickets[r] = 0;
            const int n = r * kSlHq + 2 * tid;
            float2 v[kSlUnits];
#pragma unroll
            for (int u = 0; u < kSlUnits; ++u)
                v[u] = __ldcg(reinterpret_cast<const float2*>(a.part + static_cast<int64_t>(u) * kSlH + n));
            uint32_t rt = 0u, rs = 0u;
            if (a.routed) rt = *reinterpret_cast<const uint32_t*>(a.routed + n);
            if (a.residual) rs = *reinterpret_cast<const uint32_t*>(a.residual + n);
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int u = 0; u < kSlUnits; ++u) {
                s0 += v[u].x;
                s1 += v[u].y;
            }
            const float gs = s_gs;
            float y0 = bf16r(gs * bf16r(s0)), y1 = bf16r(gs * bf16r(s1));
            if (a.routed) {
                y0 = bf16r(__uint_as_float(rt << 16) + y0);
                y1 = bf16r(__uint_as_float(rt & 0xffff0000u) + y1);
            }
            if (a.residual) {
                y0 = __uint_as_float(rs << 16) + y0;
                y1 = __uint_as_float(rs & 0xffff0000u) + y1;
            }
            *reinterpret_cast<__nv_bfloat162*>(a.out + n) = __floats2bfloat162_rn(y0, y1);
        }
    }
}

// Clusters of the kernel that fit the device at once (cached per device), or
// -1 when the kernel cannot be configured.
int shared_layer_clusters() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (cached[dev]) return cached[dev];
    if (cudaFuncSetAttribute(shared_layer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSlSmem)) != cudaSuccess) {
        cudaGetLastError();
        return cached[dev] = -1;
    }
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(kSlCluster * ((sms + kSlCluster - 1) / kSlCluster));
    q.blockDim = dim3(kSlThreads);
    q.dynamicSmemBytes = kSlSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kSlCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    q.attrs = attr;
    q.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, shared_layer_kernel, &q) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        return cached[dev] = -1;
    }
    return cached[dev] = clusters;
}

}  // namespace

bool shared_layer_supported(const DramaB200SharedExpert& m, int64_t tokens) {
    if (tokens != 1 || m.hidden != kSlH || m.intermediate != kSlI) return false;
    // the tensor maps: 16-byte aligned bases (the entry point checks) and row strides
    if ((m.gate_row_stride * 2) % 16 || (m.up_row_stride * 2) % 16 || (m.down_row_stride * 2) % 16) return false;
    if (reinterpret_cast<uintptr_t>(m.gate_weight) % 16) return false;
    return tensor_map_encoder() != nullptr && shared_layer_clusters() >= kSlUnits;
}

cudaError_t shared_layer_launch(const DramaB200SharedExpert& m, const void* x, const void* routed,
                                const void* residual, void* out, float* part, int32_t* tickets, int32_t* status,
                                cudaStream_t s) {
    const TensorMapEncode encode = tensor_map_encoder();
    if (!encode || shared_layer_clusters() < kSlUnits) return cudaErrorInvalidConfiguration;
    SharedLayerArgs a{};
    a.x = static_cast<const __nv_bfloat16*>(x);
    a.gate_weight = static_cast<const __nv_bfloat16*>(m.gate_weight);
    a.routed = static_cast<const __nv_bfloat16*>(routed);
    a.residual = static_cast<const __nv_bfloat16*>(residual);
    a.out = static_cast<__nv_bfloat16*>(out);
    a.part = part;
    a.tickets = tickets;
    a.status = status;
    const cuuint32_t ones[3] = {1, 1, 1};
    // gate_proj / up_proj [I][H] viewed as [I][H/64][64]: one box = 16 rows x
    // this CTA's quarter of K, 128-byte lines with the 128-byte swizzle.
    const void* gu[2] = {m.gate_proj, m.up_proj};
    const int64_t gu_stride[2] = {m.gate_row_stride, m.up_row_stride};
    CUtensorMap* gu_map[2] = {&a.gate_map, &a.up_map};
    for (int i = 0; i < 2; ++i) {
        const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(kSlH / 64), static_cast<cuuint64_t>(kSlI)};
        const cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(gu_stride[i]) * 2};
        const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kSlHq / 64), 16};
        if (encode(gu_map[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(gu[i]), dims, strides, box,
                   ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    // down_proj [H][I] viewed as [1][H][I]: one box = the unit's 32 columns x 256 rows.
    {
        const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kSlI), static_cast<cuuint64_t>(kSlH), 1};
        const cuuint64_t strides[2] = {static_cast<cuuint64_t>(m.down_row_stride) * 2,
                                       static_cast<cuuint64_t>(m.down_row_stride) * 2 * kSlH};
        const cuuint32_t box[3] = {static_cast<cuuint32_t>(kSlCols), 256, 1};
        if (encode(&a.down_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(m.down_proj), dims, strides,
                   box, ones, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = kSlCluster;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kSlCluster * kSlUnits);
    cfg.blockDim = dim3(kSlThreads);
    cfg.dynamicSmemBytes = kSlSmem;
    cfg.stream = s;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, shared_layer_kernel, a);
}

}  // namespace drama
