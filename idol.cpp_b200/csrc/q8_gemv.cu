// q8_gemv.cu - the Q8_0 (and Q4_K) linear for decode-sized batches (1 <= M <= 16 tokens): Y = X . dequant(W)^T + bias (+ residual)
// (-> act), the small-M strategy of the reference's GPU path (tools/idol_triton.py:36-126 fused_linear at M <= 16,
// src/kernels.cpp:246-296 gemm_quant on the CPU).
//
// At this size the launch is bound by streaming W from HBM (1.0625 bytes per weight), so the kernel is built around
// the weight stream rather than the tensor pipe:
//   * lane r of a warp owns weight row 32 q + r of a 128-row tile and reads its 64 codes of a k stage with four
//     coalesced 128-bit loads (a warp moves 512 contiguous bytes per load) plus its two fp16 scales, all issued before
//     anything else so that every warp has its whole share of W in flight at once;
//   * it dequantises in registers exactly as the large-M path does (bf16(d q), q8_common.cuh dequant16) and writes the
//     row into the warp's shared tile; ldmatrix hands the tile to mma.sync m16n8k16 (16 tokens x 8 rows x 16 k per
//     instruction, fp32 accumulation), so the arithmetic for 16 tokens costs no more issue slots than for one;
//   * the eight warps of a CTA take interleaved k stages of the same 32 rows and are reduced in shared memory in a
//     fixed order; when K is split across CTAs, they form a cluster along z and reduce through distributed shared
//     memory, again in a fixed order - no atomics, results do not depend on timing.
// Programmatic dependent launch (opt-in, see launch()): the weights do not depend on the preceding kernel, so the
// kernel streams them first and waits (griddepcontrol.wait) only before it reads X or the residual and writes Y; it
// lets its own dependents start early the same way. Without the launch attribute both instructions are no-ops.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdlib>

#include "internal.h"
#include "ptx.cuh"
#include "q8_common.cuh"

namespace idol {
namespace {

using namespace q8;

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kTokens = 16;                    // MMA rows: tokens (rows at or past M are zero)
constexpr int kMaxStagesPerCta = 2 * kWarps;   // each warp holds at most two stages of codes in registers
constexpr int kRowBytes = 64 * 2 + 16;         // one dequantised row of a stage in a warp tile (+16: no bank conflicts)
constexpr int kWarpTileBytes = 32 * kRowBytes;
constexpr int kMaxSplits = 8;

struct GemvArgs {
    const void* x;
    long long ldx;          // elements
    int stages_per_split;   // k stages per CTA (<= kMaxStagesPerCta)
};

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint16_t ld_stream_u16(const void* p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

template <bool kBF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (kBF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// grid: x = 32-row groups of the output window, z = K splits (a cluster along z when > 1); kThreads threads.
template <bool kBF16, typename OutT, int kFmt>
__global__ void __launch_bounds__(kThreads) q8_gemv_kernel(const Params p, const GemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int krange = a.stages_per_split * 64;
    const int xstride = krange * 2 + 16;                 // bytes per token row of the X tile
    uint8_t* xs = smem;                                  // [kTokens][krange] operand type
    uint8_t* wtile = xs + kTokens * xstride;             // [kWarps][32 rows][kRowBytes]
    float* red = reinterpret_cast<float*>(wtile);        // after the main loop: [kWarps][kTokens][32]
    float* total = reinterpret_cast<float*>(wtile + kWarps * kWarpTileBytes);  // [kTokens][32]

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int group = blockIdx.x;                        // 32-row group within the window
    const int row0 = p.row_begin + 32 * group;
    const int t128 = row0 / 128, q = (row0 / 32) % 4;
    const int ks0 = blockIdx.z * a.stages_per_split;
    const int ks1 = min(ks0 + a.stages_per_split, p.stages_total);

    // 1. This warp's codes and scales: stages ks0 + warp and ks0 + warp + kWarps, all loads in flight at once.
    // Q8_0: four 16-code loads and two fp16 scales per stage; Q4_K: two 32-code loads and one [A0, A1, B0, B1] load.
    constexpr int kCodeLoads = kFmt == kFmtQ4K ? 2 : 4;
    uint4 codes[2][kCodeLoads];
    uint16_t scales[2][2];
    uint4 prm[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int ks = ks0 + warp + i * kWarps;
        if (ks < ks1) {
            const uint8_t* chunk = p.tiles + ((long long)t128 * p.layout_stages + ks) * chunk_bytes<kFmt>();
            if constexpr (kFmt == kFmtQ4K) {
#pragma unroll
                for (int j = 0; j < 2; ++j) codes[i][j] = ld_stream_v4(chunk + q * 1024 + j * 512 + lane * 16);
                prm[i] = ld_stream_v4(chunk + kQ4KCodeBytes + (q * 32 + lane) * 16);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) codes[i][j] = ld_stream_v4(chunk + q * 2048 + j * 512 + lane * 16);
                scales[i][0] = ld_stream_u16(chunk + kChunkCodeBytes + q * 128 + lane * 2);
                scales[i][1] = ld_stream_u16(chunk + kChunkCodeBytes + q * 128 + 64 + lane * 2);
            }
        }
    }
    grid_dependents_launch();
    grid_dependency_wait();  // X and the residual written by the preceding kernel are visible from here on

    // 2. The X tile: tokens 0..15 (zero past M) x k in [64 ks0, 64 ks0 + krange) (zero past K), 16 bytes at a time.
    // Every load of a thread is issued before the first store, so the tile costs one memory latency, not eight.
    {
        constexpr int kPerThread = kTokens * (kMaxStagesPerCta * 64 / 8) / kThreads;
        const int chunks_per_row = krange / 8;
        const int k_begin = ks0 * 64;
        uint4 v[kPerThread];
#pragma unroll
        for (int i = 0; i < kPerThread; ++i) {
            const int idx = tid + i * kThreads;
            const int t = idx / chunks_per_row, c = idx % chunks_per_row;
            const int k = k_begin + c * 8;
            v[i] = make_uint4(0u, 0u, 0u, 0u);
            if (idx < kTokens * chunks_per_row && t < p.m && k < p.k)
                v[i] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) + (long long)t * a.ldx + k);
        }
#pragma unroll
        for (int i = 0; i < kPerThread; ++i) {
            const int idx = tid + i * kThreads;
            if (idx < kTokens * chunks_per_row)
                *reinterpret_cast<uint4*>(xs + (idx / chunks_per_row) * xstride + (idx % chunks_per_row) * 16) = v[i];
        }
    }
    __syncthreads();

    // 3. Dequantise each stage into the warp tile and multiply: 4 k16 steps x 4 blocks of 8 rows.
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.0f;
    uint8_t* my_tile = wtile + warp * kWarpTileBytes;
    const uint32_t tile_u32 = smem_u32(my_tile);
    const uint32_t xs_u32 = smem_u32(xs);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int ks = ks0 + warp + i * kWarps;
        if (ks >= ks1) break;
        uint32_t w[32];
        if constexpr (kFmt == kFmtQ4K) {
            const float4 pf = make_float4(__uint_as_float(prm[i].x), __uint_as_float(prm[i].y),
                                          __uint_as_float(prm[i].z), __uint_as_float(prm[i].w));
            dequant32_q4k<kBF16>(codes[i][0], pf.x, pf.z, w);
            dequant32_q4k<kBF16>(codes[i][1], pf.y, pf.w, w + 16);
        } else {
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const float d = __half2float(__ushort_as_half(scales[i][b]));
                const float2 dd = make_float2(d, d);
                const float2 ncd = make_float2(-32896.0f * d, -32896.0f * d);
                dequant16<kBF16>(codes[i][2 * b], dd, ncd, w + 16 * b);
                dequant16<kBF16>(codes[i][2 * b + 1], dd, ncd, w + 16 * b + 8);
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(my_tile + lane * kRowBytes + j * 16) =
                make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
        __syncwarp();
        const int kx = (ks - ks0) * 64;  // column of this stage in the X tile
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t af[4];
            {
                const int t = (lane % 8) + 8 * ((lane / 8) % 2);
                const int k = kx + 16 * kk + 8 * (lane / 16);
                ldmatrix_x4(xs_u32 + t * xstride + k * 2, af[0], af[1], af[2], af[3]);
            }
#pragma unroll
            for (int jp = 0; jp < 4; jp += 2) {
                uint32_t b00, b01, b10, b11;
                const int r = 8 * jp + (lane % 8) + 8 * (lane / 16);
                const int k = 16 * kk + 8 * ((lane / 8) % 2);
                ldmatrix_x4(tile_u32 + r * kRowBytes + k * 2, b00, b01, b10, b11);
                mma_16816<kBF16>(acc[jp], af, b00, b01);
                mma_16816<kBF16>(acc[jp + 1], af, b10, b11);
            }
        }
        __syncwarp();  // the tile is rewritten by the next stage
    }
    __syncthreads();  // every warp is done with the tiles: their space now holds the partial sums

    // 4. Partial sums [warp][token][row]: accumulator element e of block j is token g (+8 for e >= 2), row 8 j + 2 t
    // (+1 for odd e), with g = lane / 4 and t = lane % 4.
    {
        const int g = lane / 4, t = lane % 4;
        float* mine = red + warp * (kTokens * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            *reinterpret_cast<float2*>(mine + g * 32 + 8 * j + 2 * t) = make_float2(acc[j][0], acc[j][1]);
            *reinterpret_cast<float2*>(mine + (g + 8) * 32 + 8 * j + 2 * t) = make_float2(acc[j][2], acc[j][3]);
        }
    }
    __syncthreads();
    const int nsplit = gridDim.z;
    for (int idx = tid; idx < kTokens * 32; idx += kThreads) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[w * (kTokens * 32) + idx];
        if (nsplit == 1) {
            const int t = idx / 32;
            if (t < p.m) finish<OutT>(p, t, row0 + idx % 32, v);
        } else {
            total[idx] = v;
        }
    }
    if (nsplit > 1) {
        // 5. Cluster reduction in split order: CTA z finishes the outputs idx = z, z + nsplit, ...
        cluster_sync();
        const uint32_t z = cluster_ctarank();
        const uint32_t total_u32 = smem_u32(total);
        for (int idx = (int)z + tid * nsplit; idx < kTokens * 32; idx += kThreads * nsplit) {
            const int t = idx / 32;
            if (t >= p.m) continue;
            float v = 0.0f;
            for (int rk = 0; rk < nsplit; ++rk) v += ld_cluster_f32(map_to_rank(total_u32 + idx * 4, (uint32_t)rk));
            finish<OutT>(p, t, row0 + idx % 32, v);
        }
        cluster_sync();  // no CTA leaves while another may still read its partial sums
    }
}

int smem_bytes(int stages_per_split) {
    return kTokens * (stages_per_split * 64 * 2 + 16) + kWarps * kWarpTileBytes + kTokens * 32 * 4;
}

template <bool kBF16, typename OutT, int kFmt>
int launch_fmt(const Params& p, const GemvArgs& a, int groups, int splits, cudaStream_t stream) {
    auto kern = q8_gemv_kernel<kBF16, OutT, kFmt>;
    const int smem = smem_bytes(a.stages_per_split);
    static unsigned long long configured = 0;  // one bit per device: the shared-memory opt-in is set once
    int dev = 0;
    IDOL_CUDA(cudaGetDevice(&dev));
    if (!(configured >> (dev & 63) & 1ull)) {
        IDOL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_bytes(kMaxStagesPerCta)));
        configured |= 1ull << (dev & 63);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)groups, 1, (unsigned)splits);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    // Programmatic dependent launch is opt-in (IDOL_B200_PDL=1): inside CUDA graphs on B200 it measured no faster
    // than ordinary stream order for back-to-back small-M launches (5.45 against 6.5 us for 1 x 1024 x 3072).
    static const bool pdl = [] {
        const char* v = std::getenv("IDOL_B200_PDL");
        return v && v[0] == '1';
    }();
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (splits > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = (unsigned)splits;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    IDOL_CUDA(cudaLaunchKernelEx(&cfg, kern, p, a));
    return IDOL_OK;
}

template <bool kBF16, typename OutT>
int launch(int fmt, const Params& p, const GemvArgs& a, int groups, int splits, cudaStream_t stream) {
    return fmt == kFmtQ4K ? launch_fmt<kBF16, OutT, kFmtQ4K>(p, a, groups, splits, stream)
                          : launch_fmt<kBF16, OutT, kFmtQ8>(p, a, groups, splits, stream);
}

}  // namespace

// K splits for the streaming kernel: as few as the kMaxStagesPerCta limit allows. Measured on B200 (CUDA graphs,
// M = 1..16): a cluster launch costs more than the extra CTAs win back at these sizes, e.g. 4.2 us unsplit against
// 6.5 us with two splits for 1 x 1024 x 3072. 0 when K is too long for kMaxSplits splits.
int q8_gemv_splits(int device, int groups, int stages_total) {
    (void)device;
    (void)groups;
    int s = 1;
    while (s < kMaxSplits && (stages_total + s - 1) / s > kMaxStagesPerCta) s *= 2;
    return (stages_total + s - 1) / s > kMaxStagesPerCta ? 0 : s;
}

int q8_gemv(const GemmCall& c, const Params& p, int splits) {
    const int groups = (c.n_offset + c.n - p.row_begin + 31) / 32;
    GemvArgs a;
    a.x = c.x;
    a.ldx = c.ldx;
    a.stages_per_split = (p.stages_total + splits - 1) / splits;
    const bool bf16 = c.x_dtype == IDOL_BF16;
    const int fmt = c.w->format;
    if (c.y_dtype == IDOL_F32)
        return bf16 ? launch<true, float>(fmt, p, a, groups, splits, c.stream)
                    : launch<false, float>(fmt, p, a, groups, splits, c.stream);
    if (c.y_dtype == IDOL_BF16)
        return bf16 ? launch<true, __nv_bfloat16>(fmt, p, a, groups, splits, c.stream)
                    : launch<false, __nv_bfloat16>(fmt, p, a, groups, splits, c.stream);
    return bf16 ? launch<true, __half>(fmt, p, a, groups, splits, c.stream)
                : launch<false, __half>(fmt, p, a, groups, splits, c.stream);
}

}  // namespace idol
