// q8_int8act.cu - the Q8_0 linear on integer activations: the reference's second CPU kernel (src/kernels.cpp:368-479,
// quantize_activations + vnni_task + gemm_quant_int8, which the reference selects with set_quant_kernel(1) /
// IDOL_QUANT_KERNEL and which its CPU uses by default where AVX-VNNI exists), on the GPU with the same arithmetic, so
// its outputs equal the reference's bit for bit:
//   * activations, per (token, 32-deep group): amax = max |x|, sa = amax / 127, qa = rint(x * (127 / amax)) (round to
//     nearest even; 0 when amax is 0), qsum = sum qa - one warp per group (quantize_kernel);
//   * per output, groups in k order: the integer dot sum (q + 128) qa (exact in int32: 32 terms below 2^15; dp4a on
//     the signed codes plus 128 qsum), then t = fma(float(dot), d * sa, fma(-128 d, sa * float(qsum), t)) with each
//     product rounded as the reference's vector multiplies round them (d = the block's fp16 scale; -128 d is the
//     8-bit panel's stored minimum, exact) - the float order of vnni_task;
//   * then the epilogue of finish_tile (src/kernels.cpp:212-241): bias, residual, activation (the activations of the
//     tcgen05 GEMM's epilogue, q8_common.cuh).
// The tensor cores cannot take this path: a tcgen05 MMA accumulates across k without the per-group float rescaling
// the reference applies, so the dot products run on the integer pipe (dp4a), 32 tokens x 64 weight rows per CTA with
// both operands of a group staged in shared memory. It is the reference's secondary kernel, not the hot path: the
// tcgen05 GEMM (q8_gemm.cu) serves the float kernel the reference uses in production.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"
#include "q8_common.cuh"

namespace idol {
namespace {

constexpr int kTokTile = 32;   // tokens per CTA
constexpr int kRowTile = 64;   // weight rows per CTA
constexpr int kThreads = 128;  // 16 x 8 threads, 4 x 4 outputs each

__device__ __forceinline__ float load_act(const void* x, int dtype, long long i) {
    if (dtype == IDOL_F32) return static_cast<const float*>(x)[i];
    if (dtype == IDOL_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(x)[i]);
    return __half2float(static_cast<const __half*>(x)[i]);
}

// One warp per (token, group): lane = k within the group.
__global__ void quantize_kernel(const void* __restrict__ x, int dtype, long long ldx, int m, int k,
                                int8_t* __restrict__ qa, float* __restrict__ scale, int* __restrict__ qsum) {
    const int ng = k / 32;
    const long long unit = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= (long long)m * ng) return;
    const int lane = threadIdx.x % 32;
    const int r = (int)(unit / ng), g = (int)(unit % ng);
    const float v = load_act(x, dtype, (long long)r * ldx + g * 32 + lane);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    const int q = __float2int_rn(v * inv);
    int sum = q;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    qa[(long long)r * k + g * 32 + lane] = (int8_t)q;
    if (lane == 0) {
        scale[unit] = amax / 127.0f;
        qsum[unit] = sum;
    }
}

template <typename OutT>
__device__ __forceinline__ float out_to_f(OutT v) {
    if constexpr (sizeof(OutT) == 4) return v;
    else if constexpr (std::is_same<OutT, __nv_bfloat16>::value) return __bfloat162float(v);
    else return __half2float(v);
}

template <typename OutT>
__device__ __forceinline__ OutT f_to_out(float v) {
    if constexpr (sizeof(OutT) == 4) return v;
    else if constexpr (std::is_same<OutT, __nv_bfloat16>::value) return __float2bfloat16_rn(v);
    else return __float2half_rn(v);
}

struct Int8Args {
    const uint8_t* tiles;   // the matrix's tiled layout (codes and fp16 scales)
    const float* bias;      // n floats or nullptr
    const int8_t* qa;       // [m, k]
    const float* scale;     // [m, k / 32]
    const int* qsum;        // [m, k / 32]
    const void* residual;   // window layout, rows ldr apart, or nullptr
    void* y;                // window layout, rows ldy apart
    long long ldr, ldy;
    int m, k, n, layout_stages, n_offset, n_count, act;
};

// grid: x = 64-row slices of the window (from row n_offset), y = 32-token slices. Thread (ty, tx): tokens 4 ty..,
// rows 4 tx...
template <typename OutT>
__global__ void __launch_bounds__(kThreads) int8act_kernel(const Int8Args a) {
    __shared__ __align__(16) int w_s[kRowTile][9];      // 32 code bytes per row (+1 word: no bank conflicts)
    __shared__ __align__(16) int x_s[kTokTile][9];      // 32 activation bytes per token
    __shared__ float d_s[kRowTile], sa_s[kTokTile], sq_s[kTokTile];
    __shared__ int qs_s[kTokTile];
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    const int row0 = a.n_offset + blockIdx.x * kRowTile;
    const int tok0 = blockIdx.y * kTokTile;
    const int ng = a.k / 32;
    float t[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) t[i][j] = 0.0f;

    for (int g = 0; g < ng; ++g) {
        // Codes: 64 rows x 2 halves of 16 bytes (one load per thread); scales; the tokens' activations.
        {
            const int r = tid / 2, h = tid % 2;
            const int row = row0 + r;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (row < a.n && row < a.n_offset + a.n_count) {
                const uint8_t* chunk = a.tiles + ((long long)(row / kTileRows) * a.layout_stages + g / 2) * kChunkBytes;
                v = *reinterpret_cast<const uint4*>(chunk + ((row % kTileRows) / 32) * 2048 + (2 * (g % 2) + h) * 512 +
                                                    (row % 32) * 16);
                if (h == 0) {
                    const __half d = *reinterpret_cast<const __half*>(chunk + kChunkCodeBytes +
                                                                       ((row % kTileRows) / 32) * 128 + (g % 2) * 64 +
                                                                       (row % 32) * 2);
                    d_s[r] = __half2float(d);
                }
            } else if (h == 0) {
                d_s[r] = 0.0f;
            }
            w_s[r][4 * h + 0] = (int)v.x;
            w_s[r][4 * h + 1] = (int)v.y;
            w_s[r][4 * h + 2] = (int)v.z;
            w_s[r][4 * h + 3] = (int)v.w;
        }
        if (tid < 2 * kTokTile) {
            const int tk = tid / 2, h = tid % 2;
            const int tok = tok0 + tk;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (tok < a.m) v = *reinterpret_cast<const uint4*>(a.qa + (long long)tok * a.k + g * 32 + h * 16);
            x_s[tk][4 * h + 0] = (int)v.x;
            x_s[tk][4 * h + 1] = (int)v.y;
            x_s[tk][4 * h + 2] = (int)v.z;
            x_s[tk][4 * h + 3] = (int)v.w;
            if (h == 0) {
                const float s = tok < a.m ? a.scale[(long long)tok * ng + g] : 0.0f;
                const int qs = tok < a.m ? a.qsum[(long long)tok * ng + g] : 0;
                sa_s[tk] = s;
                qs_s[tk] = qs;
                sq_s[tk] = s * (float)qs;
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tk = 4 * ty + i;
            const float s = sa_s[tk], sq = sq_s[tk];
            const int qs128 = 128 * qs_s[tk];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = 4 * tx + j;
                int dot = 0;
#pragma unroll
                for (int wd = 0; wd < 8; ++wd) dot = __dp4a(w_s[r][wd], x_s[tk][wd], dot);
                const float d = d_s[r];
                t[i][j] = fmaf((float)(dot + qs128), d * s, fmaf(-128.0f * d, sq, t[i][j]));
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int tok = tok0 + 4 * ty + i;
        if (tok >= a.m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int row = row0 + 4 * tx + j;
            if (row >= a.n || row >= a.n_offset + a.n_count) continue;
            const int col = row - a.n_offset;
            float v = t[i][j] + (a.bias ? a.bias[row] : 0.0f);
            if (a.residual) v += out_to_f(static_cast<const OutT*>(a.residual)[(long long)tok * a.ldr + col]);
            static_cast<OutT*>(a.y)[(long long)tok * a.ldy + col] = f_to_out<OutT>(q8::activate(v, a.act));
        }
    }
}

int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

}  // namespace

int64_t int8act_workspace_bytes(int64_t m, int k) {
    if (m < 0 || k < 32 || k % 32) return -1;
    return align256(m * k) + 2 * align256(m * (k / 32) * 4);
}

int q8_gemm_int8act_check(const GemmCall& c, void* workspace, int64_t workspace_bytes) {
    const Q8Matrix& w = *c.w;
    if (w.format != kFmtQ8)
        return fail(IDOL_ERR_UNSUPPORTED, "q8_gemm_int8act: the integer-activation kernel takes Q8_0 matrices");
    if (c.m < 0 || c.m > 65535LL * kTokTile) return fail(IDOL_ERR_INVALID, "q8_gemm_int8act: m out of range");
    if (c.n < 0 || c.n_offset < 0 || c.n_offset + c.n > w.n)
        return fail(IDOL_ERR_INVALID, "q8_gemm_int8act: column window");
    if (c.m == 0 || c.n == 0) return IDOL_OK;
    if (c.x_dtype != IDOL_F32 && c.x_dtype != IDOL_BF16 && c.x_dtype != IDOL_F16)
        return fail(IDOL_ERR_UNSUPPORTED, "q8_gemm_int8act: activations must be f32, bf16 or f16");
    if (c.y_dtype != IDOL_F32 && c.y_dtype != IDOL_BF16 && c.y_dtype != IDOL_F16)
        return fail(IDOL_ERR_UNSUPPORTED, "q8_gemm_int8act: output must be f32, bf16 or f16");
    if (!c.x || !c.y || c.ldx < w.k || c.ldy < c.n || (c.residual && c.ldr < c.n))
        return fail(IDOL_ERR_INVALID, "q8_gemm_int8act: pointers or row strides");
    if (c.act < IDOL_ACT_NONE || c.act > IDOL_ACT_SILU) return fail(IDOL_ERR_INVALID, "q8_gemm_int8act: activation");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 ||
        workspace_bytes < int8act_workspace_bytes(c.m, w.k))
        return fail(IDOL_ERR_INVALID, "q8_gemm_int8act: workspace smaller than idol_b200_q8_gemm_int8act_workspace_"
                                      "bytes or not 256-byte aligned");
    return IDOL_OK;
}

int q8_gemm_int8act(const GemmCall& c, void* workspace, int64_t workspace_bytes) {
    const int rc = q8_gemm_int8act_check(c, workspace, workspace_bytes);
    if (rc != IDOL_OK || c.m == 0 || c.n == 0) return rc;
    const Q8Matrix& w = *c.w;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    Int8Args a;
    a.tiles = w.tiles;
    a.bias = w.bias;
    a.qa = reinterpret_cast<int8_t*>(ws);
    a.scale = reinterpret_cast<float*>(ws + align256(c.m * w.k));
    a.qsum = reinterpret_cast<int*>(ws + align256(c.m * w.k) + align256(c.m * (w.k / 32) * 4));
    a.residual = c.residual;
    a.y = c.y;
    a.ldr = c.ldr;
    a.ldy = c.ldy;
    a.m = (int)c.m;
    a.k = w.k;
    a.n = w.n;
    a.layout_stages = k_stages(w.k);
    a.n_offset = c.n_offset;
    a.n_count = c.n;
    a.act = c.act;
    const long long units = c.m * (w.k / 32);
    quantize_kernel<<<(unsigned)((units + 7) / 8), 256, 0, c.stream>>>(c.x, c.x_dtype, c.ldx, (int)c.m, w.k,
                                                                       const_cast<int8_t*>(a.qa),
                                                                       const_cast<float*>(a.scale),
                                                                       const_cast<int*>(a.qsum));
    IDOL_CUDA(cudaGetLastError());
    const dim3 grid((unsigned)((c.n + kRowTile - 1) / kRowTile), (unsigned)((c.m + kTokTile - 1) / kTokTile));
    if (c.y_dtype == IDOL_F32) int8act_kernel<float><<<grid, kThreads, 0, c.stream>>>(a);
    else if (c.y_dtype == IDOL_BF16) int8act_kernel<__nv_bfloat16><<<grid, kThreads, 0, c.stream>>>(a);
    else int8act_kernel<__half><<<grid, kThreads, 0, c.stream>>>(a);
    IDOL_CUDA(cudaGetLastError());
    return IDOL_OK;
}

}  // namespace idol
