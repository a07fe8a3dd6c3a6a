// norms.cu - the row norms between the Q8_0 linears.
//
//   norm_rows : LayerNorm as the decoders run it (src/decoders.cpp:23-42): mean and variance over each row, fp32
//               normalisation with eps, optional affine gamma/beta, optional adaLN (1 + scale) and shift. The
//               reference sums in fp64; here each row is held in registers and reduced in fp32 with a two-pass
//               (mean, then squared deviations) warp-tree sum, which stays within 1e-6 relative of the fp64 result
//               for the widths used (dim <= 8192).
//   rms_heads : per-head L2 normalisation of q or k (src/decoders.cpp:74-86): x * sqrt(hd) / max(|x|, 1e-12) * gamma,
//               applied in place to `heads` column groups of hd values in each row (rows ld apart).
//
// Both are HBM-bound: one read and one write of the activations. One warp per row (norm_rows) or per (row, head)
// group (rms_heads); 16-byte loads, and one vector store per lane and chunk (8, 16 or 32 bytes by output type).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace idol {

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v) {
    if constexpr (sizeof(T) == 4) return v;
    else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(v);
    else return __half2float(v);
}
template <typename T>
__device__ __forceinline__ T from_f(float v) {
    if constexpr (sizeof(T) == 4) return v;
    else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(v);
    else return __float2half_rn(v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Elements per lane for a row of `dim` values: dim / 32, held in registers (dim % 256 == 0, dim <= 32 * kMaxPer).
constexpr int kMaxPer = 64;

template <typename TI, typename TO, int PER>
__global__ void norm_rows_kernel(const TI* __restrict__ x, long long ldx, TO* __restrict__ y, long long ldy,
                                 long long rows, int dim, float eps, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, const float* __restrict__ shift,
                                 const float* __restrict__ scale) {
    const long long row = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (row >= rows) return;
    const int lane = threadIdx.x % 32;
    constexpr int VEC = 16 / sizeof(TI);          // elements per 16-byte load
    const TI* xr = x + row * ldx;
    float v[PER];
    // Lane l reads elements [VEC (l + 32 i), VEC (l + 32 i) + VEC) for i < PER / VEC: coalesced 16-byte loads.
#pragma unroll
    for (int i = 0; i < PER / VEC; ++i) {
        const int c = VEC * (lane + 32 * i);
        const uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
        const TI* e = reinterpret_cast<const TI*>(&raw);
#pragma unroll
        for (int j = 0; j < VEC; ++j) v[i * VEC + j] = to_f(e[j]);
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i) s += v[i];
    const float mean = warp_sum(s) / (float)dim;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const float d = v[i] - mean;
        q = fmaf(d, d, q);
    }
    const float inv = 1.0f / sqrtf(warp_sum(q) / (float)dim + eps);
    TO* yr = y + row * ldy;
#pragma unroll
    for (int i = 0; i < PER / VEC; ++i) {
        const int c = VEC * (lane + 32 * i);
        alignas(16) TO out[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            float t = (v[i * VEC + j] - mean) * inv;
            if (gamma) t = t * gamma[c + j] + beta[c + j];
            if (scale) t = t * (1.0f + scale[c + j]) + shift[c + j];
            out[j] = from_f<TO>(t);
        }
        // One vector store of the lane's VEC outputs (8, 16 or 32 bytes; the row offset c is a multiple of VEC and
        // every caller passes 16-byte aligned rows).
        if constexpr (sizeof(TO) * VEC == 8) {
            *reinterpret_cast<uint2*>(yr + c) = *reinterpret_cast<const uint2*>(out);
        } else if constexpr (sizeof(TO) * VEC == 16) {
            *reinterpret_cast<uint4*>(yr + c) = *reinterpret_cast<const uint4*>(out);
        } else {
#pragma unroll
            for (int k = 0; k < (int)(sizeof(TO) * VEC / 16); ++k)
                reinterpret_cast<uint4*>(yr + c)[k] = reinterpret_cast<const uint4*>(out)[k];
        }
    }
}

// One warp per (row, head) with hd = 64: lane l owns elements 2 l, 2 l + 1.
template <typename T>
__global__ void rms_heads_kernel(T* __restrict__ x, long long ld, long long rows, int heads,
                                 const float* __restrict__ gamma) {
    const long long unit = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= rows * heads) return;
    const int lane = threadIdx.x % 32;
    const long long row = unit / heads;
    const int h = (int)(unit % heads);
    T* p = x + row * ld + h * 64 + 2 * lane;
    const float a = to_f(p[0]), b = to_f(p[1]);
    const float ss = warp_sum(a * a + b * b);
    const float mult = 8.0f / fmaxf(sqrtf(ss), 1e-12f);  // sqrt(64) = 8
    const float* g = gamma + h * 64 + 2 * lane;
    p[0] = from_f<T>(a * mult * g[0]);
    p[1] = from_f<T>(b * mult * g[1]);
}

// rms_heads over `total` bf16 heads of a row in one pass, the first `first` heads with gamma_a and the rest with
// gamma_b (the q and k blocks of a packed projection: first = heads, total = 2 heads). Eight lanes own one 64-wide
// head (16 bytes each), a warp four heads of one row. total % 4 == 0.
__global__ void rms_heads_vec_kernel(__nv_bfloat16* __restrict__ x, long long ld, long long rows, int total, int first,
                                     const float* __restrict__ gamma_a, const float* __restrict__ gamma_b) {
    const int groups = total / 4;
    const long long unit = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= rows * groups) return;
    const int lane = threadIdx.x % 32;
    const long long row = unit / groups;
    const int col = (int)(unit % groups) * 256 + lane * 8;
    const float* g = col / 64 < first ? gamma_a + col : gamma_b + (col - first * 64);
    const uint4 raw = *reinterpret_cast<const uint4*>(x + row * ld + col);
    const __nv_bfloat162* pr = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(pr[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
    for (int o = 4; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float mult = 8.0f / fmaxf(sqrtf(ss), 1e-12f);  // sqrt(64) = 8
    const float4 g0 = *reinterpret_cast<const float4*>(g), g1 = *reinterpret_cast<const float4*>(g + 4);
    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    uint4 out;
    uint32_t* po = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 o2 = __floats2bfloat162_rn(v[2 * i] * mult * gg[2 * i], v[2 * i + 1] * mult * gg[2 * i + 1]);
        po[i] = *reinterpret_cast<const uint32_t*>(&o2);
    }
    *reinterpret_cast<uint4*>(x + row * ld + col) = out;
}

bool rms_vec_ok(const void* x, long long ld, int total, const float* ga, const float* gb) {
    return total % 4 == 0 && ld % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(ga) % 16 == 0 && reinterpret_cast<uintptr_t>(gb) % 16 == 0;
}

cudaError_t launch_rms_vec(void* x, long long ld, long long rows, int total, int first, const float* ga,
                           const float* gb, cudaStream_t s) {
    const long long units = rows * (total / 4);
    const int warps = 8;
    rms_heads_vec_kernel<<<(unsigned)((units + warps - 1) / warps), warps * 32, 0, s>>>(
        static_cast<__nv_bfloat16*>(x), ld, rows, total, first, ga, gb);
    return cudaGetLastError();
}

template <typename TI, typename TO>
cudaError_t launch_norm(const void* x, long long ldx, void* y, long long ldy, long long rows, int dim, float eps,
                        const float* gamma, const float* beta, const float* shift, const float* scale, cudaStream_t s) {
    const int per = dim / 32;
    const int warps = 8;
    const unsigned grid = (unsigned)((rows + warps - 1) / warps);
#define IDOL_NORM_CASE(P)                                                                                   \
    case P:                                                                                                 \
        norm_rows_kernel<TI, TO, P><<<grid, warps * 32, 0, s>>>(static_cast<const TI*>(x), ldx,            \
                                                                static_cast<TO*>(y), ldy, rows, dim, eps, \
                                                                gamma, beta, shift, scale);                \
        break;
    switch (per) {
        IDOL_NORM_CASE(8)
        IDOL_NORM_CASE(16)
        IDOL_NORM_CASE(24)
        IDOL_NORM_CASE(32)
        IDOL_NORM_CASE(48)
        IDOL_NORM_CASE(64)
        default: return cudaErrorInvalidValue;
    }
#undef IDOL_NORM_CASE
    return cudaGetLastError();
}

}  // namespace

bool norm_dim_ok(int dim) {
    const int per = dim / 32;
    return dim % 256 == 0 && (per == 8 || per == 16 || per == 24 || per == 32 || per == 48 || per == 64);
}

cudaError_t launch_norm_rows(const void* x, int x_dtype, long long ldx, void* y, int y_dtype, long long ldy,
                             long long rows, int dim, float eps, const float* gamma, const float* beta,
                             const float* shift, const float* scale, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    if (x_dtype == IDOL_BF16 && y_dtype == IDOL_BF16)
        return launch_norm<__nv_bfloat16, __nv_bfloat16>(x, ldx, y, ldy, rows, dim, eps, gamma, beta, shift, scale, s);
    if (x_dtype == IDOL_F32 && y_dtype == IDOL_BF16)
        return launch_norm<float, __nv_bfloat16>(x, ldx, y, ldy, rows, dim, eps, gamma, beta, shift, scale, s);
    if (x_dtype == IDOL_F32 && y_dtype == IDOL_F32)
        return launch_norm<float, float>(x, ldx, y, ldy, rows, dim, eps, gamma, beta, shift, scale, s);
    if (x_dtype == IDOL_F16 && y_dtype == IDOL_F16)
        return launch_norm<__half, __half>(x, ldx, y, ldy, rows, dim, eps, gamma, beta, shift, scale, s);
    if (x_dtype == IDOL_BF16 && y_dtype == IDOL_F32)
        return launch_norm<__nv_bfloat16, float>(x, ldx, y, ldy, rows, dim, eps, gamma, beta, shift, scale, s);
    return cudaErrorInvalidValue;
}

cudaError_t launch_rms_heads(void* x, int dtype, long long ld, long long rows, int heads, const float* gamma,
                             cudaStream_t s) {
    const long long units = rows * heads;
    if (units == 0) return cudaSuccess;
    if (dtype == IDOL_BF16 && rms_vec_ok(x, ld, heads, gamma, gamma))
        return launch_rms_vec(x, ld, rows, heads, heads, gamma, gamma, s);
    const int warps = 8;
    const unsigned grid = (unsigned)((units + warps - 1) / warps);
    if (dtype == IDOL_BF16)
        rms_heads_kernel<__nv_bfloat16><<<grid, warps * 32, 0, s>>>(static_cast<__nv_bfloat16*>(x), ld, rows, heads,
                                                                    gamma);
    else if (dtype == IDOL_F32)
        rms_heads_kernel<float><<<grid, warps * 32, 0, s>>>(static_cast<float*>(x), ld, rows, heads, gamma);
    else if (dtype == IDOL_F16)
        rms_heads_kernel<__half><<<grid, warps * 32, 0, s>>>(static_cast<__half*>(x), ld, rows, heads, gamma);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_rms_heads_qk(void* x, long long ld, long long rows, int heads, const float* gamma_q,
                                const float* gamma_k, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    if (rms_vec_ok(x, ld, 2 * heads, gamma_q, gamma_k))
        return launch_rms_vec(x, ld, rows, 2 * heads, heads, gamma_q, gamma_k, s);
    const cudaError_t e = launch_rms_heads(x, IDOL_BF16, ld, rows, heads, gamma_q, s);
    if (e != cudaSuccess) return e;
    return launch_rms_heads(static_cast<__nv_bfloat16*>(x) + heads * 64, IDOL_BF16, ld, rows, heads, gamma_k, s);
}

}  // namespace idol
