// q8_format.cu - the Q8_0 formats on the device.
//
// GGUF Q8_0 (the interchange format): per output row, K/32 blocks of 34 bytes: fp16 scale d, then 32 int8 codes;
// weight = d * q (tools/idol_packed.py:28-31, tools/idol_triton.py:24-33).
//
// Tiled device layout (what the GEMM reads): rows are grouped by 32. For row group g and Q8 block b, 1024 bytes of
// codes ordered [half h][row r][16 bytes] (k = 32 b + 16 h + j), so a warp whose lane r owns row 32 g + r reads 512
// contiguous bytes per 16-byte load; and 32 fp16 scales ordered by row. Rows past N are zero codes with a zero scale.
// The scale bits and the codes are moved, never recomputed, so unpack(repack(x)) == x byte for byte.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace idol {

namespace {

// One warp per (row group, block); lane r handles row 32 g + r.
__global__ void q8_repack_kernel(const uint8_t* __restrict__ q8, int n, int k, int8_t* __restrict__ codes,
                                 uint16_t* __restrict__ scales, int64_t units) {
    const int kb = k / 32;
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= units) return;
    const int lane = threadIdx.x % 32;
    const int64_t g = unit / kb;
    const int b = (int)(unit % kb);
    const int64_t row = g * 32 + lane;
    uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint16_t d = 0;
    if (row < n) {
        // A 34-byte block starts on a 2-byte boundary: read it as 17 halfwords.
        const uint16_t* src = reinterpret_cast<const uint16_t*>(q8 + (row * kb + b) * 34);
        d = src[0];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
    }
    int8_t* dst = codes + (g * kb + b) * 1024 + lane * 16;
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<uint4*>(dst + 512)[0] = make_uint4(w[4], w[5], w[6], w[7]);
    scales[(g * kb + b) * 32 + lane] = d;
}

__global__ void q8_unpack_kernel(const int8_t* __restrict__ codes, const uint16_t* __restrict__ scales, int n, int k,
                                 uint8_t* __restrict__ q8, int64_t units) {
    const int kb = k / 32;
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= units) return;
    const int lane = threadIdx.x % 32;
    const int64_t g = unit / kb;
    const int b = (int)(unit % kb);
    const int64_t row = g * 32 + lane;
    if (row >= n) return;
    const int8_t* src = codes + (g * kb + b) * 1024 + lane * 16;
    const uint4 lo = reinterpret_cast<const uint4*>(src)[0];
    const uint4 hi = reinterpret_cast<const uint4*>(src + 512)[0];
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint16_t* dst = reinterpret_cast<uint16_t*>(q8 + (row * kb + b) * 34);
    dst[0] = scales[(g * kb + b) * 32 + lane];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        dst[1 + 2 * i] = (uint16_t)(w[i] & 0xffffu);
        dst[2 + 2 * i] = (uint16_t)(w[i] >> 16);
    }
}

// round half away from zero, from its definition: floor(|v|) + floor(2 (|v| - floor(|v|))), signed. Every step is
// exact in fp32, so this matches gguf-py's np_roundf bit for bit.
__device__ __forceinline__ float round_half_away(float v) {
    const float a = fabsf(v);
    const float fl = floorf(a);
    const float r = __fadd_rn(fl, floorf(__fmul_rn(2.0f, __fsub_rn(a, fl))));
    return v < 0.0f ? -r : r;
}

// gguf-py 0.19.0 Q8_0.quantize_blocks semantics: d = amax / 127 (fp32), id = 1 / d (fp32, 0 when d == 0),
// q = round_half_away(w * id), scale stored as fp16(d). One warp per block, lane i owns element i.
__global__ void q8_quantize_kernel(const float* __restrict__ w, int64_t blocks, uint8_t* __restrict__ out) {
    const int64_t blk = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (blk >= blocks) return;
    const int lane = threadIdx.x % 32;
    const float x = w[blk * 32 + lane];
    float amax = fabsf(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
    const float q = round_half_away(__fmul_rn(x, id));
    // The block is 17 halfwords (it starts on a 2-byte boundary): halfword 0 is the fp16 scale, halfword 1 + i holds
    // codes 2 i and 2 i + 1. Even lanes pair their code with the next lane's and store one halfword each.
    const uint32_t code = (uint32_t)(uint8_t)(int8_t)(int)q;
    const uint32_t next = __shfl_down_sync(0xffffffffu, code, 1);
    uint16_t* dst = reinterpret_cast<uint16_t*>(out + blk * 34);
    if ((lane & 1) == 0) dst[1 + lane / 2] = (uint16_t)(code | (next << 8));
    if (lane == 1) dst[0] = __half_as_ushort(__float2half_rn(d));
}

// Tiled layout -> dense [n, k] weights d * q in fp32, bf16 or fp16 (bf16/fp16 rounded from the exact fp32 product).
__global__ void q8_dequant_kernel(const int8_t* __restrict__ codes, const uint16_t* __restrict__ scales, int n, int k,
                                  void* __restrict__ out, int dtype) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)n * k) return;
    const int64_t row = idx / k;
    const int col = (int)(idx % k);
    const int kb = k / 32;
    const int64_t g = row / 32;
    const int r = (int)(row % 32), b = col / 32, h = (col % 32) / 16, j = col % 16;
    const float q = (float)codes[((g * kb + b) * 2 + h) * 512 + r * 16 + j];
    const float d = __half2float(__ushort_as_half(scales[(g * kb + b) * 32 + r]));
    const float v = d * q;
    if (dtype == IDOL_F32)
        static_cast<float*>(out)[idx] = v;
    else if (dtype == IDOL_BF16)
        static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
    else
        static_cast<__half*>(out)[idx] = __float2half_rn(v);
}

}  // namespace

cudaError_t launch_q8_repack(const uint8_t* q8, int n, int k, int8_t* codes, uint16_t* scales, cudaStream_t s) {
    const int64_t units = (int64_t)((n + 31) / 32) * (k / 32);
    const int warps = 8;
    q8_repack_kernel<<<(unsigned)((units + warps - 1) / warps), warps * 32, 0, s>>>(q8, n, k, codes, scales, units);
    return cudaGetLastError();
}

cudaError_t launch_q8_unpack(const int8_t* codes, const uint16_t* scales, int n, int k, uint8_t* q8, cudaStream_t s) {
    const int64_t units = (int64_t)((n + 31) / 32) * (k / 32);
    const int warps = 8;
    q8_unpack_kernel<<<(unsigned)((units + warps - 1) / warps), warps * 32, 0, s>>>(codes, scales, n, k, q8, units);
    return cudaGetLastError();
}

cudaError_t launch_q8_quantize(const float* w, int64_t rows, int64_t cols, uint8_t* q8, cudaStream_t s) {
    const int64_t blocks = rows * (cols / 32);
    if (blocks == 0) return cudaSuccess;
    const int warps = 8;
    q8_quantize_kernel<<<(unsigned)((blocks + warps - 1) / warps), warps * 32, 0, s>>>(w, blocks, q8);
    return cudaGetLastError();
}

cudaError_t launch_q8_dequant(const int8_t* codes, const uint16_t* scales, int n, int k, void* w, int w_dtype,
                              cudaStream_t s) {
    const int64_t total = (int64_t)n * k;
    if (total == 0) return cudaSuccess;
    q8_dequant_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(codes, scales, n, k, w, w_dtype);
    return cudaGetLastError();
}

}  // namespace idol
