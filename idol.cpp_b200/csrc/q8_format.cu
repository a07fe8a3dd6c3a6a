// q8_format.cu - the Q8_0 formats on the device.
//
// GGUF Q8_0 (the interchange format): per output row, K/32 blocks of 34 bytes: fp16 scale d, then 32 int8 codes;
// weight = d * q (tools/idol_packed.py:28-31, tools/idol_triton.py:24-33).
//
// Tiled device layout (what the GEMM reads): the matrix is cut into chunks of 128 weight rows x 64 k (two Q8 blocks),
// ordered by (row tile, k stage). A chunk is the 8192 bytes of codes ordered [quarter q][block b][half h][lane r][16]
// (row = 128 t + 32 q + r, k = 64 s + 32 b + 16 h + j) followed by the 512 bytes of their fp16 scales ordered
// [quarter q][block b][lane r] - exactly one pipeline stage of one GEMM CTA, moved by a single bulk copy, in which a
// warp whose lane r owns row 32 q + r reads 512 contiguous bytes per 16-byte load. Rows past N and blocks past K/32
// are zero. Scale bits and codes are moved, never recomputed, so unpack(repack(x)) == x byte for byte.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"

namespace idol {

namespace {

// Byte offsets inside a chunk for lane r of quarter q, block b (code half h).
__device__ __forceinline__ int64_t chunk_of(int t, int s, int ks) { return ((int64_t)t * ks + s) * kChunkBytes; }
__device__ __forceinline__ int code_off(int q, int b, int h, int r) { return q * 2048 + b * 1024 + h * 512 + r * 16; }
__device__ __forceinline__ int scale_off(int q, int b, int r) { return kChunkCodeBytes + q * 128 + b * 64 + r * 2; }

// One warp per (row tile, stage, quarter, block); lane r handles row 128 t + 32 q + r.
__global__ void q8_repack_kernel(const uint8_t* __restrict__ q8, int n, int k, uint8_t* __restrict__ tiles,
                                 int64_t units) {
    const int kb = k / 32, ks = k_stages(k);
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= units) return;
    const int lane = threadIdx.x % 32;
    const int b = (int)(unit % 2), q = (int)((unit / 2) % 4);
    const int64_t ts = unit / 8;
    const int s = (int)(ts % ks);
    const int t = (int)(ts / ks);
    const int64_t row = (int64_t)t * kTileRows + q * 32 + lane;
    const int blk = 2 * s + b;
    uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint16_t d = 0;
    if (row < n && blk < kb) {
        // A 34-byte block starts on a 2-byte boundary: read it as 17 halfwords.
        const uint16_t* src = reinterpret_cast<const uint16_t*>(q8 + (row * kb + blk) * 34);
        d = src[0];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
    }
    uint8_t* chunk = tiles + chunk_of(t, s, ks);
    *reinterpret_cast<uint4*>(chunk + code_off(q, b, 0, lane)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(chunk + code_off(q, b, 1, lane)) = make_uint4(w[4], w[5], w[6], w[7]);
    *reinterpret_cast<uint16_t*>(chunk + scale_off(q, b, lane)) = d;
}

// GGUF Q4_0 -> the same tiled layout. An 18-byte Q4_0 block holds fp16 d and 16 bytes whose low nibbles are
// elements 0-15 and high nibbles elements 16-31, each worth d * (nibble - 8) (tools/idol_triton.py:48-61). That is
// exactly a Q8_0 block with codes nibble - 8 in [-8, 7] and the same d, so every kernel reading the tiled layout
// computes the reference's bf16(fp32(d) * code) for Q4_0 matrices unchanged. One warp per (row tile, stage, quarter,
// block) as in the Q8_0 repack; __vsub4 subtracts 8 from every byte without borrows between bytes.
__global__ void q4_0_repack_kernel(const uint8_t* __restrict__ q4, int n, int k, uint8_t* __restrict__ tiles,
                                   int64_t units) {
    const int kb = k / 32, ks = k_stages(k);
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= units) return;
    const int lane = threadIdx.x % 32;
    const int b = (int)(unit % 2), q = (int)((unit / 2) % 4);
    const int64_t ts = unit / 8;
    const int s = (int)(ts % ks);
    const int t = (int)(ts / ks);
    const int64_t row = (int64_t)t * kTileRows + q * 32 + lane;
    const int blk = 2 * s + b;
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
    uint16_t d = 0;
    if (row < n && blk < kb) {
        // An 18-byte block starts on a 2-byte boundary: read it as 9 halfwords.
        const uint16_t* src = reinterpret_cast<const uint16_t*>(q4 + (row * kb + blk) * 18);
        d = src[0];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t v = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
            lo[i] = __vsub4(v & 0x0F0F0F0Fu, 0x08080808u);
            hi[i] = __vsub4((v >> 4) & 0x0F0F0F0Fu, 0x08080808u);
        }
    }
    uint8_t* chunk = tiles + chunk_of(t, s, ks);
    *reinterpret_cast<uint4*>(chunk + code_off(q, b, 0, lane)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4*>(chunk + code_off(q, b, 1, lane)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint16_t*>(chunk + scale_off(q, b, lane)) = d;
}

__global__ void q8_unpack_kernel(const uint8_t* __restrict__ tiles, int n, int k, uint8_t* __restrict__ q8,
                                 int64_t units) {
    const int kb = k / 32, ks = k_stages(k);
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= units) return;
    const int lane = threadIdx.x % 32;
    const int b = (int)(unit % 2), q = (int)((unit / 2) % 4);
    const int64_t ts = unit / 8;
    const int s = (int)(ts % ks);
    const int t = (int)(ts / ks);
    const int64_t row = (int64_t)t * kTileRows + q * 32 + lane;
    const int blk = 2 * s + b;
    if (row >= n || blk >= kb) return;
    const uint8_t* chunk = tiles + chunk_of(t, s, ks);
    const uint4 lo = *reinterpret_cast<const uint4*>(chunk + code_off(q, b, 0, lane));
    const uint4 hi = *reinterpret_cast<const uint4*>(chunk + code_off(q, b, 1, lane));
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint16_t* dst = reinterpret_cast<uint16_t*>(q8 + (row * kb + blk) * 34);
    dst[0] = *reinterpret_cast<const uint16_t*>(chunk + scale_off(q, b, lane));
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
__global__ void q8_dequant_kernel(const uint8_t* __restrict__ tiles, int n, int k, void* __restrict__ out, int dtype) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)n * k) return;
    const int64_t row = idx / k;
    const int col = (int)(idx % k);
    const int ks = k_stages(k);
    const int t = (int)(row / kTileRows), rq = (int)(row % kTileRows);
    const int q = rq / 32, r = rq % 32, blk = col / 32, s = blk / 2, b = blk % 2, h = (col % 32) / 16, j = col % 16;
    const uint8_t* chunk = tiles + chunk_of(t, s, ks);
    const float qv = (float)(int8_t)chunk[code_off(q, b, h, r) + j];
    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(chunk + scale_off(q, b, r))));
    const float v = d * qv;
    if (dtype == IDOL_F32)
        static_cast<float*>(out)[idx] = v;
    else if (dtype == IDOL_BF16)
        static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
    else
        static_cast<__half*>(out)[idx] = __float2half_rn(v);
}

}  // namespace

cudaError_t launch_q8_repack(const uint8_t* q8, int n, int k, uint8_t* tiles, cudaStream_t s) {
    const int64_t units = (int64_t)row_tiles(n) * k_stages(k) * 8;
    const int warps = 8;
    q8_repack_kernel<<<(unsigned)((units + warps - 1) / warps), warps * 32, 0, s>>>(q8, n, k, tiles, units);
    return cudaGetLastError();
}

cudaError_t launch_q4_0_repack(const uint8_t* q4, int n, int k, uint8_t* tiles, cudaStream_t s) {
    const int64_t units = (int64_t)row_tiles(n) * k_stages(k) * 8;
    const int warps = 8;
    q4_0_repack_kernel<<<(unsigned)((units + warps - 1) / warps), warps * 32, 0, s>>>(q4, n, k, tiles, units);
    return cudaGetLastError();
}

cudaError_t launch_q8_unpack(const uint8_t* tiles, int n, int k, uint8_t* q8, cudaStream_t s) {
    const int64_t units = (int64_t)row_tiles(n) * k_stages(k) * 8;
    const int warps = 8;
    q8_unpack_kernel<<<(unsigned)((units + warps - 1) / warps), warps * 32, 0, s>>>(tiles, n, k, q8, units);
    return cudaGetLastError();
}

cudaError_t launch_q8_quantize(const float* w, int64_t rows, int64_t cols, uint8_t* q8, cudaStream_t s) {
    const int64_t blocks = rows * (cols / 32);
    if (blocks == 0) return cudaSuccess;
    const int warps = 8;
    q8_quantize_kernel<<<(unsigned)((blocks + warps - 1) / warps), warps * 32, 0, s>>>(w, blocks, q8);
    return cudaGetLastError();
}

cudaError_t launch_q8_dequant(const uint8_t* tiles, int n, int k, void* w, int w_dtype, cudaStream_t s) {
    const int64_t total = (int64_t)n * k;
    if (total == 0) return cudaSuccess;
    q8_dequant_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(tiles, n, k, w, w_dtype);
    return cudaGetLastError();
}

}  // namespace idol
