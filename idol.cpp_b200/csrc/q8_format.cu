// q8_format.cu - the Q8_0 (and Q4_0, Q4_K) formats on the device.
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

// GGUF Q4_K -> the Q4_K tiled layout. A 144-byte Q4_K super-block covers 256 k of one row: fp16 d, fp16 dmin, 12 bytes
// packing a 6-bit scale and a 6-bit min for each of its eight 32-deep sub-blocks, then 128 bytes of 4-bit codes
// (sub-blocks 2g and 2g + 1 are the low and high nibbles of bytes 32 g .. 32 g + 31); weight = d sc code - dmin m
// (tools/idol_triton.py:64-82, tools/idol_packed.py:41-54). A 64-deep stage s is sub-blocks 2g, 2g + 1 of super-block
// s / 4 with g = s % 4. The repack stores A = d sc and B = dmin m as fp32 - both products of an 11-bit and a 6-bit
// integer, hence exact - and the codes two per byte in k order, so a kernel forms fl(A code - B): the reference's
// fp32 weight bit for bit (A code is exact too). One warp per (row tile, stage, quarter); lane r handles row
// 128 t + 32 q + r. The source must be 16-byte aligned (144 = 9 x 16, so every super-block is).
__global__ void q4_k_repack_kernel(const uint8_t* __restrict__ q4k, int n, int k, uint8_t* __restrict__ tiles,
                                   int64_t units) {
    const int ks = k_stages(k), sbs = k / 256;
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= units) return;
    const int lane = threadIdx.x % 32;
    const int q = (int)(unit % 4);
    const int64_t ts = unit / 4;
    const int s = (int)(ts % ks);
    const int t = (int)(ts / ks);
    const int64_t row = (int64_t)t * kTileRows + q * 32 + lane;
    uint32_t codes[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
    float4 prm = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (row < n) {
        const uint8_t* sb = q4k + (row * sbs + s / 4) * 144;
        const uint4 hdr = *reinterpret_cast<const uint4*>(sb);
        const int g = s % 4;
        uint8_t qs[32];
        *reinterpret_cast<uint4*>(qs) = *reinterpret_cast<const uint4*>(sb + 16 + 32 * g);
        *reinterpret_cast<uint4*>(qs + 16) = *reinterpret_cast<const uint4*>(sb + 32 + 32 * g);
        uint8_t sc8[12];
        *reinterpret_cast<uint32_t*>(sc8) = hdr.y;
        *reinterpret_cast<uint32_t*>(sc8 + 4) = hdr.z;
        *reinterpret_cast<uint32_t*>(sc8 + 8) = hdr.w;
        const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
        float a[2], bm[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * g + h;
            const int sc = j < 4 ? (sc8[j] & 63) : ((sc8[j + 4] & 15) | ((sc8[j - 4] >> 6) << 4));
            const int mn = j < 4 ? (sc8[j + 4] & 63) : ((sc8[j + 4] >> 4) | ((sc8[j] >> 6) << 4));
            a[h] = d * (float)sc;
            bm[h] = dmin * (float)mn;
        }
        prm = make_float4(a[0], a[1], bm[0], bm[1]);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t lo = (qs[2 * i] >> (4 * h)) & 15u, hi = (qs[2 * i + 1] >> (4 * h)) & 15u;
                codes[h][i / 4] |= (lo | (hi << 4)) << (8 * (i % 4));
            }
    }
    uint8_t* chunk = tiles + ((int64_t)t * ks + s) * kQ4KChunkBytes;
#pragma unroll
    for (int h = 0; h < 2; ++h)
        *reinterpret_cast<uint4*>(chunk + q * 1024 + h * 512 + lane * 16) =
            make_uint4(codes[h][0], codes[h][1], codes[h][2], codes[h][3]);
    *reinterpret_cast<float4*>(chunk + kQ4KCodeBytes + (q * 32 + lane) * 16) = prm;
}

__global__ void q4_k_dequant_kernel(const uint8_t* __restrict__ tiles, int n, int k, void* __restrict__ out,
                                    int dtype) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)n * k) return;
    const int64_t row = idx / k;
    const int col = (int)(idx % k);
    const int ks = k_stages(k);
    const int t = (int)(row / kTileRows), rq = (int)(row % kTileRows);
    const int q = rq / 32, r = rq % 32, s = col / 64, b = (col % 64) / 32, e = col % 32;
    const uint8_t* chunk = tiles + ((int64_t)t * ks + s) * kQ4KChunkBytes;
    const int code = (chunk[q * 1024 + b * 512 + r * 16 + e / 2] >> (4 * (e % 2))) & 15;
    const float* prm = reinterpret_cast<const float*>(chunk + kQ4KCodeBytes + (q * 32 + r) * 16);
    const float v = fmaf(prm[b], (float)code, -prm[2 + b]);  // A code is exact: one rounding, as A * code - B
    if (dtype == IDOL_F32)
        static_cast<float*>(out)[idx] = v;
    else if (dtype == IDOL_BF16)
        static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
    else
        static_cast<__half*>(out)[idx] = __float2half_rn(v);
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

cudaError_t launch_q4_k_repack(const uint8_t* q4k, int n, int k, uint8_t* tiles, cudaStream_t s) {
    const int64_t units = (int64_t)row_tiles(n) * k_stages(k) * 4;
    const int warps = 8;
    q4_k_repack_kernel<<<(unsigned)((units + warps - 1) / warps), warps * 32, 0, s>>>(q4k, n, k, tiles, units);
    return cudaGetLastError();
}

cudaError_t launch_q4_k_dequant(const uint8_t* tiles, int n, int k, void* w, int w_dtype, cudaStream_t s) {
    const int64_t total = (int64_t)n * k;
    if (total == 0) return cudaSuccess;
    q4_k_dequant_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(tiles, n, k, w, w_dtype);
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
