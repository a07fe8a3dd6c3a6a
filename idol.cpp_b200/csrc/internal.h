// internal.h - host-side declarations shared by the library's translation units (not part of the C-ABI).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "idol_b200.h"  // include/ (on the compiler include path)

namespace idol {

// Tiled device layout of a Q8_0 matrix (see q8_format.cu): stage chunks of 128 weight rows x 64 k, each
// kChunkBytes = 8192 bytes of codes ([quarter][block][half][lane][16]) followed by 512 bytes of fp16 scales
// ([quarter][block][lane]), chunks ordered by (row tile, k stage). Rows past N and blocks past K/32 are zero.
constexpr int kTileRows = 128;
constexpr int kTileK = 64;
constexpr int kChunkCodeBytes = 8192;
constexpr int kChunkBytes = 8704;
__host__ __device__ inline int row_tiles(int n) { return (n + kTileRows - 1) / kTileRows; }
__host__ __device__ inline int k_stages(int k) { return (k + kTileK - 1) / kTileK; }
__host__ __device__ inline int64_t tiled_bytes(int n, int k) {
    return (int64_t)row_tiles(n) * k_stages(k) * kChunkBytes;
}

// Tiled device layout of a Q4_K matrix (see q8_format.cu): the same chunk grid, each chunk 4096 bytes of 4-bit codes
// ([quarter][block][lane][16]: byte i holds the codes of k = 2i (low nibble) and 2i + 1 (high nibble) of the 32-deep
// sub-block) followed by 2048 bytes of fp32 [A0, A1, B0, B1] per row ([quarter][lane]), weight = A code - B.
constexpr int kQ4KCodeBytes = 4096;
constexpr int kQ4KChunkBytes = 6144;
__host__ __device__ inline int64_t q4k_tiled_bytes(int n, int k) {
    return (int64_t)row_tiles(n) * k_stages(k) * kQ4KChunkBytes;
}

// Weight formats a matrix handle can hold.
enum : int { kFmtQ8 = 0, kFmtQ4K = 1 };
template <int kFmt>
__host__ __device__ constexpr int chunk_bytes() { return kFmt == kFmtQ4K ? kQ4KChunkBytes : kChunkBytes; }

// Device-resident quantized matrix in a tiled layout.
struct Q8Matrix {
    int device = 0;
    int n = 0, k = 0;         // out, in features
    uint8_t* tiles = nullptr;
    float* bias = nullptr;    // n floats on the device, or nullptr
    bool owns = true;         // false for matrices over caller memory
    int format = kFmtQ8;      // kFmtQ8: Q8_0 (and converted Q4_0) tiles; kFmtQ4K: Q4_K tiles
};

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define IDOL_CUDA(call)                                           \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return ::idol::cuda_fail(e_, #call); \
    } while (0)

// Format kernels (q8_format.cu).
cudaError_t launch_q8_repack(const uint8_t* q8, int n, int k, uint8_t* tiles, cudaStream_t s);
cudaError_t launch_q8_unpack(const uint8_t* tiles, int n, int k, uint8_t* q8, cudaStream_t s);
cudaError_t launch_q4_0_repack(const uint8_t* q4, int n, int k, uint8_t* tiles, cudaStream_t s);
cudaError_t launch_q8_quantize(const float* w, int64_t rows, int64_t cols, uint8_t* q8, cudaStream_t s);
cudaError_t launch_q8_dequant(const uint8_t* tiles, int n, int k, void* w, int w_dtype, cudaStream_t s);
cudaError_t launch_q4_k_repack(const uint8_t* q4k, int n, int k, uint8_t* tiles, cudaStream_t s);
cudaError_t launch_q4_k_dequant(const uint8_t* tiles, int n, int k, void* w, int w_dtype, cudaStream_t s);

// The Q8_0 GEMM (q8_gemm.cu).
struct GemmCall {
    const Q8Matrix* w;
    const void* x;
    int x_dtype;
    int64_t m, ldx;
    int n_offset, n;
    const void* residual;
    int64_t ldr;
    int act;
    int flags;
    void* y;
    int y_dtype;
    int64_t ldy;
    cudaStream_t stream;
    // Optional rms_heads of the output (bf16 or f16, window starting at column 0, no activation or residual):
    // columns [0, head_split) with head_gamma_a, [head_split, head_cols) with head_gamma_b, heads of 64. Fused into
    // the epilogue where the GEMM leaves through a staging tile, else a separate launch right after it.
    const float* head_gamma_a = nullptr;
    const float* head_gamma_b = nullptr;
    int head_cols = 0, head_split = 0;
};
int q8_gemm(const GemmCall& c);
// While one of these lives on the calling thread, q8_gemm allocates nothing of its own: calls that would take the
// large-M dense path (which dequantises into a scratch the library allocates per device and stream) take the fused
// kernel instead. The allocation-free entry points run their GEMMs inside one.
struct NoScratchScope {
    NoScratchScope();
    ~NoScratchScope();
    NoScratchScope(const NoScratchScope&) = delete;
    NoScratchScope& operator=(const NoScratchScope&) = delete;
};
// The integer-activation form of the same linear (q8_int8act.cu): flags unused; workspace for the quantized
// activations (int8act_workspace_bytes).
int64_t int8act_workspace_bytes(int64_t m, int k);
int q8_gemm_int8act_check(const GemmCall& c, void* workspace, int64_t workspace_bytes);  // arguments only
int q8_gemm_int8act(const GemmCall& c, void* workspace, int64_t workspace_bytes);

// Tensor-map creation through the driver entry point (no link-time dependency on libcuda).
int encode_tmap_nd(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const cuuint64_t* dims,
                   const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swizzle);
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

int num_sms(int device);

// Row norms (norms.cu).
bool norm_dim_ok(int dim);
cudaError_t launch_norm_rows(const void* x, int x_dtype, long long ldx, void* y, int y_dtype, long long ldy,
                             long long rows, int dim, float eps, const float* gamma, const float* beta,
                             const float* shift, const float* scale, cudaStream_t s);
cudaError_t launch_rms_heads(void* x, int dtype, long long ld, long long rows, int heads, const float* gamma,
                             cudaStream_t s);
// rms_heads of adjacent bf16 q and k blocks (heads x 64 columns each, rows ld apart) in one launch.
cudaError_t launch_rms_heads_qk(void* x, long long ld, long long rows, int heads, const float* gamma_q,
                                const float* gamma_k, cudaStream_t s);

// Attention (attention.cu).
struct AttentionCall {
    const void* q;
    const void* k;
    const void* v;
    void* out;
    long long lq, lk, ldq, ldkv, ldo;
    int heads, head_dim, batch;
    cudaStream_t stream;
    bool out_f32;  // fp32 output rows instead of bf16 (false when left out of an aggregate initialiser)
};
int attention(const AttentionCall& c);

// Per translation unit readers of the sticky device error word (ptx.cuh IDOL_DEVICE_ERROR_READER).
cudaError_t take_device_error_gemm(unsigned int* flags);
cudaError_t take_device_error_attention(unsigned int* flags);

cudaError_t launch_gaussian_heads(const void* raw, int raw_dtype, long long points, long long ld, float* out,
                                  cudaStream_t s);
// The decoders' input (in_proj of 3 coordinates + bias + pos_embed, bf16 out) and the dense fp32 key/value projection
// of the condition rows (block.cu).
cudaError_t launch_decoder_input(const float* points, long long rows, int dim, const float* w, const float* b,
                                 const float* freqs, int fd, __nv_bfloat16* out, cudaStream_t s);
// kv = cond w^T + b as bf16 [rows, cols]; with k_gamma, the first cols / 2 columns (the keys) also get rms_heads
// (heads of 64) with that gamma, fused into the projection when cdim is 16.
cudaError_t launch_kv_project(const float* cond, long long rows, int cdim, const float* w, const float* b, int cols,
                              __nv_bfloat16* kv, cudaStream_t s, const float* k_gamma = nullptr, int heads = 0);

}  // namespace idol

// The opaque C-ABI handle around a device matrix (shared by the translation units that compose kernels).
struct idol_q8_matrix {
    idol::Q8Matrix m;
};
