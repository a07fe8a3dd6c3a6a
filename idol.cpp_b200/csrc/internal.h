// internal.h - host-side declarations shared by the library's translation units (not part of the C-ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "idol_b200.h"  // include/ (on the compiler include path)

namespace idol {

// Device-resident Q8_0 matrix in the tiled layout (see q8_format.cu):
//   codes : ceil(N/32) row groups x K/32 blocks x [2 halves][32 rows][16 bytes] int8
//   scales: ceil(N/32) row groups x K/32 blocks x [32 rows] fp16 (the Q8_0 block scale d, bit for bit)
struct Q8Matrix {
    int device = 0;
    int n = 0, k = 0;         // out, in features
    int groups = 0;           // ceil(n / 32)
    int8_t* codes = nullptr;
    uint16_t* scales = nullptr;
    float* bias = nullptr;    // n floats on the device, or nullptr
    bool owns = true;         // false for matrices over caller memory
};

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define IDOL_CUDA(call)                                           \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return ::idol::cuda_fail(e_, #call); \
    } while (0)

inline int64_t codes_bytes(int n, int k) { return (int64_t)((n + 31) / 32) * 32 * k; }
inline int64_t scales_bytes(int n, int k) { return (int64_t)((n + 31) / 32) * 32 * (k / 32) * 2; }

// Format kernels (q8_format.cu).
cudaError_t launch_q8_repack(const uint8_t* q8, int n, int k, int8_t* codes, uint16_t* scales, cudaStream_t s);
cudaError_t launch_q8_unpack(const int8_t* codes, const uint16_t* scales, int n, int k, uint8_t* q8, cudaStream_t s);
cudaError_t launch_q8_quantize(const float* w, int64_t rows, int64_t cols, uint8_t* q8, cudaStream_t s);
cudaError_t launch_q8_dequant(const int8_t* codes, const uint16_t* scales, int n, int k, void* w, int w_dtype,
                              cudaStream_t s);

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
};
int q8_gemm(const GemmCall& c);

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

// Attention (attention.cu).
struct AttentionCall {
    const void* q;
    const void* k;
    const void* v;
    void* out;
    long long lq, lk, ldq, ldkv, ldo;
    int heads, head_dim, batch;
    cudaStream_t stream;
};
int attention(const AttentionCall& c);

// Per translation unit readers of the sticky device error word (ptx.cuh IDOL_DEVICE_ERROR_READER).
cudaError_t take_device_error_gemm(unsigned int* flags);
cudaError_t take_device_error_attention(unsigned int* flags);

cudaError_t launch_gaussian_heads(const void* raw, int raw_dtype, long long points, long long ld, float* out,
                                  cudaStream_t s);

}  // namespace idol

// The opaque C-ABI handle around a device matrix (shared by the translation units that compose kernels).
struct idol_q8_matrix {
    idol::Q8Matrix m;
};
