// capi.cu - the extern "C" entry points declared in include/idol_b200.h, and the host helpers they share.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "internal.h"

namespace idol {

namespace {
thread_local std::string g_last_error;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int g_sms[64] = {0};
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return IDOL_ERR_CUDA;
}

int num_sms(int device) {
    if (device < 0 || device >= 64) return 148;
    if (!g_sms[device]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
        g_sms[device] = v;
    }
    return g_sms[device];
}

int encode_tmap_nd(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const cuuint64_t* dims,
                   const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(IDOL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(IDOL_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return IDOL_OK;
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(IDOL_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(IDOL_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return IDOL_OK;
}

}  // namespace idol

using idol::fail;

namespace {

bool shape_ok(int out, int in) { return out >= 1 && in >= 32 && in % 32 == 0; }

int alloc_matrix(int out, int in, int device, idol_q8_matrix** result) {
    auto* h = new idol_q8_matrix();
    h->m.device = device;
    h->m.n = out;
    h->m.k = in;
    const cudaError_t e = cudaMalloc(&h->m.tiles, idol::tiled_bytes(out, in));
    if (e != cudaSuccess) {
        delete h;
        return idol::cuda_fail(e, "cudaMalloc (Q8_0 matrix)");
    }
    *result = h;
    return IDOL_OK;
}

}  // namespace

extern "C" {

const char* idol_b200_last_error(void) { return idol::g_last_error.c_str(); }

int idol_b200_version(void) { return 100; }

int idol_b200_device_status(int device, unsigned int* flags) {
    if (!flags) return fail(IDOL_ERR_INVALID, "device_status: flags is NULL");
    IDOL_CUDA(cudaSetDevice(device));
    unsigned int v = 0, all = 0;
    IDOL_CUDA(idol::take_device_error_gemm(&v));
    all |= v;
    IDOL_CUDA(idol::take_device_error_attention(&v));
    all |= v;
    *flags = all;
    return IDOL_OK;
}

int64_t idol_b200_q8_bytes(int out, int in) { return shape_ok(out, in) ? (int64_t)out * (in / 32) * 34 : -1; }
int64_t idol_b200_q8_tiled_bytes(int out, int in) { return shape_ok(out, in) ? idol::tiled_bytes(out, in) : -1; }

int idol_b200_q8_quantize(const float* w, int64_t rows, int64_t cols, void* q8, void* stream) {
    if (rows < 0 || cols < 0 || cols % 32) return fail(IDOL_ERR_INVALID, "q8_quantize: cols must be a multiple of 32");
    if (rows * cols == 0) return IDOL_OK;
    if (!w || !q8) return fail(IDOL_ERR_INVALID, "q8_quantize: NULL pointer");
    IDOL_CUDA(idol::launch_q8_quantize(w, rows, cols, static_cast<uint8_t*>(q8), static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

int idol_b200_q8_repack(const void* q8, int out, int in, void* tiles, void* stream) {
    if (!shape_ok(out, in)) return fail(IDOL_ERR_INVALID, "q8_repack: out >= 1 and in a positive multiple of 32");
    if (!q8 || !tiles) return fail(IDOL_ERR_INVALID, "q8_repack: NULL pointer");
    if (reinterpret_cast<uintptr_t>(q8) % 2 || reinterpret_cast<uintptr_t>(tiles) % 16)
        return fail(IDOL_ERR_INVALID, "q8_repack: q8 must be 2-byte, tiles 16-byte aligned");
    IDOL_CUDA(idol::launch_q8_repack(static_cast<const uint8_t*>(q8), out, in, static_cast<uint8_t*>(tiles),
                                     static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

int64_t idol_b200_q4_0_bytes(int out, int in) { return shape_ok(out, in) ? (int64_t)out * (in / 32) * 18 : -1; }

int idol_b200_q4_0_repack(const void* q4_0, int out, int in, void* tiles, void* stream) {
    if (!shape_ok(out, in)) return fail(IDOL_ERR_INVALID, "q4_0_repack: out >= 1 and in a positive multiple of 32");
    if (!q4_0 || !tiles) return fail(IDOL_ERR_INVALID, "q4_0_repack: NULL pointer");
    if (reinterpret_cast<uintptr_t>(q4_0) % 2 || reinterpret_cast<uintptr_t>(tiles) % 16)
        return fail(IDOL_ERR_INVALID, "q4_0_repack: q4_0 must be 2-byte, tiles 16-byte aligned");
    IDOL_CUDA(idol::launch_q4_0_repack(static_cast<const uint8_t*>(q4_0), out, in, static_cast<uint8_t*>(tiles),
                                       static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

int64_t idol_b200_q4_k_bytes(int out, int in) {
    return (out >= 1 && in >= 256 && in % 256 == 0) ? (int64_t)out * (in / 256) * 144 : -1;
}

int64_t idol_b200_q4_k_tiled_bytes(int out, int in) {
    return (out >= 1 && in >= 256 && in % 256 == 0) ? idol::q4k_tiled_bytes(out, in) : -1;
}

int idol_b200_q4_k_repack(const void* q4_k, int out, int in, void* tiles, void* stream) {
    if (out < 1 || in < 256 || in % 256)
        return fail(IDOL_ERR_INVALID, "q4_k_repack: out >= 1 and in a positive multiple of 256");
    if (!q4_k || !tiles) return fail(IDOL_ERR_INVALID, "q4_k_repack: NULL pointer");
    if (reinterpret_cast<uintptr_t>(q4_k) % 16 || reinterpret_cast<uintptr_t>(tiles) % 16)
        return fail(IDOL_ERR_INVALID, "q4_k_repack: q4_k and tiles must be 16-byte aligned");
    IDOL_CUDA(idol::launch_q4_k_repack(static_cast<const uint8_t*>(q4_k), out, in, static_cast<uint8_t*>(tiles),
                                       static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

int idol_b200_q4_k_dequantize(const void* tiles, int out, int in, void* w, int w_dtype, void* stream) {
    if (out < 1 || in < 256 || in % 256)
        return fail(IDOL_ERR_INVALID, "q4_k_dequantize: out >= 1 and in a positive multiple of 256");
    if (!tiles || !w) return fail(IDOL_ERR_INVALID, "q4_k_dequantize: NULL pointer");
    if (reinterpret_cast<uintptr_t>(tiles) % 16)
        return fail(IDOL_ERR_INVALID, "q4_k_dequantize: tiles not 16-byte aligned");
    if (w_dtype != IDOL_F32 && w_dtype != IDOL_BF16 && w_dtype != IDOL_F16)
        return fail(IDOL_ERR_UNSUPPORTED, "q4_k_dequantize: output must be f32, bf16 or f16");
    IDOL_CUDA(idol::launch_q4_k_dequant(static_cast<const uint8_t*>(tiles), out, in, w, w_dtype,
                                        static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

int idol_b200_q4_k_view(const void* tiles, const float* bias_dev, int out, int in, int device,
                        idol_q8_matrix** matrix) {
    if (!matrix) return fail(IDOL_ERR_INVALID, "q4_k_view: matrix is NULL");
    *matrix = nullptr;
    if (out < 1 || in < 256 || in % 256)
        return fail(IDOL_ERR_INVALID, "q4_k_view: out >= 1 and in a positive multiple of 256");
    if (!tiles || reinterpret_cast<uintptr_t>(tiles) % 16)
        return fail(IDOL_ERR_INVALID, "q4_k_view: tiles must be a 16-byte aligned device pointer");
    auto* h = new idol_q8_matrix();
    h->m.device = device;
    h->m.n = out;
    h->m.k = in;
    h->m.tiles = static_cast<uint8_t*>(const_cast<void*>(tiles));
    h->m.bias = const_cast<float*>(bias_dev);
    h->m.owns = false;
    h->m.format = idol::kFmtQ4K;
    *matrix = h;
    return IDOL_OK;
}

int idol_b200_q8_unpack(const void* tiles, int out, int in, void* q8, void* stream) {
    if (!shape_ok(out, in)) return fail(IDOL_ERR_INVALID, "q8_unpack: out >= 1 and in a positive multiple of 32");
    if (!q8 || !tiles) return fail(IDOL_ERR_INVALID, "q8_unpack: NULL pointer");
    if (reinterpret_cast<uintptr_t>(q8) % 2 || reinterpret_cast<uintptr_t>(tiles) % 16)
        return fail(IDOL_ERR_INVALID, "q8_unpack: q8 must be 2-byte, tiles 16-byte aligned");
    IDOL_CUDA(idol::launch_q8_unpack(static_cast<const uint8_t*>(tiles), out, in, static_cast<uint8_t*>(q8),
                                     static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

int idol_b200_q8_dequantize(const void* tiles, int out, int in, void* w, int w_dtype, void* stream) {
    if (!shape_ok(out, in)) return fail(IDOL_ERR_INVALID, "q8_dequantize: out >= 1 and in a positive multiple of 32");
    if (!tiles || !w) return fail(IDOL_ERR_INVALID, "q8_dequantize: NULL pointer");
    if (reinterpret_cast<uintptr_t>(tiles) % 16) return fail(IDOL_ERR_INVALID, "q8_dequantize: tiles not 16-byte aligned");
    if (w_dtype != IDOL_F32 && w_dtype != IDOL_BF16 && w_dtype != IDOL_F16)
        return fail(IDOL_ERR_UNSUPPORTED, "q8_dequantize: output must be f32, bf16 or f16");
    IDOL_CUDA(idol::launch_q8_dequant(static_cast<const uint8_t*>(tiles), out, in, w, w_dtype,
                                      static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

int idol_b200_q8_upload(const void* q8_host, int64_t nbytes, int out, int in, const float* bias_host, int device,
                        idol_q8_matrix** matrix) {
    if (!matrix) return fail(IDOL_ERR_INVALID, "q8_upload: matrix is NULL");
    *matrix = nullptr;
    if (!shape_ok(out, in)) return fail(IDOL_ERR_INVALID, "q8_upload: out >= 1 and in a positive multiple of 32");
    if (!q8_host || nbytes != (int64_t)out * (in / 32) * 34)
        return fail(IDOL_ERR_INVALID, "q8_upload: Q8_0 byte count does not match the shape");
    IDOL_CUDA(cudaSetDevice(device));
    idol_q8_matrix* h = nullptr;
    int rc = alloc_matrix(out, in, device, &h);
    if (rc != IDOL_OK) return rc;
    void* staging = nullptr;
    cudaError_t e = cudaMalloc(&staging, (size_t)nbytes);
    if (e == cudaSuccess) e = cudaMemcpy(staging, q8_host, (size_t)nbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && bias_host) {
        e = cudaMalloc(&h->m.bias, sizeof(float) * out);
        if (e == cudaSuccess) e = cudaMemcpy(h->m.bias, bias_host, sizeof(float) * out, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess)
        e = idol::launch_q8_repack(static_cast<const uint8_t*>(staging), out, in, h->m.tiles, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(staging);
    if (e != cudaSuccess) {
        idol_b200_q8_free(h);
        return idol::cuda_fail(e, "q8_upload");
    }
    *matrix = h;
    return IDOL_OK;
}

int idol_b200_q8_import(const void* q8_dev, int64_t nbytes, int out, int in, const float* bias_dev, int device,
                        void* stream, idol_q8_matrix** matrix) {
    if (!matrix) return fail(IDOL_ERR_INVALID, "q8_import: matrix is NULL");
    *matrix = nullptr;
    if (!shape_ok(out, in)) return fail(IDOL_ERR_INVALID, "q8_import: out >= 1 and in a positive multiple of 32");
    if (!q8_dev || nbytes != (int64_t)out * (in / 32) * 34)
        return fail(IDOL_ERR_INVALID, "q8_import: Q8_0 byte count does not match the shape");
    if (reinterpret_cast<uintptr_t>(q8_dev) % 2) return fail(IDOL_ERR_INVALID, "q8_import: q8 must be 2-byte aligned");
    IDOL_CUDA(cudaSetDevice(device));
    idol_q8_matrix* h = nullptr;
    int rc = alloc_matrix(out, in, device, &h);
    if (rc != IDOL_OK) return rc;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (bias_dev) {
        e = cudaMalloc(&h->m.bias, sizeof(float) * out);
        if (e == cudaSuccess) e = cudaMemcpyAsync(h->m.bias, bias_dev, sizeof(float) * out, cudaMemcpyDeviceToDevice, s);
    }
    if (e == cudaSuccess)
        e = idol::launch_q8_repack(static_cast<const uint8_t*>(q8_dev), out, in, h->m.tiles, s);
    if (e != cudaSuccess) {
        idol_b200_q8_free(h);
        return idol::cuda_fail(e, "q8_import");
    }
    *matrix = h;
    return IDOL_OK;
}

int idol_b200_q8_view(const void* tiles, const float* bias_dev, int out, int in, int device, idol_q8_matrix** matrix) {
    if (!matrix) return fail(IDOL_ERR_INVALID, "q8_view: matrix is NULL");
    *matrix = nullptr;
    if (!shape_ok(out, in)) return fail(IDOL_ERR_INVALID, "q8_view: out >= 1 and in a positive multiple of 32");
    if (!tiles || reinterpret_cast<uintptr_t>(tiles) % 16)
        return fail(IDOL_ERR_INVALID, "q8_view: tiles must be a 16-byte aligned device pointer");
    auto* h = new idol_q8_matrix();
    h->m.device = device;
    h->m.n = out;
    h->m.k = in;
    h->m.tiles = static_cast<uint8_t*>(const_cast<void*>(tiles));
    h->m.bias = const_cast<float*>(bias_dev);
    h->m.owns = false;
    *matrix = h;
    return IDOL_OK;
}

int idol_b200_q8_free(idol_q8_matrix* matrix) {
    if (!matrix) return IDOL_OK;
    if (matrix->m.owns) {
        cudaSetDevice(matrix->m.device);
        cudaFree(matrix->m.tiles);
        cudaFree(matrix->m.bias);
    }
    delete matrix;
    return IDOL_OK;
}

int idol_b200_q8_info(const idol_q8_matrix* matrix, int* out, int* in, int* device, int64_t* device_bytes) {
    if (!matrix) return fail(IDOL_ERR_INVALID, "q8_info: matrix is NULL");
    if (out) *out = matrix->m.n;
    if (in) *in = matrix->m.k;
    if (device) *device = matrix->m.device;
    if (device_bytes)
        *device_bytes = (matrix->m.format == idol::kFmtQ4K ? idol::q4k_tiled_bytes(matrix->m.n, matrix->m.k)
                                                            : idol::tiled_bytes(matrix->m.n, matrix->m.k)) +
                        (matrix->m.bias ? 4 * (int64_t)matrix->m.n : 0);
    return IDOL_OK;
}

int idol_b200_q8_export(const idol_q8_matrix* matrix, void* q8_dev, int64_t nbytes, void* stream) {
    if (!matrix || !q8_dev) return fail(IDOL_ERR_INVALID, "q8_export: NULL pointer");
    if (matrix->m.format != idol::kFmtQ8) return fail(IDOL_ERR_UNSUPPORTED, "q8_export: the matrix holds Q4_K tiles");
    if (nbytes != (int64_t)matrix->m.n * (matrix->m.k / 32) * 34)
        return fail(IDOL_ERR_INVALID, "q8_export: byte count does not match the shape");
    IDOL_CUDA(cudaSetDevice(matrix->m.device));
    IDOL_CUDA(idol::launch_q8_unpack(matrix->m.tiles, matrix->m.n, matrix->m.k,
                                     static_cast<uint8_t*>(q8_dev), static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

int idol_b200_q8_gemm(const idol_q8_matrix* matrix, const void* x, int x_dtype, int64_t m, int64_t ldx, int n_offset,
                      int n, const void* residual, int64_t ldr, int act, int flags, void* y, int y_dtype, int64_t ldy,
                      void* stream) {
    if (!matrix) return fail(IDOL_ERR_INVALID, "q8_gemm: matrix is NULL");
    if (m > 0 && n > 0 && (!x || !y)) return fail(IDOL_ERR_INVALID, "q8_gemm: NULL pointer");
    IDOL_CUDA(cudaSetDevice(matrix->m.device));
    idol::GemmCall c = {&matrix->m, x, x_dtype, m, ldx, n_offset, n, residual, ldr, act, flags, y, y_dtype, ldy,
                        static_cast<cudaStream_t>(stream)};
    return idol::q8_gemm(c);
}

int idol_b200_q8_gemm_heads(const idol_q8_matrix* matrix, const void* x, int64_t m, int64_t ldx, void* y, int64_t ldy,
                            int head_cols, int head_split, const float* gamma_a, const float* gamma_b, void* stream) {
    if (!matrix) return fail(IDOL_ERR_INVALID, "q8_gemm_heads: matrix is NULL");
    if (m > 0 && (!x || !y)) return fail(IDOL_ERR_INVALID, "q8_gemm_heads: NULL pointer");
    if (head_cols < 1) return fail(IDOL_ERR_INVALID, "q8_gemm_heads: head_cols must be >= 64");
    IDOL_CUDA(cudaSetDevice(matrix->m.device));
    idol::GemmCall c = {&matrix->m, x, IDOL_BF16, m, ldx, 0, matrix->m.n, nullptr, 0, IDOL_ACT_NONE, 0, y, IDOL_BF16,
                        ldy, static_cast<cudaStream_t>(stream)};
    c.head_gamma_a = gamma_a;
    c.head_gamma_b = gamma_b;
    c.head_cols = head_cols;
    c.head_split = head_split;
    return idol::q8_gemm(c);
}

int64_t idol_b200_q8_gemm_int8act_workspace_bytes(int64_t m, int in) { return idol::int8act_workspace_bytes(m, in); }

int idol_b200_q8_gemm_int8act(const idol_q8_matrix* matrix, const void* x, int x_dtype, int64_t m, int64_t ldx,
                              int n_offset, int n, const void* residual, int64_t ldr, int act, void* y, int y_dtype,
                              int64_t ldy, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!matrix) return fail(IDOL_ERR_INVALID, "q8_gemm_int8act: matrix is NULL");
    if (m < 0 || n < 0) return fail(IDOL_ERR_INVALID, "q8_gemm_int8act: sizes");
    idol::GemmCall c = {&matrix->m, x, x_dtype, m, ldx, n_offset, n, residual, ldr, act, 0, y, y_dtype, ldy,
                        static_cast<cudaStream_t>(stream)};
    const int rc = idol::q8_gemm_int8act_check(c, workspace, workspace_bytes);  // refused before any device call
    if (rc != IDOL_OK || m == 0 || n == 0) return rc;
    IDOL_CUDA(cudaSetDevice(matrix->m.device));
    return idol::q8_gemm_int8act(c, workspace, workspace_bytes);
}

int idol_b200_norm_rows(const void* x, int x_dtype, int64_t rows, int dim, int64_t ldx, float eps, const float* gamma,
                        const float* beta, const float* shift, const float* scale, void* y, int y_dtype, int64_t ldy,
                        void* stream) {
    if (rows < 0) return fail(IDOL_ERR_INVALID, "norm_rows: rows < 0");
    if (!idol::norm_dim_ok(dim)) return fail(IDOL_ERR_UNSUPPORTED, "norm_rows: dim must be 256, 512, 768, 1024, 1536 or 2048");
    if (rows == 0) return IDOL_OK;
    if (!x || !y || (gamma && !beta) || (!gamma && beta) || (shift && !scale) || (!shift && scale))
        return fail(IDOL_ERR_INVALID, "norm_rows: NULL pointer (gamma/beta and shift/scale come in pairs)");
    const int xs = x_dtype == IDOL_F32 ? 4 : 2, ys = y_dtype == IDOL_F32 ? 4 : 2;
    if (ldx < dim || ldy < dim || (ldx * xs) % 16 || (ldy * ys) % 16 || reinterpret_cast<uintptr_t>(x) % 16 ||
        reinterpret_cast<uintptr_t>(y) % 16)
        return fail(IDOL_ERR_INVALID, "norm_rows: rows must be 16-byte aligned");
    const cudaError_t e = idol::launch_norm_rows(x, x_dtype, ldx, y, y_dtype, ldy, rows, dim, eps, gamma, beta, shift,
                                                 scale, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue) return fail(IDOL_ERR_UNSUPPORTED, "norm_rows: dtype pair not implemented");
    IDOL_CUDA(e);
    return IDOL_OK;
}

int idol_b200_rms_heads(void* x, int dtype, int64_t rows, int64_t ld, int heads, int head_dim, const float* gamma,
                        void* stream) {
    if (head_dim != 64) return fail(IDOL_ERR_UNSUPPORTED, "rms_heads: only head_dim 64 is implemented");
    if (rows < 0 || heads < 1 || ld < (int64_t)heads * head_dim) return fail(IDOL_ERR_INVALID, "rms_heads: sizes");
    if (rows == 0) return IDOL_OK;
    if (!x || !gamma) return fail(IDOL_ERR_INVALID, "rms_heads: NULL pointer");
    const cudaError_t e = idol::launch_rms_heads(x, dtype, ld, rows, heads, gamma, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue) return fail(IDOL_ERR_UNSUPPORTED, "rms_heads: dtype not implemented");
    IDOL_CUDA(e);
    return IDOL_OK;
}

int idol_b200_attention(const void* q, int64_t lq, int64_t ldq, const void* k, const void* v, int64_t lk, int64_t ldkv,
                        int heads, int head_dim, void* out, int out_dtype, int64_t ldo, int batch, void* stream) {
    if (out_dtype != IDOL_BF16 && out_dtype != IDOL_F32)
        return fail(IDOL_ERR_UNSUPPORTED, "attention: the output dtype must be IDOL_BF16 or IDOL_F32");
    idol::AttentionCall c = {q, k, v, out, lq, lk, ldq, ldkv, ldo, heads, head_dim, batch,
                             static_cast<cudaStream_t>(stream), out_dtype == IDOL_F32};
    return idol::attention(c);
}

}  // extern "C"
