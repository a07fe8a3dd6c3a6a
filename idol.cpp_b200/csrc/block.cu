// block.cu - compositions of the hot-path kernels, for callers that hand over a whole layer stack.
//
//   denoiser block (scope row A14; src/decoders.cpp:296-313 without the cross-attention, which the synthetic
//   config-3 block leaves out):
//       h = LN(x, eps)                                   norm_rows
//       qkv = h W_qkv^T + b                              q8 GEMM          (rows x 3D, bf16)
//       q, k <- rms_heads(q, gamma_q), rms_heads(k, gamma_k)
//       a = attention(q, k, v) per image                 tcgen05 flash attention
//       x = a W_out^T + b + x                            q8 GEMM, residual in place
//       h = LN(x, eps)
//       f = gelu_tanh(h W_ff1^T + b)                     q8 GEMM, activation in the epilogue
//       x = f W_ff2^T + b + x                            q8 GEMM, residual in place
//   The residual stream x is fp32 (as the reference's X) or bf16; everything a GEMM reads is bf16.
//
//   Gaussian decoder block (src/decoders.cpp:296-313, with the cross-attention): the block above with, between the
//   self-attention and the MLP, h = LN(x) * gamma2 + beta2; q = rms(h W_q^T); kv = cond W_kv^T + b (dense fp32,
//   the 16-wide condition), rms on k; a = attention of each image's rows over its cond rows; x = a W_o^T + b + x.
//
//   Gaussian MLP (scope row A15, config 4): 128 -> 512 (SiLU) -> 512 (SiLU) -> 14, then the output heads
//   (pos identity, scale exp, rotation f * 0.1 + (1, 0, 0, 0) normalised as src/decoders.cpp:422-428, colour and
//   opacity sigmoid as :429).
//
// Both take a caller-provided device workspace (idol_b200_*_workspace_bytes) and allocate nothing themselves.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <mutex>
#include <string>

#include "internal.h"

namespace idol {

namespace {

__device__ __forceinline__ float load_f(const void* p, int dtype, long long i) {
    if (dtype == IDOL_F32) return static_cast<const float*>(p)[i];
    if (dtype == IDOL_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(static_cast<const __half*>(p)[i]);
}

// One thread per point: 14 raw values -> 14 activated values (fp32).
__global__ void gaussian_heads_kernel(const void* __restrict__ raw, int dtype, long long points, long long ld,
                                      float* __restrict__ out) {
    const long long pt = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (pt >= points) return;
    float f[14];
#pragma unroll
    for (int c = 0; c < 14; ++c) f[c] = load_f(raw, dtype, pt * ld + c);
    float* o = out + pt * 14;
#pragma unroll
    for (int c = 0; c < 3; ++c) o[c] = f[c];
#pragma unroll
    for (int c = 3; c < 6; ++c) o[c] = expf(f[c]);
    // Rotation as src/decoders.cpp:422-428: r = f * lr_rotation + (1, 0, 0, 0), lr_rotation = 0.1 (the
    // Representation default, src/weights.hpp:27), then divided by max(|r|, 1e-12).
    float r[4], nrm = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        r[c] = f[6 + c] * 0.1f + (c == 0 ? 1.0f : 0.0f);
        nrm += r[c] * r[c];
    }
    nrm = fmaxf(sqrtf(nrm), 1e-12f);
#pragma unroll
    for (int c = 0; c < 4; ++c) o[6 + c] = r[c] / nrm;
#pragma unroll
    for (int c = 10; c < 14; ++c) o[c] = 1.0f / (1.0f + expf(-f[c]));
}

// The cross-attention's key/value projection of the latent tokens (src/decoders.cpp:237, `to_kv`, which the
// reference keeps as a dense fp32 matrix since its depth is the 16-wide condition): kv[r, j] = sum_c cond[r, c]
// w[j, c] (fp32 FMA chain in c order) + b[j], stored as bf16 [rows, 2D]. A block takes 256 output columns and 16 rows:
// each thread keeps its column's weights in registers, the rows' conditions are staged in shared memory.
constexpr int kKvMaxCond = 64;
__global__ void kv_project_kernel(const float* __restrict__ cond, long long rows, int cdim,
                                  const float* __restrict__ w, const float* __restrict__ b, int cols,
                                  __nv_bfloat16* __restrict__ kv) {
    __shared__ float cs[16][kKvMaxCond];
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const long long r0 = (long long)blockIdx.y * 16;
    for (int i = threadIdx.x; i < 16 * cdim; i += blockDim.x) {
        const long long r = r0 + i / cdim;
        cs[i / cdim][i % cdim] = r < rows ? cond[r * cdim + i % cdim] : 0.0f;
    }
    __syncthreads();
    if (j >= cols) return;
    float wr[kKvMaxCond];
#pragma unroll
    for (int c = 0; c < kKvMaxCond; ++c) wr[c] = c < cdim ? w[(long long)j * cdim + c] : 0.0f;
    const float bj = b ? b[j] : 0.0f;
    for (int i = 0; i < 16; ++i) {
        const long long r = r0 + i;
        if (r >= rows) break;
        float acc = 0.0f;
#pragma unroll
        for (int c = 0; c < kKvMaxCond; ++c)
            if (c < cdim) acc = fmaf(cs[i][c], wr[c], acc);
        kv[r * cols + j] = __float2bfloat16_rn(acc + bj);
    }
}

}  // namespace

cudaError_t launch_gaussian_heads(const void* raw, int raw_dtype, long long points, long long ld, float* out,
                                  cudaStream_t s) {
    if (points == 0) return cudaSuccess;
    gaussian_heads_kernel<<<(unsigned)((points + 255) / 256), 256, 0, s>>>(raw, raw_dtype, points, ld, out);
    return cudaGetLastError();
}

}  // namespace idol

using idol::fail;

struct idol_block {
    const idol_q8_matrix* qkv;
    const idol_q8_matrix* out;
    const idol_q8_matrix* ff1;
    const idol_q8_matrix* ff2;
    const float* q_gamma;
    const float* k_gamma;
    int heads, dim, hidden, device;
    float eps;
};

struct idol_gs_block {
    idol_block self;                     // LN -> QKV -> rms -> self-attention -> out, and the MLP
    const idol_q8_matrix* cross_q;
    const idol_q8_matrix* cross_out;
    const float* cq_gamma;
    const float* ck_gamma;
    const float* norm2_gamma;
    const float* norm2_beta;
    const float* kv_w;                   // fp32 [2D, cond_dim]
    const float* kv_b;                   // fp32 [2D] or NULL
    int cond_dim;
};

struct idol_gaussian_mlp {
    const idol_q8_matrix* l0;
    const idol_q8_matrix* l1;
    const idol_q8_matrix* l2;
    int device;
};

namespace {

inline int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

int gemm(const idol_q8_matrix* w, const void* x, int64_t m, int64_t ldx, const void* residual, int64_t ldr, int act,
         void* y, int y_dtype, int64_t ldy, cudaStream_t s, int x_dtype = IDOL_BF16) {
    idol::GemmCall c = {&w->m, x, x_dtype, m, ldx, 0, w->m.n, residual, ldr, act, 0, y, y_dtype, ldy, s};
    return idol::q8_gemm(c);
}

}  // namespace

extern "C" {

int idol_b200_block_create(const idol_q8_matrix* qkv, const idol_q8_matrix* out, const idol_q8_matrix* ff1,
                           const idol_q8_matrix* ff2, const float* q_gamma, const float* k_gamma, int heads,
                           float eps, idol_block** block) {
    if (!block) return fail(IDOL_ERR_INVALID, "block_create: block is NULL");
    *block = nullptr;
    if (!qkv || !out || !ff1 || !ff2 || !q_gamma || !k_gamma) return fail(IDOL_ERR_INVALID, "block_create: NULL");
    const int D = out->m.n;
    if (heads < 1 || D != heads * 64) return fail(IDOL_ERR_UNSUPPORTED, "block_create: head_dim must be 64");
    if (qkv->m.n != 3 * D || qkv->m.k != D || out->m.k != D || ff1->m.k != D || ff2->m.n != D ||
        ff2->m.k != ff1->m.n)
        return fail(IDOL_ERR_INVALID, "block_create: qkv (3D x D), out (D x D), ff1 (H x D), ff2 (D x H) expected");
    if (!idol::norm_dim_ok(D)) return fail(IDOL_ERR_UNSUPPORTED, "block_create: model width not supported by norm_rows");
    const int dev = qkv->m.device;
    if (out->m.device != dev || ff1->m.device != dev || ff2->m.device != dev)
        return fail(IDOL_ERR_INVALID, "block_create: matrices on different devices");
    *block = new idol_block{qkv, out, ff1, ff2, q_gamma, k_gamma, heads, D, ff1->m.n, dev, eps};
    return IDOL_OK;
}

int idol_b200_block_free(idol_block* block) {
    delete block;
    return IDOL_OK;
}

int64_t idol_b200_block_workspace_bytes(const idol_block* b, int64_t rows) {
    if (!b || rows < 0) return -1;
    const int64_t big = b->hidden > 3 * b->dim ? b->hidden : 3 * b->dim;
    return align256(rows * b->dim * 2) + align256(rows * big * 2);
}

int idol_b200_block_forward(const idol_block* b, void* x, int x_dtype, int64_t tokens, int images, void* workspace,
                            int64_t workspace_bytes, void* stream) {
    if (!b || !x) return fail(IDOL_ERR_INVALID, "block_forward: NULL");
    if (x_dtype != IDOL_F32 && x_dtype != IDOL_BF16) return fail(IDOL_ERR_UNSUPPORTED, "block_forward: x is f32 or bf16");
    if (tokens < 1 || images < 1) return fail(IDOL_ERR_INVALID, "block_forward: tokens and images must be >= 1");
    const int64_t rows = tokens * images;
    if (!workspace || workspace_bytes < idol_b200_block_workspace_bytes(b, rows) ||
        reinterpret_cast<uintptr_t>(workspace) % 256)
        return fail(IDOL_ERR_INVALID, "block_forward: workspace smaller than idol_b200_block_workspace_bytes or not "
                                      "256-byte aligned");
    IDOL_CUDA(cudaSetDevice(b->device));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int D = b->dim;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(ws);                       // rows x D
    __nv_bfloat16* big = reinterpret_cast<__nv_bfloat16*>(ws + align256(rows * D * 2));  // rows x max(3D, H)

    IDOL_CUDA(idol::launch_norm_rows(x, x_dtype, D, h, IDOL_BF16, D, rows, D, b->eps, nullptr, nullptr, nullptr,
                                     nullptr, s));
    int rc = gemm(b->qkv, h, rows, D, nullptr, 0, IDOL_ACT_NONE, big, IDOL_BF16, 3 * D, s);
    if (rc != IDOL_OK) return rc;
    IDOL_CUDA(idol::launch_rms_heads(big, IDOL_BF16, 3 * D, rows, b->heads, b->q_gamma, s));
    IDOL_CUDA(idol::launch_rms_heads(big + D, IDOL_BF16, 3 * D, rows, b->heads, b->k_gamma, s));
    idol::AttentionCall ac = {big, big + D, big + 2 * D, h, tokens, tokens, 3 * D, 3 * D, D, b->heads, 64, images, s};
    rc = idol::attention(ac);
    if (rc != IDOL_OK) return rc;
    rc = gemm(b->out, h, rows, D, x, D, IDOL_ACT_NONE, x, x_dtype, D, s);
    if (rc != IDOL_OK) return rc;
    IDOL_CUDA(idol::launch_norm_rows(x, x_dtype, D, h, IDOL_BF16, D, rows, D, b->eps, nullptr, nullptr, nullptr,
                                     nullptr, s));
    rc = gemm(b->ff1, h, rows, D, nullptr, 0, IDOL_ACT_GELU_TANH, big, IDOL_BF16, b->hidden, s);
    if (rc != IDOL_OK) return rc;
    return gemm(b->ff2, big, rows, b->hidden, x, D, IDOL_ACT_NONE, x, x_dtype, D, s);
}

int idol_b200_gs_block_create(const idol_q8_matrix* qkv, const idol_q8_matrix* out, const idol_q8_matrix* cross_q,
                              const idol_q8_matrix* cross_out, const idol_q8_matrix* ff1, const idol_q8_matrix* ff2,
                              const float* q_gamma, const float* k_gamma, const float* cross_q_gamma,
                              const float* cross_k_gamma, const float* norm2_gamma, const float* norm2_beta,
                              const float* kv_weight, const float* kv_bias, int cond_dim, int heads, float eps,
                              idol_gs_block** block) {
    if (!block) return fail(IDOL_ERR_INVALID, "gs_block_create: block is NULL");
    *block = nullptr;
    idol_block* self = nullptr;
    int rc = idol_b200_block_create(qkv, out, ff1, ff2, q_gamma, k_gamma, heads, eps, &self);
    if (rc != IDOL_OK) return rc;
    const int D = self->dim;
    if (!cross_q || !cross_out || !cross_q_gamma || !cross_k_gamma || !norm2_gamma || !norm2_beta || !kv_weight) {
        delete self;
        return fail(IDOL_ERR_INVALID, "gs_block_create: NULL");
    }
    if (cross_q->m.n != D || cross_q->m.k != D || cross_out->m.n != D || cross_out->m.k != D ||
        cross_q->m.device != self->device || cross_out->m.device != self->device) {
        delete self;
        return fail(IDOL_ERR_INVALID, "gs_block_create: cross q and out must be D x D on the block's device");
    }
    if (cond_dim < 1 || cond_dim > idol::kKvMaxCond) {
        delete self;
        return fail(IDOL_ERR_UNSUPPORTED, "gs_block_create: cond_dim must be 1..64");
    }
    *block = new idol_gs_block{*self, cross_q, cross_out, cross_q_gamma, cross_k_gamma, norm2_gamma, norm2_beta,
                               kv_weight, kv_bias, cond_dim};
    delete self;
    return IDOL_OK;
}

int idol_b200_gs_block_free(idol_gs_block* block) {
    delete block;
    return IDOL_OK;
}

int64_t idol_b200_gs_block_workspace_bytes(const idol_gs_block* b, int64_t rows, int64_t cond_rows_total) {
    if (!b || rows < 0 || cond_rows_total < 0) return -1;
    return idol_b200_block_workspace_bytes(&b->self, rows) + align256(cond_rows_total * 2 * b->self.dim * 2);
}

int idol_b200_gs_block_forward(const idol_gs_block* g, void* x, int x_dtype, int64_t tokens, int images,
                               const float* cond, int64_t cond_rows, void* workspace, int64_t workspace_bytes,
                               void* stream) {
    if (!g || !x || !cond) return fail(IDOL_ERR_INVALID, "gs_block_forward: NULL");
    if (x_dtype != IDOL_F32 && x_dtype != IDOL_BF16)
        return fail(IDOL_ERR_UNSUPPORTED, "gs_block_forward: x is f32 or bf16");
    if (tokens < 1 || images < 1 || cond_rows < 1)
        return fail(IDOL_ERR_INVALID, "gs_block_forward: tokens, images and cond_rows must be >= 1");
    if (cond_rows * images > 65535LL * 16)
        return fail(IDOL_ERR_INVALID, "gs_block_forward: more than 1,048,560 condition rows in one call");
    const idol_block* b = &g->self;
    const int64_t rows = tokens * images, crows = cond_rows * images;
    if (!workspace || workspace_bytes < idol_b200_gs_block_workspace_bytes(g, rows, crows) ||
        reinterpret_cast<uintptr_t>(workspace) % 256)
        return fail(IDOL_ERR_INVALID, "gs_block_forward: workspace smaller than idol_b200_gs_block_workspace_bytes "
                                      "or not 256-byte aligned");
    IDOL_CUDA(cudaSetDevice(b->device));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int D = b->dim;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int64_t self_bytes = idol_b200_block_workspace_bytes(b, rows);
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(ws);                            // rows x D
    __nv_bfloat16* big = reinterpret_cast<__nv_bfloat16*>(ws + align256(rows * D * 2));  // rows x max(3D, H)
    __nv_bfloat16* kv = reinterpret_cast<__nv_bfloat16*>(ws + self_bytes);              // crows x 2D

    // Self-attention sublayer.
    IDOL_CUDA(idol::launch_norm_rows(x, x_dtype, D, h, IDOL_BF16, D, rows, D, b->eps, nullptr, nullptr, nullptr,
                                     nullptr, s));
    int rc = gemm(b->qkv, h, rows, D, nullptr, 0, IDOL_ACT_NONE, big, IDOL_BF16, 3 * D, s);
    if (rc != IDOL_OK) return rc;
    IDOL_CUDA(idol::launch_rms_heads(big, IDOL_BF16, 3 * D, rows, b->heads, b->q_gamma, s));
    IDOL_CUDA(idol::launch_rms_heads(big + D, IDOL_BF16, 3 * D, rows, b->heads, b->k_gamma, s));
    idol::AttentionCall sa = {big, big + D, big + 2 * D, h, tokens, tokens, 3 * D, 3 * D, D, b->heads, 64, images, s};
    rc = idol::attention(sa);
    if (rc != IDOL_OK) return rc;
    rc = gemm(b->out, h, rows, D, x, D, IDOL_ACT_NONE, x, x_dtype, D, s);
    if (rc != IDOL_OK) return rc;

    // Cross-attention sublayer (src/decoders.cpp:304-306, 232-240).
    IDOL_CUDA(idol::launch_norm_rows(x, x_dtype, D, h, IDOL_BF16, D, rows, D, b->eps, g->norm2_gamma, g->norm2_beta,
                                     nullptr, nullptr, s));
    rc = gemm(g->cross_q, h, rows, D, nullptr, 0, IDOL_ACT_NONE, big, IDOL_BF16, D, s);
    if (rc != IDOL_OK) return rc;
    IDOL_CUDA(idol::launch_rms_heads(big, IDOL_BF16, D, rows, b->heads, g->cq_gamma, s));
    {
        const dim3 grid((unsigned)((2 * D + 255) / 256), (unsigned)((crows + 15) / 16));
        idol::kv_project_kernel<<<grid, 256, 0, s>>>(cond, crows, g->cond_dim, g->kv_w, g->kv_b, 2 * D, kv);
        IDOL_CUDA(cudaGetLastError());
    }
    IDOL_CUDA(idol::launch_rms_heads(kv, IDOL_BF16, 2 * D, crows, b->heads, g->ck_gamma, s));
    idol::AttentionCall ca = {big, kv, kv + D, h, tokens, cond_rows, D, 2 * D, D, b->heads, 64, images, s};
    rc = idol::attention(ca);
    if (rc != IDOL_OK) return rc;
    rc = gemm(g->cross_out, h, rows, D, x, D, IDOL_ACT_NONE, x, x_dtype, D, s);
    if (rc != IDOL_OK) return rc;

    // MLP sublayer.
    IDOL_CUDA(idol::launch_norm_rows(x, x_dtype, D, h, IDOL_BF16, D, rows, D, b->eps, nullptr, nullptr, nullptr,
                                     nullptr, s));
    rc = gemm(b->ff1, h, rows, D, nullptr, 0, IDOL_ACT_GELU_TANH, big, IDOL_BF16, b->hidden, s);
    if (rc != IDOL_OK) return rc;
    return gemm(b->ff2, big, rows, b->hidden, x, D, IDOL_ACT_NONE, x, x_dtype, D, s);
}

int idol_b200_gaussian_mlp_create(const idol_q8_matrix* l0, const idol_q8_matrix* l1, const idol_q8_matrix* l2,
                                  idol_gaussian_mlp** mlp) {
    if (!mlp) return fail(IDOL_ERR_INVALID, "gaussian_mlp_create: mlp is NULL");
    *mlp = nullptr;
    if (!l0 || !l1 || !l2) return fail(IDOL_ERR_INVALID, "gaussian_mlp_create: NULL");
    if (l1->m.k != l0->m.n || l2->m.k != l1->m.n || l2->m.n != 14)
        return fail(IDOL_ERR_INVALID, "gaussian_mlp_create: layer shapes must chain and end in 14 outputs");
    if (l0->m.n % 8 || l1->m.n % 8) return fail(IDOL_ERR_INVALID, "gaussian_mlp_create: hidden widths % 8 != 0");
    *mlp = new idol_gaussian_mlp{l0, l1, l2, l0->m.device};
    return IDOL_OK;
}

int idol_b200_gaussian_mlp_free(idol_gaussian_mlp* mlp) {
    delete mlp;
    return IDOL_OK;
}

int64_t idol_b200_gaussian_mlp_workspace_bytes(const idol_gaussian_mlp* mlp, int64_t points) {
    if (!mlp || points < 0) return -1;
    return align256(points * mlp->l0->m.n * 2) + align256(points * mlp->l1->m.n * 2) + align256(points * 14 * 4);
}

int idol_b200_gaussian_mlp_forward(const idol_gaussian_mlp* mlp, const void* x, int64_t points, int64_t ldx,
                                   void* workspace, int64_t workspace_bytes, float* raw_out, float* out,
                                   void* stream) {
    if (!mlp || !x || !out) return fail(IDOL_ERR_INVALID, "gaussian_mlp_forward: NULL");
    if (points < 0) return fail(IDOL_ERR_INVALID, "gaussian_mlp_forward: points < 0");
    if (points == 0) return IDOL_OK;
    if (!workspace || workspace_bytes < idol_b200_gaussian_mlp_workspace_bytes(mlp, points) ||
        reinterpret_cast<uintptr_t>(workspace) % 256)
        return fail(IDOL_ERR_INVALID, "gaussian_mlp_forward: workspace too small or not 256-byte aligned");
    IDOL_CUDA(cudaSetDevice(mlp->device));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int h0 = mlp->l0->m.n, h1 = mlp->l1->m.n;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    // The two hidden activations stay in fp16 (8x finer than bf16; SiLU outputs of this MLP are far inside its
    // range), so layers 1 and 2 run the kernel's f16 operand path with fp16(d * q) weights.
    __half* a = reinterpret_cast<__half*>(ws);
    __half* b = reinterpret_cast<__half*>(ws + align256(points * h0 * 2));
    float* raw = raw_out ? raw_out : reinterpret_cast<float*>(ws + align256(points * h0 * 2) + align256(points * h1 * 2));
    int rc = gemm(mlp->l0, x, points, ldx, nullptr, 0, IDOL_ACT_SILU, a, IDOL_F16, h0, s);
    if (rc != IDOL_OK) return rc;
    rc = gemm(mlp->l1, a, points, h0, nullptr, 0, IDOL_ACT_SILU, b, IDOL_F16, h1, s, IDOL_F16);
    if (rc != IDOL_OK) return rc;
    rc = gemm(mlp->l2, b, points, h1, nullptr, 0, IDOL_ACT_NONE, raw, IDOL_F32, 14, s, IDOL_F16);
    if (rc != IDOL_OK) return rc;
    IDOL_CUDA(idol::launch_gaussian_heads(raw, IDOL_F32, points, 14, out, s));
    return IDOL_OK;
}

}  // extern "C"

namespace {

// Scratch of idol_b200_gaussian_mlp_forward_static: a fixed 8 MiB per GPU, reserved when the library's device code
// is loaded on that GPU and held until the process exits. Host code must not use this name as an address (on the
// host it is only a stand-in for the device symbol): the device address comes from cudaGetSymbolAddress below.
constexpr int64_t kStaticMlpScratchBytes = 8ll << 20;
static __device__ __align__(256) unsigned char g_mlp_static_scratch[kStaticMlpScratchBytes];

std::mutex g_static_scratch_mutex;
void* g_static_scratch_ptr[64] = {};

// Device address of the scratch on the current device (`device`), looked up once per device.
int static_scratch(int device, void** ptr) {
    if (device < 0 || device >= 64) return fail(IDOL_ERR_INVALID, "gaussian_mlp_forward_static: device index");
    std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
    if (!g_static_scratch_ptr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_mlp_static_scratch);
        if (e != cudaSuccess) return idol::cuda_fail(e, "cudaGetSymbolAddress (static MLP scratch)");
        g_static_scratch_ptr[device] = p;
    }
    *ptr = g_static_scratch_ptr[device];
    return IDOL_OK;
}

}  // namespace

extern "C" {

int idol_b200_gaussian_mlp_forward_static(const idol_gaussian_mlp* mlp, const void* x, int64_t points, int64_t ldx,
                                          float* raw_out, float* out, void* stream) {
    if (!mlp) return fail(IDOL_ERR_INVALID, "gaussian_mlp_forward_static: mlp is NULL");
    const int64_t need = idol_b200_gaussian_mlp_workspace_bytes(mlp, points);
    if (need < 0) return fail(IDOL_ERR_INVALID, "gaussian_mlp_forward_static: points < 0");
    if (need > kStaticMlpScratchBytes)
        return fail(IDOL_ERR_INVALID, "gaussian_mlp_forward_static: " + std::to_string(points) + " points need " +
                                          std::to_string(need) + " bytes of scratch, more than the fixed " +
                                          std::to_string(kStaticMlpScratchBytes) +
                                          " bytes this entry point has; split the batch or pass a workspace to "
                                          "idol_b200_gaussian_mlp_forward");
    IDOL_CUDA(cudaSetDevice(mlp->device));
    void* scratch = nullptr;
    const int rc = static_scratch(mlp->device, &scratch);
    if (rc != IDOL_OK) return rc;
    return idol_b200_gaussian_mlp_forward(mlp, x, points, ldx, scratch, kStaticMlpScratchBytes, raw_out, out, stream);
}

int idol_b200_gaussian_heads(const void* raw, int raw_dtype, int64_t points, int64_t ld, float* out, void* stream) {
    if (points < 0 || ld < 14) return fail(IDOL_ERR_INVALID, "gaussian_heads: sizes");
    if (points == 0) return IDOL_OK;
    if (!raw || !out) return fail(IDOL_ERR_INVALID, "gaussian_heads: NULL");
    IDOL_CUDA(idol::launch_gaussian_heads(raw, raw_dtype, points, ld, out, static_cast<cudaStream_t>(stream)));
    return IDOL_OK;
}

}  // extern "C"
