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
#include <vector>

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

// The Gaussian decoder's input (src/decoders.cpp:289-290): x[r, j] = sum_c points[r, c] w_in[j, c] (fp32 FMA chain)
// + b_in[j] + pos_embed(points[r])[j], where pos_embed (src/decoders.cpp:215-230) is sin((v f) pi) for column
// 2 c fd + i and cos((v f) pi) for 2 c fd + fd + i (v the row's coordinate c, f = freqs[i]), zero from 6 fd on.
// The sines use the full-range sinf/cosf: the angles reach thousands of radians. Written as bf16 (the next GEMM's
// input). One thread per element.
constexpr float kPiF = 3.14159265358979323846f;
__global__ void gs_input_kernel(const float* __restrict__ points, long long rows, int dim,
                                const float* __restrict__ w, const float* __restrict__ b,
                                const float* __restrict__ freqs, int fd, __nv_bfloat16* __restrict__ out) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * dim) return;
    const long long r = idx / dim;
    const int j = (int)(idx % dim);
    const float p0 = points[r * 3], p1 = points[r * 3 + 1], p2 = points[r * 3 + 2];
    float acc = fmaf(p0, w[j * 3], 0.0f);
    acc = fmaf(p1, w[j * 3 + 1], acc);
    acc = fmaf(p2, w[j * 3 + 2], acc);
    float v = acc + (b ? b[j] : 0.0f);
    if (j < 6 * fd) {
        const int c = j / (2 * fd), i = j % (2 * fd);
        const float coord = c == 0 ? p0 : (c == 1 ? p1 : p2);
        const float ang = (coord * freqs[i < fd ? i : i - fd]) * kPiF;
        v += i < fd ? sinf(ang) : cosf(ang);
    }
    out[idx] = __float2bfloat16_rn(v);
}

// Decoders::to_gaussians (src/decoders.cpp:393-433), one thread per Gaussian (anchor a, g < G): from the anchor's
// 15 G raw features, offset xyz = tanh(f lr_xyz + perturbation) 0.5 perturbe softplus(f_os + base_offset_scale)
// placed around the anchor and shifted by -0.5; colour f lr_dc; scale sqrt(softplus(f lr_scaling + scale_offset)^2 +
// kernel^2); rotation (f lr_rotation + (1, 0, 0, 0)) normalised (|.| floored at 1e-12); opacity sigmoid(f lr_opacity
// + opacity_offset). softplus(x) = x above 20, else log1p(exp(x)) (src/decoders.cpp:90). The offsets are computed
// on the host in double as the reference does.
struct GsRep {
    float perturbe, kernel, lr_xyz, lr_dc, lr_opacity, lr_scaling, lr_rotation, scale_offset, opacity_offset,
        base_offset_scale;
};
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
__global__ void to_gaussians_kernel(const float* __restrict__ anchors, long long rows, const float* __restrict__ f,
                                    int G, const float* __restrict__ perturbation, GsRep rp,
                                    float* __restrict__ xyz, float* __restrict__ f_dc, float* __restrict__ scale,
                                    float* __restrict__ rotation, float* __restrict__ opacity) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * G) return;
    const long long a = i / G;
    const int g = (int)(i % G);
    const float* fa = f + a * (long long)G * 15;
    const float offset_scale = softplus_f(fa[G * 14 + g] + rp.base_offset_scale);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float o = tanhf(fa[g * 3 + c] * rp.lr_xyz + perturbation[g * 3 + c]) * 0.5f * rp.perturbe *
                        offset_scale;
        xyz[i * 3 + c] = (o + anchors[a * 3 + c]) - 0.5f;
        f_dc[i * 3 + c] = fa[G * 3 + g * 3 + c] * rp.lr_dc;
        const float sp = softplus_f(fa[G * 6 + g * 3 + c] * rp.lr_scaling + rp.scale_offset);
        scale[i * 3 + c] = sqrtf(sp * sp + rp.kernel * rp.kernel);
    }
    float q[4], norm = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        q[c] = fa[G * 9 + g * 4 + c] * rp.lr_rotation + (c == 0 ? 1.0f : 0.0f);
        norm += q[c] * q[c];
    }
    norm = fmaxf(sqrtf(norm), 1e-12f);
#pragma unroll
    for (int c = 0; c < 4; ++c) rotation[i * 4 + c] = q[c] / norm;
    opacity[i] = 1.0f / (1.0f + expf(-(fa[G * 13 + g] * rp.lr_opacity + rp.opacity_offset)));
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


// The same projection for the 16-wide condition of the real model, with rms_heads of the key half fused in
// (src/decoders.cpp:237 then :238): a half-warp owns one 64-column head and a lane four adjacent columns, whose 64
// weights stay in registers; a CTA covers 1024 columns of 32 rows, the rows' conditions staged in shared memory. Each
// value is the FMA chain of kv_project_kernel rounded to bf16; a key head is then normalised from those rounded
// values, x * 8 / max(|x|, 1e-12) * gamma (head dim 64), and rounded again, as rms_heads does to the stored row; each
// lane stores its four columns as one 8-byte word.
constexpr int kKv16Rows = 32;
__global__ void __launch_bounds__(256) kv_project16_kernel(const float* __restrict__ cond, long long rows,
                                                           const float* __restrict__ w, const float* __restrict__ b,
                                                           int cols, int key_cols, const float* __restrict__ k_gamma,
                                                           __nv_bfloat16* __restrict__ kv) {
    __shared__ float cs[kKv16Rows][16];
    const long long r0 = (long long)blockIdx.y * kKv16Rows;
    for (int i = threadIdx.x; i < kKv16Rows * 16; i += blockDim.x) {
        const long long r = r0 + i / 16;
        cs[i / 16][i % 16] = r < rows ? cond[r * 16 + i % 16] : 0.0f;
    }
    __syncthreads();
    const int j0 = blockIdx.x * 1024 + threadIdx.x * 4;  // this lane's four columns; a warp's 128 are whole heads
    if (j0 >= cols) return;
    float wr[4][16];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int c = 0; c < 16; c += 4) {
            const float4 v = *reinterpret_cast<const float4*>(w + (long long)(j0 + u) * 16 + c);
            wr[u][c] = v.x;
            wr[u][c + 1] = v.y;
            wr[u][c + 2] = v.z;
            wr[u][c + 3] = v.w;
        }
    float bj[4], gj[4];
    const bool key = k_gamma != nullptr && j0 < key_cols;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        bj[u] = b ? b[j0 + u] : 0.0f;
        gj[u] = key ? k_gamma[(j0 + u) % key_cols] : 1.0f;
    }
    for (int i = 0; i < kKv16Rows; ++i) {
        const long long r = r0 + i;
        if (r >= rows) break;
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float acc = 0.0f;
#pragma unroll
            for (int c = 0; c < 16; ++c) acc = fmaf(cs[i][c], wr[u][c], acc);
            v[u] = __bfloat162float(__float2bfloat16_rn(acc + bj[u]));
        }
        // The half-warp holds one head: its sum of squares over the 16 lanes (every lane of the warp takes part in
        // the shuffles; value heads discard the result).
        float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (key) {
            const float mult = 8.0f / fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = v[u] * mult * gj[u];
        }
        __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
        uint2 pkt;
        pkt.x = *reinterpret_cast<uint32_t*>(&lo);
        pkt.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(kv + r * cols + j0) = pkt;
    }
}

}  // namespace

cudaError_t launch_decoder_input(const float* points, long long rows, int dim, const float* w, const float* b,
                                 const float* freqs, int fd, __nv_bfloat16* out, cudaStream_t s) {
    const long long n = rows * dim;
    if (n == 0) return cudaSuccess;
    gs_input_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(points, rows, dim, w, b, freqs, fd, out);
    return cudaGetLastError();
}

cudaError_t launch_kv_project(const float* cond, long long rows, int cdim, const float* w, const float* b, int cols,
                              __nv_bfloat16* kv, cudaStream_t s, const float* k_gamma, int heads) {
    if (rows == 0) return cudaSuccess;
    const int key_cols = cols / 2;
    const bool fast = cdim == 16 && cols % 128 == 0 && key_cols % 64 == 0 &&
                      reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(kv) % 8 == 0 &&
                      (rows + kKv16Rows - 1) / kKv16Rows <= 65535;
    if (fast) {
        const dim3 grid((unsigned)((cols + 1023) / 1024), (unsigned)((rows + kKv16Rows - 1) / kKv16Rows));
        kv_project16_kernel<<<grid, 256, 0, s>>>(cond, rows, w, b, cols, key_cols, k_gamma, kv);
        return cudaGetLastError();
    }
    if (cdim < 1 || cdim > kKvMaxCond || rows > 65535LL * 16) return cudaErrorInvalidValue;
    const dim3 grid((unsigned)((cols + 255) / 256), (unsigned)((rows + 15) / 16));
    kv_project_kernel<<<grid, 256, 0, s>>>(cond, rows, cdim, w, b, cols, kv);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !k_gamma) return e;
    return launch_rms_heads(kv, IDOL_BF16, cols, rows, heads, k_gamma, s);
}

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

struct idol_gs_decoder {
    std::vector<const idol_gs_block*> blocks;
    const float* in_w;                   // fp32 [D, 3]
    const float* in_b;                   // fp32 [D] or NULL
    const idol_q8_matrix* input_layer;   // D x D
    const idol_q8_matrix* out_proj;      // per_anchor * 15 x D
    const float* freqs;                  // fp32 [n_freqs]
    int n_freqs, per_anchor, dim, device;
    const float* perturbation;           // fp32 [per_anchor * 3]
    idol::GsRep rep;
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

// A projection into bf16 followed by rms_heads (src/decoders.cpp:74-86) of its first `cols` columns: [0, split) with
// gamma_a, [split, cols) with gamma_b. The norm runs in the GEMM's epilogue where it can, else right after it.
int gemm_heads(const idol_q8_matrix* w, const void* x, int64_t m, int64_t ldx, void* y, int64_t ldy, int cols, int split,
               const float* gamma_a, const float* gamma_b, cudaStream_t s) {
    idol::GemmCall c = {&w->m, x, IDOL_BF16, m, ldx, 0, w->m.n, nullptr, 0, IDOL_ACT_NONE, 0, y, IDOL_BF16, ldy, s};
    c.head_gamma_a = gamma_a;
    c.head_gamma_b = gamma_b;
    c.head_cols = cols;
    c.head_split = split;
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
    int rc = gemm_heads(b->qkv, h, rows, D, big, 3 * D, 2 * D, D, b->q_gamma, b->k_gamma, s);  // with rms q, k
    if (rc != IDOL_OK) return rc;
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
    int rc = gemm_heads(b->qkv, h, rows, D, big, 3 * D, 2 * D, D, b->q_gamma, b->k_gamma, s);  // with rms q, k
    if (rc != IDOL_OK) return rc;
    idol::AttentionCall sa = {big, big + D, big + 2 * D, h, tokens, tokens, 3 * D, 3 * D, D, b->heads, 64, images, s};
    rc = idol::attention(sa);
    if (rc != IDOL_OK) return rc;
    rc = gemm(b->out, h, rows, D, x, D, IDOL_ACT_NONE, x, x_dtype, D, s);
    if (rc != IDOL_OK) return rc;

    // Cross-attention sublayer (src/decoders.cpp:304-306, 232-240).
    IDOL_CUDA(idol::launch_norm_rows(x, x_dtype, D, h, IDOL_BF16, D, rows, D, b->eps, g->norm2_gamma, g->norm2_beta,
                                     nullptr, nullptr, s));
    rc = gemm_heads(g->cross_q, h, rows, D, big, D, D, D, g->cq_gamma, nullptr, s);  // with rms q
    if (rc != IDOL_OK) return rc;
    // to_kv of the condition rows with the key half's rms_heads fused in.
    IDOL_CUDA(idol::launch_kv_project(cond, crows, g->cond_dim, g->kv_w, g->kv_b, 2 * D, kv, s, g->ck_gamma,
                                      b->heads));
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

int idol_b200_gs_decoder_create(const idol_gs_block* const* blocks, int nblocks, const float* in_w, const float* in_b,
                                const idol_q8_matrix* input_layer, const idol_q8_matrix* out_proj, const float* freqs,
                                int n_freqs, int per_anchor, const float* perturbation, float base_offset_scale,
                                const float* rep, idol_gs_decoder** decoder) {
    if (!decoder) return fail(IDOL_ERR_INVALID, "gs_decoder_create: decoder is NULL");
    *decoder = nullptr;
    if (nblocks < 0 || (nblocks > 0 && !blocks) || !in_w || !input_layer || !out_proj || !freqs || !perturbation ||
        !rep)
        return fail(IDOL_ERR_INVALID, "gs_decoder_create: NULL");
    const int D = input_layer->m.n;
    if (input_layer->m.k != D || out_proj->m.k != D || per_anchor < 1 || out_proj->m.n != per_anchor * 15)
        return fail(IDOL_ERR_INVALID, "gs_decoder_create: input_layer D x D and out_proj (15 per_anchor) x D expected");
    if (n_freqs < 0 || 6 * n_freqs > D) return fail(IDOL_ERR_INVALID, "gs_decoder_create: 6 n_freqs must be <= D");
    if (!idol::norm_dim_ok(D)) return fail(IDOL_ERR_UNSUPPORTED, "gs_decoder_create: width not supported by norm_rows");
    const int dev = input_layer->m.device;
    for (int i = 0; i < nblocks; ++i)
        if (!blocks[i] || blocks[i]->self.dim != D || blocks[i]->self.device != dev)
            return fail(IDOL_ERR_INVALID, "gs_decoder_create: every block must have width D on the decoder's device");
    if (out_proj->m.device != dev) return fail(IDOL_ERR_INVALID, "gs_decoder_create: matrices on different devices");
    // rep: perturbe, kernel, scaling_bias, opacity_bias, lr_xyz, lr_dc, lr_opacity, lr_scaling, lr_rotation
    // (src/weights.hpp:25-28); the two activation offsets in double as src/decoders.cpp:397-399 forms them.
    const double sb = rep[2], ob = rep[3];
    if (!(sb > 0.0) || !(ob > 0.0 && ob < 1.0))
        return fail(IDOL_ERR_INVALID, "gs_decoder_create: scaling_bias > 0 and 0 < opacity_bias < 1 expected");
    idol::GsRep rp = {rep[0], rep[1], rep[4], rep[5], rep[6], rep[7], rep[8],
                      (float)(sb + std::log(-std::expm1(-sb))), (float)std::log(ob / (1.0 - ob)), base_offset_scale};
    auto* d = new idol_gs_decoder();
    d->blocks.assign(blocks, blocks + nblocks);
    d->in_w = in_w;
    d->in_b = in_b;
    d->input_layer = input_layer;
    d->out_proj = out_proj;
    d->freqs = freqs;
    d->n_freqs = n_freqs;
    d->per_anchor = per_anchor;
    d->dim = D;
    d->device = dev;
    d->perturbation = perturbation;
    d->rep = rp;
    *decoder = d;
    return IDOL_OK;
}

int idol_b200_gs_decoder_free(idol_gs_decoder* decoder) {
    delete decoder;
    return IDOL_OK;
}

int64_t idol_b200_gs_decoder_workspace_bytes(const idol_gs_decoder* d, int64_t rows, int64_t cond_rows) {
    if (!d || rows < 0 || cond_rows < 0) return -1;
    int64_t blk = 0;
    for (const idol_gs_block* b : d->blocks) {
        const int64_t v = idol_b200_gs_block_workspace_bytes(b, rows, cond_rows);
        blk = v > blk ? v : blk;
    }
    const int64_t own = align256(rows * d->dim * 4) + align256(rows * d->dim * 2);  // x (fp32) + h (bf16)
    return own + blk;
}

int idol_b200_gs_decoder_features(const idol_gs_decoder* d, const float* points, int64_t rows, const float* cond,
                                  int64_t cond_rows, float* features, void* workspace, int64_t workspace_bytes,
                                  void* stream) {
    if (!d || !points || !features || (!d->blocks.empty() && !cond))
        return fail(IDOL_ERR_INVALID, "gs_decoder_features: NULL");
    if (rows < 1 || cond_rows < 1) return fail(IDOL_ERR_INVALID, "gs_decoder_features: rows and cond_rows >= 1");
    if (!workspace || workspace_bytes < idol_b200_gs_decoder_workspace_bytes(d, rows, cond_rows) ||
        reinterpret_cast<uintptr_t>(workspace) % 256)
        return fail(IDOL_ERR_INVALID, "gs_decoder_features: workspace smaller than "
                                      "idol_b200_gs_decoder_workspace_bytes or not 256-byte aligned");
    IDOL_CUDA(cudaSetDevice(d->device));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int D = d->dim;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* x = reinterpret_cast<float*>(ws);                                          // rows x D fp32
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(ws + align256(rows * D * 4));  // rows x D bf16
    uint8_t* blk_ws = ws + align256(rows * D * 4) + align256(rows * D * 2);
    const int64_t blk_bytes = workspace_bytes - (blk_ws - ws);

    const long long n = rows * D;
    idol::gs_input_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(points, rows, D, d->in_w, d->in_b, d->freqs,
                                                                       d->n_freqs, h);
    IDOL_CUDA(cudaGetLastError());
    int rc = gemm(d->input_layer, h, rows, D, nullptr, 0, IDOL_ACT_NONE, x, IDOL_F32, D, s);
    if (rc != IDOL_OK) return rc;
    for (const idol_gs_block* b : d->blocks) {
        rc = idol_b200_gs_block_forward(b, x, IDOL_F32, rows, 1, cond, cond_rows, blk_ws, blk_bytes, stream);
        if (rc != IDOL_OK) return rc;
    }
    IDOL_CUDA(idol::launch_norm_rows(x, IDOL_F32, D, h, IDOL_BF16, D, rows, D, 1e-5f, nullptr, nullptr, nullptr,
                                     nullptr, s));
    return gemm(d->out_proj, h, rows, D, nullptr, 0, IDOL_ACT_NONE, features, IDOL_F32, d->out_proj->m.n, s);
}

int idol_b200_gs_to_gaussians(const idol_gs_decoder* d, const float* anchors, int64_t rows, const float* features,
                              float* xyz, float* f_dc, float* scale, float* rotation, float* opacity, void* stream) {
    if (!d || !anchors || !features || !xyz || !f_dc || !scale || !rotation || !opacity)
        return fail(IDOL_ERR_INVALID, "gs_to_gaussians: NULL");
    if (rows < 0) return fail(IDOL_ERR_INVALID, "gs_to_gaussians: rows < 0");
    if (rows == 0) return IDOL_OK;
    IDOL_CUDA(cudaSetDevice(d->device));
    const long long n = rows * d->per_anchor;
    idol::to_gaussians_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        anchors, rows, features, d->per_anchor, d->perturbation, d->rep, xyz, f_dc, scale, rotation, opacity);
    IDOL_CUDA(cudaGetLastError());
    return IDOL_OK;
}

int idol_b200_gaussian_mlp_create(const idol_q8_matrix* l0, const idol_q8_matrix* l1, const idol_q8_matrix* l2,
                                  idol_gaussian_mlp** mlp) {
    if (!mlp) return fail(IDOL_ERR_INVALID, "gaussian_mlp_create: mlp is NULL");
    *mlp = nullptr;
    if (!l0 || !l1 || !l2) return fail(IDOL_ERR_INVALID, "gaussian_mlp_create: NULL");
    if (l1->m.device != l0->m.device || l2->m.device != l0->m.device)
        return fail(IDOL_ERR_INVALID, "gaussian_mlp_create: matrices on different devices");
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
    const idol::NoScratchScope no_library_scratch;  // the GEMMs keep the kernels that need no scratch of their own
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
