// octree.cu - the octree decoder (Decoders::octree_logits and sample_anchors, src/decoders.cpp:242-282, 335-391).
//
//   logits(x, resolution):                         x: cell centres [rows, 3] in [0, 1]^3
//       X = in_proj(x) + pos_embed(x) -> input_layer                      the decoders' input kernel + q8 GEMM
//       mod = ada(silu(l2(silu(l1(level_embed(resolution))))))            one 256-wide embedding, three M = 1 GEMVs
//       per block: h = LN(X) * (1 + scale_a) + shift_a; a = cross-attention(h, cond); X += (a W_o^T + b) * gate_a
//                  h = LN(X) * (1 + scale_m) + shift_m; X += (gelu_tanh(h W_1^T + b) W_2^T + b) * gate_m
//       logits = LN(X, 1e-5) W_out^T + b                                  8 per cell
//   sample_anchors(num_points, level, seed): from the root cell, per level the occupied cells' logits are computed on
//   the GPU and copied back; the host takes a softmax over the eight children and resamples each cell's points among
//   them systematically with one uniform draw per cell, exactly in the reference's order and arithmetic (mt19937_64,
//   uniform_real_distribution<float>), so the same seed draws the same numbers; the leaf points are placed uniformly
//   inside their cells. The GPU does the dense work; the host keeps the sampling, whose cost is a few floats per cell.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <vector>

#include "internal.h"

namespace idol {
namespace {

constexpr float kPiF = 3.14159265358979323846f;

// The level embedding (src/decoders.cpp:254-259): cos(((resolution f) 2) pi) for the 128 level frequencies, then sin,
// as the bf16 input of the first embedding GEMV.
__global__ void level_embed_kernel(float resolution, const float* __restrict__ freqs,
                                   __nv_bfloat16* __restrict__ out) {
    const int i = threadIdx.x;
    if (i >= 128) return;
    const float ang = ((resolution * freqs[i]) * 2.0f) * kPiF;
    out[i] = __float2bfloat16_rn(cosf(ang));
    out[128 + i] = __float2bfloat16_rn(sinf(ang));
}

// x[r, c] += h[r, c] * gate[c] (src/decoders.cpp:45-52 add_gated), fp32.
__global__ void add_gated_kernel(float* __restrict__ x, const float* __restrict__ h, long long rows, int dim,
                                 const float* __restrict__ gate) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * dim) return;
    x[i] += h[i] * gate[i % dim];
}

inline int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

int gemm(const idol_q8_matrix* w, const void* x, int64_t m, int64_t ldx, int act, void* y, int y_dtype, int64_t ldy,
         cudaStream_t s) {
    GemmCall c = {&w->m, x, IDOL_BF16, m, ldx, 0, w->m.n, nullptr, 0, act, 0, y, y_dtype, ldy, s};
    return q8_gemm(c);
}

}  // namespace
}  // namespace idol

using idol::fail;

struct idol_oct_block {
    const idol_q8_matrix* cross_q;
    const idol_q8_matrix* cross_out;
    const idol_q8_matrix* ff1;
    const idol_q8_matrix* ff2;
    const float* cq_gamma;
    const float* ck_gamma;
    const float* kv_w;  // fp32 [2D, cond_dim]
    const float* kv_b;  // fp32 [2D] or NULL
    int cond_dim, dim, hidden, heads, device;
};

struct idol_oct_decoder {
    std::vector<const idol_oct_block*> blocks;
    const float* in_w;
    const float* in_b;
    const idol_q8_matrix* input_layer;
    const idol_q8_matrix* l1;
    const idol_q8_matrix* l2;
    const idol_q8_matrix* ada;
    const idol_q8_matrix* out_proj;
    const float* freqs;
    const float* level_freqs;
    int n_freqs, dim, hidden, heads, cond_dim, device;
    float eps;
};

struct idol_oct_sampler {
    std::mt19937_64 rng;
    std::uniform_real_distribution<float> uniform{0.0f, 1.0f};
    std::vector<uint32_t> coords{0, 0, 0};
    std::vector<int64_t> counts;
    int level = 0, levels = 0;  // levels resampled so far, and in all
    int num_points = 0;
};

namespace {

// Workspace layout of a logits call over `rows` cells and `cond_rows` condition rows.
struct OctWorkspace {
    float* x;               // rows x D fp32 (residual stream)
    __nv_bfloat16* h;       // rows x D
    __nv_bfloat16* big;     // rows x max(D, hidden)
    float* tmp;             // rows x D fp32 (sublayer output before the gate)
    __nv_bfloat16* kv;      // cond_rows x 2D
    float* mod;             // 6 D
    __nv_bfloat16* emb;     // 256
    __nv_bfloat16* l1o;     // D
    __nv_bfloat16* l2o;     // D
    float* centres;         // rows x 3 (sample_anchors)
    float* logits;          // rows x 8 (sample_anchors)
    int64_t bytes;
};

OctWorkspace oct_layout(const idol_oct_decoder* d, int64_t rows, int64_t cond_rows, uint8_t* base) {
    const int64_t D = d->dim, big = std::max<int64_t>(d->dim, d->hidden);
    const int64_t sizes[11] = {rows * D * 4, rows * D * 2, rows * big * 2, rows * D * 4, cond_rows * 2 * D * 2,
                               6 * D * 4,   256 * 2,      D * 2,          D * 2,        rows * 3 * 4,
                               rows * 8 * 4};
    int64_t off[11], total = 0;
    for (int i = 0; i < 11; ++i) {
        off[i] = total;
        total += idol::align256(sizes[i]);
    }
    OctWorkspace w = {};
    w.bytes = total;
    if (!base) return w;  // sizing only
    w.x = reinterpret_cast<float*>(base + off[0]);
    w.h = reinterpret_cast<__nv_bfloat16*>(base + off[1]);
    w.big = reinterpret_cast<__nv_bfloat16*>(base + off[2]);
    w.tmp = reinterpret_cast<float*>(base + off[3]);
    w.kv = reinterpret_cast<__nv_bfloat16*>(base + off[4]);
    w.mod = reinterpret_cast<float*>(base + off[5]);
    w.emb = reinterpret_cast<__nv_bfloat16*>(base + off[6]);
    w.l1o = reinterpret_cast<__nv_bfloat16*>(base + off[7]);
    w.l2o = reinterpret_cast<__nv_bfloat16*>(base + off[8]);
    w.centres = reinterpret_cast<float*>(base + off[9]);
    w.logits = reinterpret_cast<float*>(base + off[10]);
    return w;
}

int oct_logits(const idol_oct_decoder* d, const float* x, int64_t rows, float resolution, const float* cond,
               int64_t cond_rows, float* out, const OctWorkspace& w, cudaStream_t s) {
    const int D = d->dim;
    IDOL_CUDA(idol::launch_decoder_input(x, rows, D, d->in_w, d->in_b, d->freqs, d->n_freqs, w.h, s));
    int rc = idol::gemm(d->input_layer, w.h, rows, D, IDOL_ACT_NONE, w.x, IDOL_F32, D, s);
    if (rc != IDOL_OK) return rc;
    idol::level_embed_kernel<<<1, 128, 0, s>>>(resolution, d->level_freqs, w.emb);
    IDOL_CUDA(cudaGetLastError());
    if ((rc = idol::gemm(d->l1, w.emb, 1, 256, IDOL_ACT_SILU, w.l1o, IDOL_BF16, D, s)) != IDOL_OK) return rc;
    if ((rc = idol::gemm(d->l2, w.l1o, 1, D, IDOL_ACT_SILU, w.l2o, IDOL_BF16, D, s)) != IDOL_OK) return rc;
    if ((rc = idol::gemm(d->ada, w.l2o, 1, D, IDOL_ACT_NONE, w.mod, IDOL_F32, 6 * D, s)) != IDOL_OK) return rc;
    const float *shift_a = w.mod, *scale_a = w.mod + D, *gate_a = w.mod + 2 * D, *shift_m = w.mod + 3 * D,
                *scale_m = w.mod + 4 * D, *gate_m = w.mod + 5 * D;
    const long long n = rows * D;
    const unsigned grid = (unsigned)((n + 255) / 256);
    for (const idol_oct_block* b : d->blocks) {
        IDOL_CUDA(idol::launch_norm_rows(w.x, IDOL_F32, D, w.h, IDOL_BF16, D, rows, D, d->eps, nullptr, nullptr,
                                         shift_a, scale_a, s));
        if ((rc = idol::gemm(b->cross_q, w.h, rows, D, IDOL_ACT_NONE, w.big, IDOL_BF16, D, s)) != IDOL_OK) return rc;
        IDOL_CUDA(idol::launch_rms_heads(w.big, IDOL_BF16, D, rows, d->heads, b->cq_gamma, s));
        IDOL_CUDA(idol::launch_kv_project(cond, cond_rows, b->cond_dim, b->kv_w, b->kv_b, 2 * D, w.kv, s, b->ck_gamma,
                                          d->heads));
        idol::AttentionCall ac = {w.big, w.kv, w.kv + D, w.h, rows, cond_rows, D, 2 * D, D, d->heads, 64, 1, s};
        if ((rc = idol::attention(ac)) != IDOL_OK) return rc;
        if ((rc = idol::gemm(b->cross_out, w.h, rows, D, IDOL_ACT_NONE, w.tmp, IDOL_F32, D, s)) != IDOL_OK) return rc;
        idol::add_gated_kernel<<<grid, 256, 0, s>>>(w.x, w.tmp, rows, D, gate_a);
        IDOL_CUDA(cudaGetLastError());
        IDOL_CUDA(idol::launch_norm_rows(w.x, IDOL_F32, D, w.h, IDOL_BF16, D, rows, D, d->eps, nullptr, nullptr,
                                         shift_m, scale_m, s));
        if ((rc = idol::gemm(b->ff1, w.h, rows, D, IDOL_ACT_GELU_TANH, w.big, IDOL_BF16, b->hidden, s)) != IDOL_OK)
            return rc;
        if ((rc = idol::gemm(b->ff2, w.big, rows, b->hidden, IDOL_ACT_NONE, w.tmp, IDOL_F32, D, s)) != IDOL_OK)
            return rc;
        idol::add_gated_kernel<<<grid, 256, 0, s>>>(w.x, w.tmp, rows, D, gate_m);
        IDOL_CUDA(cudaGetLastError());
    }
    IDOL_CUDA(idol::launch_norm_rows(w.x, IDOL_F32, D, w.h, IDOL_BF16, D, rows, D, 1e-5f, nullptr, nullptr, nullptr,
                                     nullptr, s));
    return idol::gemm(d->out_proj, w.h, rows, D, IDOL_ACT_NONE, out, IDOL_F32, 8, s);
}

}  // namespace

extern "C" {

int idol_b200_oct_block_create(const idol_q8_matrix* cross_q, const idol_q8_matrix* cross_out,
                               const idol_q8_matrix* ff1, const idol_q8_matrix* ff2, const float* cross_q_gamma,
                               const float* cross_k_gamma, const float* kv_weight, const float* kv_bias, int cond_dim,
                               int heads, idol_oct_block** block) {
    if (!block) return fail(IDOL_ERR_INVALID, "oct_block_create: block is NULL");
    *block = nullptr;
    if (!cross_q || !cross_out || !ff1 || !ff2 || !cross_q_gamma || !cross_k_gamma || !kv_weight)
        return fail(IDOL_ERR_INVALID, "oct_block_create: NULL");
    const int D = cross_q->m.n;
    if (heads < 1 || D != heads * 64) return fail(IDOL_ERR_UNSUPPORTED, "oct_block_create: head_dim must be 64");
    if (cross_q->m.k != D || cross_out->m.n != D || cross_out->m.k != D || ff1->m.k != D || ff2->m.n != D ||
        ff2->m.k != ff1->m.n)
        return fail(IDOL_ERR_INVALID, "oct_block_create: to_q, to_out (D x D), ff1 (H x D), ff2 (D x H) expected");
    if (cond_dim < 1 || cond_dim > 64) return fail(IDOL_ERR_UNSUPPORTED, "oct_block_create: cond_dim must be 1..64");
    const int dev = cross_q->m.device;
    if (cross_out->m.device != dev || ff1->m.device != dev || ff2->m.device != dev)
        return fail(IDOL_ERR_INVALID, "oct_block_create: matrices on different devices");
    *block = new idol_oct_block{cross_q, cross_out,  ff1,      ff2, cross_q_gamma, cross_k_gamma, kv_weight, kv_bias,
                                cond_dim, D,       ff1->m.n, heads, dev};
    return IDOL_OK;
}

int idol_b200_oct_block_free(idol_oct_block* block) {
    delete block;
    return IDOL_OK;
}

int idol_b200_oct_decoder_create(const idol_oct_block* const* blocks, int nblocks, const float* in_w, const float* in_b,
                                 const idol_q8_matrix* input_layer, const idol_q8_matrix* l1,
                                 const idol_q8_matrix* l2, const idol_q8_matrix* ada, const idol_q8_matrix* out_proj,
                                 const float* freqs, int n_freqs, const float* level_freqs, int heads, float eps,
                                 idol_oct_decoder** decoder) {
    if (!decoder) return fail(IDOL_ERR_INVALID, "oct_decoder_create: decoder is NULL");
    *decoder = nullptr;
    if (nblocks < 0 || (nblocks > 0 && !blocks) || !in_w || !input_layer || !l1 || !l2 || !ada || !out_proj ||
        !freqs || !level_freqs)
        return fail(IDOL_ERR_INVALID, "oct_decoder_create: NULL");
    const int D = input_layer->m.n;
    if (heads < 1 || D != heads * 64) return fail(IDOL_ERR_UNSUPPORTED, "oct_decoder_create: head_dim must be 64");
    if (input_layer->m.k != D || l1->m.n != D || l1->m.k != 256 || l2->m.n != D || l2->m.k != D ||
        ada->m.n != 6 * D || ada->m.k != D || out_proj->m.n != 8 || out_proj->m.k != D)
        return fail(IDOL_ERR_INVALID, "oct_decoder_create: input_layer D x D, l1 D x 256, l2 D x D, ada 6D x D and "
                                      "out_proj 8 x D expected");
    if (n_freqs < 0 || 6 * n_freqs > D) return fail(IDOL_ERR_INVALID, "oct_decoder_create: 6 n_freqs must be <= D");
    if (!idol::norm_dim_ok(D))
        return fail(IDOL_ERR_UNSUPPORTED, "oct_decoder_create: width not supported by norm_rows");
    const int dev = input_layer->m.device;
    for (const idol_q8_matrix* m : {l1, l2, ada, out_proj})
        if (m->m.device != dev) return fail(IDOL_ERR_INVALID, "oct_decoder_create: matrices on different devices");
    int hidden = D, cond_dim = 0;
    for (int i = 0; i < nblocks; ++i) {
        if (!blocks[i] || blocks[i]->dim != D || blocks[i]->device != dev || blocks[i]->heads != heads ||
            (cond_dim && blocks[i]->cond_dim != cond_dim))
            return fail(IDOL_ERR_INVALID, "oct_decoder_create: blocks must share D, heads, cond_dim and the device");
        hidden = std::max(hidden, blocks[i]->hidden);
        cond_dim = blocks[i]->cond_dim;
    }
    auto* d = new idol_oct_decoder();
    d->blocks.assign(blocks, blocks + nblocks);
    d->in_w = in_w;
    d->in_b = in_b;
    d->input_layer = input_layer;
    d->l1 = l1;
    d->l2 = l2;
    d->ada = ada;
    d->out_proj = out_proj;
    d->freqs = freqs;
    d->level_freqs = level_freqs;
    d->n_freqs = n_freqs;
    d->dim = D;
    d->hidden = hidden;
    d->heads = heads;
    d->cond_dim = cond_dim;
    d->device = dev;
    d->eps = eps;
    *decoder = d;
    return IDOL_OK;
}

int idol_b200_oct_decoder_free(idol_oct_decoder* decoder) {
    delete decoder;
    return IDOL_OK;
}

int64_t idol_b200_oct_decoder_workspace_bytes(const idol_oct_decoder* d, int64_t rows, int64_t cond_rows) {
    if (!d || rows < 0 || cond_rows < 0) return -1;
    return oct_layout(d, rows, cond_rows, nullptr).bytes;
}

int idol_b200_oct_logits(const idol_oct_decoder* d, const float* x, int64_t rows, float resolution, const float* cond,
                         int64_t cond_rows, float* logits, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!d || !x || !logits || (!d->blocks.empty() && !cond)) return fail(IDOL_ERR_INVALID, "oct_logits: NULL");
    if (rows < 1 || cond_rows < 1) return fail(IDOL_ERR_INVALID, "oct_logits: rows and cond_rows must be >= 1");
    if (cond_rows > 65535LL * 16) return fail(IDOL_ERR_INVALID, "oct_logits: more than 1,048,560 condition rows");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 ||
        workspace_bytes < idol_b200_oct_decoder_workspace_bytes(d, rows, cond_rows))
        return fail(IDOL_ERR_INVALID, "oct_logits: workspace smaller than idol_b200_oct_decoder_workspace_bytes or "
                                      "not 256-byte aligned");
    IDOL_CUDA(cudaSetDevice(d->device));
    const OctWorkspace w = oct_layout(d, rows, cond_rows, static_cast<uint8_t*>(workspace));
    return oct_logits(d, x, rows, resolution, cond, cond_rows, logits, w, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------------------------------------ the host sampler
int idol_b200_oct_sampler_create(int num_points, int level, uint64_t seed, idol_oct_sampler** sampler) {
    if (!sampler) return fail(IDOL_ERR_INVALID, "oct_sampler_create: sampler is NULL");
    *sampler = nullptr;
    if (num_points < 1 || level < 1 || level > 20)
        return fail(IDOL_ERR_INVALID, "oct_sampler_create: num_points >= 1 and 1 <= level <= 20 expected");
    auto* s = new idol_oct_sampler();
    s->rng.seed(seed);
    s->counts = {num_points};
    s->levels = level;
    s->num_points = num_points;
    *sampler = s;
    return IDOL_OK;
}

int idol_b200_oct_sampler_free(idol_oct_sampler* sampler) {
    delete sampler;
    return IDOL_OK;
}

int idol_b200_oct_sampler_cells(const idol_oct_sampler* s, int64_t* parents, float* resolution) {
    if (!s || !parents) return fail(IDOL_ERR_INVALID, "oct_sampler_cells: NULL");
    *parents = s->level < s->levels ? (int64_t)s->counts.size() : 0;
    if (resolution) *resolution = (float)(1u << (s->level + 1));
    return IDOL_OK;
}

int idol_b200_oct_sampler_centres(const idol_oct_sampler* s, float* centres) {
    if (!s || !centres) return fail(IDOL_ERR_INVALID, "oct_sampler_centres: NULL");
    if (s->level >= s->levels) return fail(IDOL_ERR_INVALID, "oct_sampler_centres: every level is resampled");
    const float res_p = (float)(1u << s->level);
    for (size_t i = 0; i < s->coords.size(); ++i) centres[i] = ((float)s->coords[i] + 0.5f) / res_p;
    return IDOL_OK;
}

int idol_b200_oct_sampler_step(idol_oct_sampler* s, const float* logits) {
    if (!s || !logits) return fail(IDOL_ERR_INVALID, "oct_sampler_step: NULL");
    if (s->level >= s->levels) return fail(IDOL_ERR_INVALID, "oct_sampler_step: every level is resampled");
    const int parents = (int)s->counts.size();
    std::vector<uint32_t> next_coords;
    std::vector<int64_t> next_counts;
    for (int p = 0; p < parents; ++p) {
        // This cell's points are shared out among its eight child cells: child probabilities from the logits (max
        // subtracted, exponentiated, normalised), then one uniform draw places an evenly spaced comb of the points
        // on the cumulative distribution.
        float e[8];
        float mx = logits[(size_t)p * 8];
        for (int c = 1; c < 8; ++c) mx = std::max(mx, logits[(size_t)p * 8 + c]);
        float total = 0.0f;
        for (int c = 0; c < 8; ++c) total += (e[c] = std::exp(logits[(size_t)p * 8 + c] - mx));
        float cdf[8], acc = 0.0f;
        for (int c = 0; c < 8; ++c) cdf[c] = std::min(acc += e[c] / total, 1.0f - 1e-7f);
        const int64_t n = s->counts[p];
        int64_t got[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const float u0 = s->uniform(s->rng) / (float)n;
        for (int64_t k = 0; k < n; ++k) {
            const float u = std::min(u0 + (float)k / (float)n, 1.0f - 1e-7f);
            got[std::min<int>(7, (int)(std::lower_bound(cdf, cdf + 8, u) - cdf))]++;
        }
        for (int c = 0; c < 8; ++c)
            if (got[c] > 0) {
                next_coords.push_back(s->coords[(size_t)p * 3 + 0] * 2 + (c & 1));
                next_coords.push_back(s->coords[(size_t)p * 3 + 1] * 2 + ((c >> 1) & 1));
                next_coords.push_back(s->coords[(size_t)p * 3 + 2] * 2 + ((c >> 2) & 1));
                next_counts.push_back(got[c]);
            }
    }
    s->coords = std::move(next_coords);
    s->counts = std::move(next_counts);
    ++s->level;
    return IDOL_OK;
}

int idol_b200_oct_sampler_points(idol_oct_sampler* s, float* points) {
    if (!s || !points) return fail(IDOL_ERR_INVALID, "oct_sampler_points: NULL");
    if (s->level < s->levels) return fail(IDOL_ERR_INVALID, "oct_sampler_points: levels remain to be resampled");
    const float cells = (float)(1u << s->levels);
    size_t o = 0;
    for (size_t cell = 0; cell < s->counts.size(); ++cell)
        for (int64_t k = 0; k < s->counts[cell]; ++k)
            for (int c = 0; c < 3; ++c) points[o++] = ((float)s->coords[cell * 3 + c] + s->uniform(s->rng)) / cells;
    return IDOL_OK;
}

int idol_b200_oct_sample_anchors(const idol_oct_decoder* d, const float* cond, int64_t cond_rows, int num_points,
                                 int level, uint64_t seed, float* points, void* workspace, int64_t workspace_bytes,
                                 void* stream) {
    if (!d || !points || (!d->blocks.empty() && !cond)) return fail(IDOL_ERR_INVALID, "oct_sample_anchors: NULL");
    if (cond_rows < 1 || cond_rows > 65535LL * 16)
        return fail(IDOL_ERR_INVALID, "oct_sample_anchors: cond_rows must be 1..1,048,560");
    if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 ||
        workspace_bytes < idol_b200_oct_decoder_workspace_bytes(d, num_points, cond_rows))
        return fail(IDOL_ERR_INVALID, "oct_sample_anchors: workspace smaller than "
                                      "idol_b200_oct_decoder_workspace_bytes(decoder, num_points, cond_rows) or not "
                                      "256-byte aligned");
    IDOL_CUDA(cudaSetDevice(d->device));
    idol_oct_sampler* s = nullptr;
    int rc = idol_b200_oct_sampler_create(num_points, level, seed, &s);
    if (rc != IDOL_OK) return rc;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::vector<float> centres, logits;
    for (int l = 0; l < level && rc == IDOL_OK; ++l) {
        int64_t parents = 0;
        float res = 0.0f;
        idol_b200_oct_sampler_cells(s, &parents, &res);
        centres.resize((size_t)parents * 3);
        logits.resize((size_t)parents * 8);
        idol_b200_oct_sampler_centres(s, centres.data());
        // The cells of one level are at most num_points, the size the workspace was checked for.
        const OctWorkspace w = oct_layout(d, parents, cond_rows, static_cast<uint8_t*>(workspace));
        cudaError_t e = cudaMemcpyAsync(w.centres, centres.data(), centres.size() * sizeof(float),
                                        cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) {
            rc = idol::cuda_fail(e, "cudaMemcpyAsync (cell centres)");
            break;
        }
        rc = oct_logits(d, w.centres, parents, res, cond, cond_rows, w.logits, w, st);
        if (rc != IDOL_OK) break;
        e = cudaMemcpyAsync(logits.data(), w.logits, logits.size() * sizeof(float), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) {
            rc = idol::cuda_fail(e, "cudaMemcpyAsync (cell logits)");
            break;
        }
        rc = idol_b200_oct_sampler_step(s, logits.data());
    }
    if (rc == IDOL_OK) rc = idol_b200_oct_sampler_points(s, points);
    idol_b200_oct_sampler_free(s);
    return rc;
}

}  // extern "C"
