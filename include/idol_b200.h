/*
 * idol_b200.h - C ABI of the B200 (sm_100a) Q8_0 linear hot path.
 *
 * Plain pointers and sizes only. Every entry point returns IDOL_OK (0) or an IDOL_ERR_* status and never throws or
 * aborts; idol_b200_last_error() gives the message for the calling thread. Device entry points take device pointers
 * and a cudaStream_t passed as void* (NULL = the legacy default stream) and are asynchronous with respect to the host,
 * like the kernels they launch. Host entry points (the *_host names) take host pointers and return when the result is
 * in host memory.
 *
 * Each declaration names the reference interface it replaces (file:line inside TimeLordRaps/idol.cpp).
 */
#ifndef IDOL_B200_H
#define IDOL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define IDOL_OK 0
#define IDOL_ERR_INVALID 1     /* an argument the format or the kernel cannot take (the reference's std::invalid_argument) */
#define IDOL_ERR_CUDA 2        /* a CUDA runtime or driver call failed */
#define IDOL_ERR_UNSUPPORTED 3 /* a dtype or option this build does not implement */
#define IDOL_ERR_DEVICE 4      /* a kernel reported a bounded wait that ran out (see idol_b200_device_status) */

/* Element types. */
#define IDOL_F32 0
#define IDOL_F16 1
#define IDOL_BF16 2

/* Epilogue activations. */
#define IDOL_ACT_NONE 0
#define IDOL_ACT_GELU_ERF 1  /* exact GELU, 0.5 x (1 + erf(x / sqrt 2)): src/kernels.cpp:212-241 finish_tile */
#define IDOL_ACT_GELU_TANH 2 /* tanh GELU: src/decoders.cpp:55-71 gelu_tanh */
#define IDOL_ACT_SILU 3      /* x sigmoid(x): src/decoders.cpp:88 silu */

/* Epilogue flags. */
#define IDOL_EPI_BIAS_AFTER_ROUND 0x1 /* round the product to the output type before adding the bias, as
                                          tools/idol_triton.py:84-89 does; default adds it in fp32 like finish_tile */
#define IDOL_GEMM_WHOLE_K 0x2         /* never split K across CTAs: each output is summed in the order the unsplit
                                          full-width GEMM uses, so a column window (one rank's slice of a
                                          column-parallel linear) equals those columns of the whole product bit for
                                          bit whatever its width */

/* Message of the last failed call on this thread ("" if none). */
const char* idol_b200_last_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
int idol_b200_version(void);

/* Reads and clears the sticky device error word of `device` (bit 0: a kernel's bounded wait ran out). */
int idol_b200_device_status(int device, unsigned int* flags);

/* ------------------------------------------------------------------------------------------------ Q8_0 formats */

/* Bytes of GGUF Q8_0 data for an out x in matrix: out * in / 32 * 34 (tools/idol_triton.py:104). */
int64_t idol_b200_q8_bytes(int out, int in);
/* Bytes of the tiled device layout: chunks of 128 rows x 64 k, each 8192 code bytes then their 512 bytes of fp16
 * scales, ordered by (row tile, k stage); rows past `out` and blocks past in/32 are zero. */
int64_t idol_b200_q8_tiled_bytes(int out, int in);

/* fp32 weights [rows, cols] (device) -> Q8_0 blocks (device), byte-equal to gguf-py 0.19.0 gguf.quantize(W, Q8_0)
 * (called by tools/export_full_gguf.py:335). cols must be a multiple of 32. */
int idol_b200_q8_quantize(const float* w, int64_t rows, int64_t cols, void* q8, void* stream);

/* Q8_0 blocks -> tiled layout (device to device), and the exact inverse. Replaces the GGUF->native conversion
 * tools/gguf_to_decoder.py:16-40 + tools/idolq.py:137-166 (pack_blob) with a layout one GEMM pipeline stage moves with
 * a single bulk copy. tiles: idol_b200_q8_tiled_bytes(out, in) bytes, 16-byte aligned. */
int idol_b200_q8_repack(const void* q8, int out, int in, void* tiles, void* stream);
int idol_b200_q8_unpack(const void* tiles, int out, int in, void* q8, void* stream);

/* GGUF Q4_0 (kind 4): bytes for an out x in matrix, out * in / 32 * 18 (tools/idol_triton.py:103-104), and the device
 * conversion into the same tiled layout. A Q4_0 block (fp16 d, 16 bytes of nibbles: low nibbles elements 0-15, high
 * nibbles 16-31) is worth d * (nibble - 8) (tools/idol_triton.py:48-61), i.e. exactly a Q8_0 block with codes in
 * [-8, 7], so every entry point taking a tiled matrix (q8_view, q8_gemm, q8_dequantize) serves Q4_0 unchanged.
 * tiles: idol_b200_q8_tiled_bytes(out, in) bytes, 16-byte aligned; q4_0 2-byte aligned. */
int64_t idol_b200_q4_0_bytes(int out, int in);
int idol_b200_q4_0_repack(const void* q4_0, int out, int in, void* tiles, void* stream);

/* GGUF Q4_K (fused_linear kind 44, tools/idol_triton.py:64-82, 103-104; tools/idol_packed.py:41-54 dequantize): 144
 * bytes per 256 weights of a row (fp16 d, fp16 dmin, 12 bytes of 6-bit sub-block scales and mins, 128 bytes of
 * 4-bit codes), weight = d sc code - dmin m. `in` must be a positive multiple of 256. q4_k_repack converts it into
 * the Q4_K tiled layout (q4_k_tiled_bytes bytes; both pointers 16-byte aligned), which keeps fp32 A = d sc and
 * B = dmin m per 32-deep sub-block so that the kernels form the reference's fp32 weight A code - B exactly.
 * idol_b200_q4_k_view (below) wraps such tiles in a matrix handle for idol_b200_q8_gemm and the block / MLP
 * builders; q4_k_dequantize writes the dense [out, in] weights (f32 exact; bf16 / f16 rounded from the f32 value). */
int64_t idol_b200_q4_k_bytes(int out, int in);
int64_t idol_b200_q4_k_tiled_bytes(int out, int in);
int idol_b200_q4_k_repack(const void* q4_k, int out, int in, void* tiles, void* stream);
int idol_b200_q4_k_dequantize(const void* tiles, int out, int in, void* w, int w_dtype, void* stream);

/* Tiled layout -> dense out x in weights d * q (w_dtype IDOL_F32 exact; IDOL_BF16 / IDOL_F16 rounded from the fp32
 * product). Replaces src/kernels.cpp:535-550 dequantize_linear and tools/idol_packed.py:25-31 dequantize. */
int idol_b200_q8_dequantize(const void* tiles, int out, int in, void* w, int w_dtype, void* stream);

/* ------------------------------------------------------------------------------------------- resident matrices */

/* A Q8_0 weight matrix (plus optional fp32 bias) resident in one GPU's memory in the tiled layout. */
typedef struct idol_q8_matrix idol_q8_matrix;

/* Uploads host Q8_0 bytes (nbytes == idol_b200_q8_bytes(out, in)) and an optional host fp32 bias[out] to `device`,
 * once. Replaces src/kernels.cpp:516-533 quantized_linear and the qtensor load of src/weights.cpp:67-80. Returns when
 * the matrix is ready. */
int idol_b200_q8_upload(const void* q8_host, int64_t nbytes, int out, int in, const float* bias_host, int device,
                        idol_q8_matrix** matrix);

/* The same from Q8_0 bytes and an optional fp32 bias already on `device` (PackedLinear.packed,
 * tools/idol_packed.py:21). Ordered on `stream`. */
int idol_b200_q8_import(const void* q8_dev, int64_t nbytes, int out, int in, const float* bias_dev, int device,
                        void* stream, idol_q8_matrix** matrix);

/* A matrix handle over a tiled buffer (and an optional fp32 bias) that the caller already holds on `device`, e.g.
 * tensors of a PyTorch module; nothing is allocated on the device and idol_b200_q8_free releases only the handle. */
int idol_b200_q8_view(const void* tiles, const float* bias_dev, int out, int in, int device, idol_q8_matrix** matrix);
/* The same over Q4_K tiles (idol_b200_q4_k_repack); idol_b200_q8_export refuses such a handle. */
int idol_b200_q4_k_view(const void* tiles, const float* bias_dev, int out, int in, int device,
                        idol_q8_matrix** matrix);

int idol_b200_q8_free(idol_q8_matrix* matrix);

/* Shape and device footprint. */
int idol_b200_q8_info(const idol_q8_matrix* matrix, int* out, int* in, int* device, int64_t* device_bytes);

/* Writes the matrix back as Q8_0 blocks into q8_dev (device), the bit-exact inverse of the upload. */
int idol_b200_q8_export(const idol_q8_matrix* matrix, void* q8_dev, int64_t nbytes, void* stream);

/* ---------------------------------------------------------------------------------------------------- the GEMM */

/* y[m, 0:n] = x[m, in] . W[n_offset : n_offset + n]^T + bias (+ residual) (-> act), on the matrix's device.
 * Replaces src/kernels.cpp:75-76 gemm_packed (window, residual that may alias y, activation after the residual) and
 * tools/idol_triton.py:94-126 fused_linear.
 *   x        : device, x_dtype IDOL_BF16 or IDOL_F16, rows ldx elements apart (ldx >= in, ldx % 8 == 0, 16-byte base).
 *   residual : device, y_dtype, rows ldr apart, or NULL. May alias y.
 *   y        : device, y_dtype IDOL_BF16, IDOL_F16 or IDOL_F32, rows ldy apart.
 *   flags    : IDOL_EPI_* bits.
 * m == 0 or n == 0 is a no-op.
 * From m = 1024 tokens (when the output tiles fill the GPU's SM pairs) the call dequantises the window's weights into
 * a scratch buffer and runs a dense GEMM on it: the buffer belongs to the library, one per device and stream, 2 bytes
 * per weight of the largest matrix used on that stream, allocated on first need (never while the stream is being
 * captured into a CUDA graph: such a call takes the fused kernel) and kept until the process exits. Calls on one
 * stream share it in stream order. The environment variable IDOL_B200_GEMM_DENSE=0 turns this path off, so that the
 * library allocates nothing of its own. */
int idol_b200_q8_gemm(const idol_q8_matrix* matrix, const void* x, int x_dtype, int64_t m, int64_t ldx, int n_offset,
                      int n, const void* residual, int64_t ldr, int act, int flags, void* y, int y_dtype, int64_t ldy,
                      void* stream);

/* A projection followed by the per-head norm of its first head_cols output columns, as the decoders run them
 * (src/decoders.cpp:234-237 and :298-300: gemm_packed, then rms_heads of q and of k): y[m, 0:n] = bf16(x . W^T + bias),
 * then columns [0, head_split) normalised per 64-wide head with gamma_a and [head_split, head_cols) with gamma_b
 * (x * 8 / max(|x|, 1e-12) * gamma on the stored bf16 row). The norm runs in the GEMM's epilogue when the GEMM leaves
 * through its staging tile and head_cols is a multiple of 128, else as a launch right after it; the result is the
 * same bits either way. y: bf16, rows ldy apart. gamma_b may be NULL when head_split == head_cols. */
int idol_b200_q8_gemm_heads(const idol_q8_matrix* matrix, const void* x, int64_t m, int64_t ldx, void* y, int64_t ldy,
                            int head_cols, int head_split, const float* gamma_a, const float* gamma_b, void* stream);

/* The same linear on integer activations: the reference's second CPU kernel (src/kernels.cpp:368-479,
 * quantize_activations + vnni_task + gemm_quant_int8, chosen there by set_quant_kernel(1)), bit for bit on Q8_0
 * matrices. x (IDOL_F32, IDOL_BF16 or IDOL_F16, rows ldx apart) is quantized per (row, 32-deep group) to int8 with
 * scale amax / 127 into the workspace; each output sums the groups' integer dot products scaled as the reference
 * does, then bias, residual (y_dtype, window layout, may alias y) and act. Output IDOL_F32 (the reference's), IDOL_BF16
 * or IDOL_F16. workspace: device, 256-byte aligned, >= idol_b200_q8_gemm_int8act_workspace_bytes(m, in). Q4_K
 * matrices are refused (IDOL_ERR_UNSUPPORTED). */
int64_t idol_b200_q8_gemm_int8act_workspace_bytes(int64_t m, int in);
int idol_b200_q8_gemm_int8act(const idol_q8_matrix* matrix, const void* x, int x_dtype, int64_t m, int64_t ldx,
                              int n_offset, int n, const void* residual, int64_t ldr, int act, void* y, int y_dtype,
                              int64_t ldy, void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------ norms and attention */

/* y = LayerNorm(x) per row of `dim` values (eps as given), then optionally * gamma + beta, then optionally
 * * (1 + scale) + shift: src/decoders.cpp:23-42 norm_rows (gamma/beta and shift/scale come in pairs; fp32 vectors of
 * dim on the device, or NULL). x/y dtypes: bf16->bf16, f32->bf16, f32->f32, f16->f16, bf16->f32. y may alias x.
 * dim in {256, 512, 768, 1024, 1536, 2048}; rows 16-byte aligned. */
int idol_b200_norm_rows(const void* x, int x_dtype, int64_t rows, int dim, int64_t ldx, float eps, const float* gamma,
                        const float* beta, const float* shift, const float* scale, void* y, int y_dtype, int64_t ldy,
                        void* stream);

/* In place: each of `heads` groups of head_dim columns of each row (rows ld apart) becomes
 * x * sqrt(hd) / max(|x|, 1e-12) * gamma[h * hd + d]: src/decoders.cpp:74-86 rms_heads. head_dim 64. */
int idol_b200_rms_heads(void* x, int dtype, int64_t rows, int64_t ld, int heads, int head_dim, const float* gamma,
                        void* stream);

/* Multi-head attention, bf16 q/k/v: for each of `batch` independent sequences (q rows b*lq.., k/v rows b*lk..), per
 * head h out[:, h*hd:(h+1)*hd] = softmax(q_h k_h^T / sqrt(hd)) v_h. Replaces src/kernels.cpp:737-746 attention
 * (q lq rows ldq apart; k, v lk rows ldkv apart, e.g. k = kv and v = kv + dim as src/decoders.cpp:239 passes them; out
 * rows ldo apart). out_dtype IDOL_BF16 (what the next Q8_0 GEMM consumes) or IDOL_F32 (the reference's own output
 * type). head_dim 64; pointers 16-byte aligned; strides multiples of 8 elements. */
int idol_b200_attention(const void* q, int64_t lq, int64_t ldq, const void* k, const void* v, int64_t lk, int64_t ldkv,
                        int heads, int head_dim, void* out, int out_dtype, int64_t ldo, int batch, void* stream);

/* ------------------------------------------------------------------------------------------------ compositions */

/* A denoiser-style transformer block over resident matrices (scope row A14: src/decoders.cpp:296-313 without the
 * cross-attention): LN -> QKV -> rms q,k -> self-attention -> out + residual -> LN -> ff1 (GELU tanh) -> ff2 +
 * residual. qkv is 3D x D, out D x D, ff1 H x D, ff2 D x H, D = heads * 64; q_gamma/k_gamma are fp32 [D] on the
 * device. The handle keeps pointers only; the matrices must outlive it. */
typedef struct idol_block idol_block;
int idol_b200_block_create(const idol_q8_matrix* qkv, const idol_q8_matrix* out, const idol_q8_matrix* ff1,
                           const idol_q8_matrix* ff2, const float* q_gamma, const float* k_gamma, int heads,
                           float eps, idol_block** block);
int idol_b200_block_free(idol_block* block);
/* Device workspace the forward needs for `rows` = tokens * images rows. */
int64_t idol_b200_block_workspace_bytes(const idol_block* block, int64_t rows);
/* x: [images * tokens, D] residual stream (IDOL_F32 or IDOL_BF16), updated in place; each image attends within its
 * own `tokens` rows. workspace: device, 256-byte aligned, >= idol_b200_block_workspace_bytes. */
int idol_b200_block_forward(const idol_block* block, void* x, int x_dtype, int64_t tokens, int images, void* workspace,
                            int64_t workspace_bytes, void* stream);

/* The Gaussian decoder's block (src/decoders.cpp:296-313, next-row (f)1): the block above with a cross-attention
 * sublayer between the self-attention and the MLP: h = LN(x, eps) * norm2_gamma + norm2_beta; q = h W_q^T (cross_q,
 * D x D) then rms_heads with cross_q_gamma; kv = cond W_kv^T + kv_bias with W_kv dense fp32 [2D, cond_dim] on the
 * device (the reference keeps this 16-deep `to_kv` in fp32), then rms_heads of its k half with cross_k_gamma; each
 * image's rows attend over that image's cond_rows latent rows (src/decoders.cpp:232-240); x += a W_o^T + b
 * (cross_out, D x D). cond_dim 1..64 (the real decoder's is 16); all vectors fp32 on the device. */
typedef struct idol_gs_block idol_gs_block;
int idol_b200_gs_block_create(const idol_q8_matrix* qkv, const idol_q8_matrix* out, const idol_q8_matrix* cross_q,
                              const idol_q8_matrix* cross_out, const idol_q8_matrix* ff1, const idol_q8_matrix* ff2,
                              const float* q_gamma, const float* k_gamma, const float* cross_q_gamma,
                              const float* cross_k_gamma, const float* norm2_gamma, const float* norm2_beta,
                              const float* kv_weight, const float* kv_bias, int cond_dim, int heads, float eps,
                              idol_gs_block** block);
int idol_b200_gs_block_free(idol_gs_block* block);
/* Device workspace for `rows` = tokens * images rows and cond_rows_total = cond_rows * images condition rows. */
int64_t idol_b200_gs_block_workspace_bytes(const idol_gs_block* block, int64_t rows, int64_t cond_rows_total);
/* x: [images * tokens, D] residual stream (IDOL_F32 or IDOL_BF16), in place; cond: fp32 [images * cond_rows,
 * cond_dim] on the device, image i's latent rows at i * cond_rows. */
int idol_b200_gs_block_forward(const idol_gs_block* block, void* x, int x_dtype, int64_t tokens, int images,
                               const float* cond, int64_t cond_rows, void* workspace, int64_t workspace_bytes,
                               void* stream);

/* The Gaussian decoder (Decoders::gaussian_features and to_gaussians, src/decoders.cpp:284-316, 393-433) over
 * resident weights, for one image: x = in_proj(points) + pos_embed(points) (in_w dense fp32 [D, 3], in_b [D] or NULL;
 * pos_embed with the export's n_freqs fp32 frequencies, 6 n_freqs <= D) -> input_layer (D x D) -> the blocks ->
 * LN (eps 1e-5) -> out_proj (per_anchor * 15 x D) = features. rep: 9 host floats perturbe, kernel, scaling_bias,
 * opacity_bias, lr_xyz, lr_dc, lr_opacity, lr_scaling, lr_rotation (src/weights.hpp:25-28); perturbation fp32
 * [per_anchor * 3] on the device. The handle keeps pointers only. */
typedef struct idol_gs_decoder idol_gs_decoder;
int idol_b200_gs_decoder_create(const idol_gs_block* const* blocks, int nblocks, const float* in_w, const float* in_b,
                                const idol_q8_matrix* input_layer, const idol_q8_matrix* out_proj, const float* freqs,
                                int n_freqs, int per_anchor, const float* perturbation, float base_offset_scale,
                                const float* rep, idol_gs_decoder** decoder);
int idol_b200_gs_decoder_free(idol_gs_decoder* decoder);
int64_t idol_b200_gs_decoder_workspace_bytes(const idol_gs_decoder* decoder, int64_t rows, int64_t cond_rows);
/* points fp32 [rows, 3] (anchors in [0, 1]^3), cond fp32 [cond_rows, cond_dim] -> features fp32
 * [rows, 15 per_anchor]. */
int idol_b200_gs_decoder_features(const idol_gs_decoder* decoder, const float* points, int64_t rows, const float* cond,
                                  int64_t cond_rows, float* features, void* workspace, int64_t workspace_bytes,
                                  void* stream);
/* Activated Gaussians: xyz, f_dc, scale fp32 [rows * per_anchor, 3], rotation [.., 4], opacity [..]. */
int idol_b200_gs_to_gaussians(const idol_gs_decoder* decoder, const float* anchors, int64_t rows,
                              const float* features, float* xyz, float* f_dc, float* scale, float* rotation,
                              float* opacity, void* stream);

/* The octree decoder (Decoders::octree_logits and sample_anchors, src/decoders.cpp:242-282, 335-391) over resident
 * weights. A block is the cross-attention half and the MLP half of src/decoders.cpp:268-279, each added to the
 * residual stream through its adaLN gate: to_q / to_out D x D, ff1 H x D, ff2 D x H, the dense fp32 to_kv [2D,
 * cond_dim] (+ bias [2D] or NULL), q/k rms gammas [D]. The decoder: in_proj dense fp32 [D, 3] (+ bias), input_layer
 * D x D, the level embedder l1 D x 256 and l2 D x D, the adaLN modulation ada 6D x D, out_proj 8 x D, pos_embed
 * frequencies [n_freqs] (6 n_freqs <= D) and the 128 level frequencies, all on the device; eps is the blocks' LN
 * epsilon (1e-6 in the reference). Handles keep pointers only. */
typedef struct idol_oct_block idol_oct_block;
typedef struct idol_oct_decoder idol_oct_decoder;
int idol_b200_oct_block_create(const idol_q8_matrix* cross_q, const idol_q8_matrix* cross_out,
                               const idol_q8_matrix* ff1, const idol_q8_matrix* ff2, const float* cross_q_gamma,
                               const float* cross_k_gamma, const float* kv_weight, const float* kv_bias, int cond_dim,
                               int heads, idol_oct_block** block);
int idol_b200_oct_block_free(idol_oct_block* block);
int idol_b200_oct_decoder_create(const idol_oct_block* const* blocks, int nblocks, const float* in_w, const float* in_b,
                                 const idol_q8_matrix* input_layer, const idol_q8_matrix* l1,
                                 const idol_q8_matrix* l2, const idol_q8_matrix* ada, const idol_q8_matrix* out_proj,
                                 const float* freqs, int n_freqs, const float* level_freqs, int heads, float eps,
                                 idol_oct_decoder** decoder);
int idol_b200_oct_decoder_free(idol_oct_decoder* decoder);
/* Device workspace for a logits call over `rows` cells (for sample_anchors: rows = num_points). */
int64_t idol_b200_oct_decoder_workspace_bytes(const idol_oct_decoder* decoder, int64_t rows, int64_t cond_rows);
/* x: cell centres fp32 [rows, 3] on the device; resolution: the cells' octree resolution 2^level; cond fp32
 * [cond_rows, cond_dim]; logits fp32 [rows, 8] (how a cell's points split among its children). */
int idol_b200_oct_logits(const idol_oct_decoder* decoder, const float* x, int64_t rows, float resolution,
                         const float* cond, int64_t cond_rows, float* logits, void* workspace, int64_t workspace_bytes,
                         void* stream);
/* Decoders::sample_anchors: descends from the root to `level` (1..20), the logits of each level's occupied cells
 * on the GPU, the resampling on the host with the reference's generator and arithmetic (mt19937_64 seeded with
 * `seed`); points: host fp32 [num_points, 3]. Synchronises `stream` once per level. */
int idol_b200_oct_sample_anchors(const idol_oct_decoder* decoder, const float* cond, int64_t cond_rows,
                                 int num_points, int level, uint64_t seed, float* points, void* workspace,
                                 int64_t workspace_bytes, void* stream);
/* The host half of sample_anchors on its own, for callers that compute the logits themselves: create, then per level
 * cells (the number of occupied cells and the resolution to evaluate them at; 0 cells once every level is done),
 * centres (host fp32 [cells, 3]) and step (host fp32 logits [cells, 8]); finally points (host fp32 [num_points, 3]). */
typedef struct idol_oct_sampler idol_oct_sampler;
int idol_b200_oct_sampler_create(int num_points, int level, uint64_t seed, idol_oct_sampler** sampler);
int idol_b200_oct_sampler_free(idol_oct_sampler* sampler);
int idol_b200_oct_sampler_cells(const idol_oct_sampler* sampler, int64_t* cells, float* resolution);
int idol_b200_oct_sampler_centres(const idol_oct_sampler* sampler, float* centres);
int idol_b200_oct_sampler_step(idol_oct_sampler* sampler, const float* logits);
int idol_b200_oct_sampler_points(idol_oct_sampler* sampler, float* points);

/* The Gaussian decoder MLP of config 4 (scope row A15): x [points, in] bf16 -> l0 (SiLU) -> l1 (SiLU) -> l2 (14
 * outputs) -> heads: pos identity, scale exp, rotation r = f * 0.1 + (1, 0, 0, 0) divided by max(|r|, 1e-12)
 * (src/decoders.cpp:422-428 with the default lr_rotation), colour and opacity sigmoid (:429). out: fp32 [points, 14]; raw_out: fp32 [points, 14] pre-activation values, or NULL. */
typedef struct idol_gaussian_mlp idol_gaussian_mlp;
int idol_b200_gaussian_mlp_create(const idol_q8_matrix* l0, const idol_q8_matrix* l1, const idol_q8_matrix* l2,
                                  idol_gaussian_mlp** mlp);
int idol_b200_gaussian_mlp_free(idol_gaussian_mlp* mlp);
int64_t idol_b200_gaussian_mlp_workspace_bytes(const idol_gaussian_mlp* mlp, int64_t points);
int idol_b200_gaussian_mlp_forward(const idol_gaussian_mlp* mlp, const void* x, int64_t points, int64_t ldx,
                                   void* workspace, int64_t workspace_bytes, float* raw_out, float* out, void* stream);
/* The same Gaussian MLP forward for callers that cannot allocate device memory at all, not even once for a
 * workspace: a process whose device memory another allocator (a framework's caching pool, an inference server's
 * arena) has already reserved in full, so a cudaMalloc of its own would fail or fragment that pool. It is a regular
 * host-side call - it selects the device and launches kernels - so it must not be made from a stream callback
 * (cudaLaunchHostFunc), where no CUDA call is allowed. It allocates nothing:
 * its scratch is a fixed 8 MiB array in the library's device code, reserved on every GPU that loads the library and
 * held until exit; the caller still passes x, raw_out (or NULL) and out. A batch whose scratch would not fit
 * (idol_b200_gaussian_mlp_workspace_bytes(mlp, points) > 8 MiB: about 3,980 points for 128 -> 512 -> 512 -> 14) is
 * rejected with IDOL_ERR_INVALID. The first call on a device looks the array's address up on that device; make that
 * first call before any stream capture. Every call on a device shares the one array, which keeps the last call's
 * contents (nothing in it needs to start at zero): calls that overlap on the GPU, on different streams or different
 * host threads, race on it and must be ordered by the caller. With matrices made by idol_b200_q8_view over memory
 * the caller already holds, the whole path runs without a device allocation. No counterpart in the reference. */
int idol_b200_gaussian_mlp_forward_static(const idol_gaussian_mlp* mlp, const void* x, int64_t points, int64_t ldx,
                                          float* raw_out, float* out, void* stream);
/* The output heads alone: raw [points, >= 14] (rows ld apart, raw_dtype) -> out fp32 [points, 14]. */
int idol_b200_gaussian_heads(const void* raw, int raw_dtype, int64_t points, int64_t ld, float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IDOL_B200_H */
