/*
 * q8_oracle.c - CPU restatement of idol.cpp's Q8_0 linear hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker, never the product: only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs may load it. The CUDA library never links it and never falls back to it.
 *
 * Parity pins (see tests/test_oracle.py):
 *   - orc_q8_quantize is byte-equal to gguf-py 0.19.0 `gguf.quantize(W, Q8_0)` (golden fixtures in tests/golden/).
 *   - orc_gemm_q8 is bit-equal to the reference's own float kernel (src/kernels.cpp gemm_quant, compiled from the
 *     reference sources into oracle/_ref by oracle/Makefile) on the same inputs.
 *   - the norms, activations and attention agree with the reference's compiled functions within float rounding.
 *
 * Build with -ffp-contract=off: every fused multiply-add below is an explicit fmaf(), as in the reference's
 * intrinsics, and no other product may be fused.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------------------------------
 * IEEE binary16 conversions (round to nearest even), written from the format definition.
 * ---------------------------------------------------------------------------------------------------------------- */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to infinity */
    if (ax < 0x38800000u) {                                   /* below 2^-14: a subnormal half or zero */
        if (ax < 0x33000000u) return (uint16_t)sign;          /* below 2^-25: rounds to zero */
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const int shift = 126 - (int)e; /* units of 2^-24 */
        uint32_t k = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (k & 1u))) ++k;
        return (uint16_t)(sign | k);
    }
    const uint32_t e = (ax >> 23) - 127u + 15u;
    const uint32_t m = ax & 0x7fffffu;
    uint32_t r = (e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r; /* a carry into the exponent is the right answer */
    return (uint16_t)(sign | r);
}

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        float v = ldexpf((float)m, -24);
        memcpy(&x, &v, 4);
        x |= sign;
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e - 15u + 127u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* bf16 from fp32 with round to nearest even (NaN kept quiet). */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    const uint32_t lsb = (x >> 16) & 1u;
    x += 0x7fffu + lsb;
    return (uint16_t)(x >> 16);
}

float orc_bf16_to_f32(uint16_t b) {
    const uint32_t x = (uint32_t)b << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------------------------------------------------------------
 * Q8_0 blocks: 34 bytes per 32 consecutive weights of one row (fp16 scale d, then 32 int8 codes).
 * Encoder: gguf-py 0.19.0 Q8_0.quantize_blocks (third-party, called by tools/export_full_gguf.py:335): d = amax/127 in
 * fp32, id = 1/d in fp32 (0 when d == 0), q = round-half-away-from-zero(w * id), then d stored as fp16.
 * Decoder: w = fp16(d) * q (tools/idol_packed.py:28-31, tools/idol_triton.py:24-33).
 * ---------------------------------------------------------------------------------------------------------------- */
static float round_half_away(float v) {
    /* floor(|v|) + floor(2 * (|v| - floor(|v|))), with the sign of v; every step is exact in fp32. */
    const float a = fabsf(v);
    const float fl = floorf(a);
    const float r = fl + floorf(2.0f * (a - fl));
    return v < 0.0f ? -r : r;
}

void orc_q8_quantize(const float* w, int64_t rows, int64_t cols, uint8_t* out) {
    const int64_t nb = cols / 32;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            const float* x = w + r * cols + b * 32;
            uint8_t* blk = out + (r * nb + b) * 34;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) {
                const float a = fabsf(x[i]);
                if (a > amax) amax = a;
            }
            const float d = amax / 127.0f;
            const float id = d == 0.0f ? 0.0f : 1.0f / d;
            const uint16_t dh = orc_f32_to_f16(d);
            blk[0] = (uint8_t)(dh & 0xffu);
            blk[1] = (uint8_t)(dh >> 8);
            for (int i = 0; i < 32; ++i) {
                const float q = round_half_away(x[i] * id);
                blk[2 + i] = (uint8_t)(int8_t)(int)q;
            }
        }
}

void orc_q8_dequantize(const uint8_t* blocks, int64_t rows, int64_t cols, float* w) {
    const int64_t nb = cols / 32;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t* blk = blocks + (r * nb + b) * 34;
            const float d = orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int i = 0; i < 32; ++i) w[r * cols + b * 32 + i] = d * (float)(int8_t)blk[2 + i];
        }
}

/* ------------------------------------------------------------------------------------------------------------------
 * GGUF Q4_0 (kind 4): 18-byte blocks of fp16 d and 16 bytes; element i of a block is nibble (i % 16) of byte i % 16,
 * the low nibble for i < 16 and the high nibble after, worth d * (nibble - 8): restates tools/idol_triton.py:48-61
 * (the fused kernel's decoder) and tools/idol_packed.py:32-36 (the expansion path). orc_q4_0_to_q8 writes the same
 * weights as Q8_0 blocks (codes nibble - 8, same d), which is exact, so orc_gemm_q8 computes a Q4_0 linear too.
 * ---------------------------------------------------------------------------------------------------------------- */
static int orc_q4_0_code(const uint8_t* blk, int i) {
    const uint8_t byte = blk[2 + (i % 16)];
    return (int)(i < 16 ? (byte & 15) : (byte >> 4)) - 8;
}

void orc_q4_0_dequantize(const uint8_t* blocks, int64_t rows, int64_t cols, float* w) {
    const int64_t nb = cols / 32;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t* blk = blocks + (r * nb + b) * 18;
            const float d = orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int i = 0; i < 32; ++i) w[r * cols + b * 32 + i] = d * (float)orc_q4_0_code(blk, i);
        }
}

void orc_q4_0_to_q8(const uint8_t* q4, int64_t rows, int64_t cols, uint8_t* q8) {
    const int64_t nb = cols / 32;
    for (int64_t blk = 0; blk < rows * nb; ++blk) {
        const uint8_t* src = q4 + blk * 18;
        uint8_t* dst = q8 + blk * 34;
        dst[0] = src[0];
        dst[1] = src[1];
        for (int i = 0; i < 32; ++i) dst[2 + i] = (uint8_t)(int8_t)orc_q4_0_code(src, i);
    }
}

/* ------------------------------------------------------------------------------------------------------------------
 * GGUF Q4_K (kind 44): 144-byte super-blocks of 256 elements: fp16 d, fp16 dmin, 12 bytes of 6-bit scales and mins
 * for the eight 32-element sub-blocks (sub-block j < 4: scale = s[j] & 63, min = s[j + 4] & 63; j >= 4: scale =
 * (s[j + 4] & 15) | (s[j - 4] >> 6) << 4, min = (s[j + 4] >> 4) | (s[j] >> 6) << 4), then 128 bytes of codes
 * (sub-blocks 2g and 2g + 1 are the low and high nibbles of bytes 32 g .. 32 g + 31). Element = (d scale) code -
 * dmin min in fp32, each product formed first: restates tools/idol_packed.py:41-54 (the expansion path) and
 * tools/idol_triton.py:64-82 (the fused kernel's decoder), and gguf-py 0.19.0 Q4_K.dequantize_blocks.
 * ---------------------------------------------------------------------------------------------------------------- */
void orc_q4_k_dequantize(const uint8_t* blocks, int64_t rows, int64_t cols, float* w) {
    const int64_t nsb = cols / 256;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < nsb; ++b) {
            const uint8_t* sb = blocks + (r * nsb + b) * 144;
            const float d = orc_f16_to_f32((uint16_t)(sb[0] | (sb[1] << 8)));
            const float dmin = orc_f16_to_f32((uint16_t)(sb[2] | (sb[3] << 8)));
            const uint8_t* s = sb + 4;
            const uint8_t* qs = sb + 16;
            for (int j = 0; j < 8; ++j) {
                const int sc = j < 4 ? (s[j] & 63) : ((s[j + 4] & 15) | ((s[j - 4] >> 6) << 4));
                const int mn = j < 4 ? (s[j + 4] & 63) : ((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
                const float a = d * (float)sc, bm = dmin * (float)mn;
                for (int i = 0; i < 32; ++i) {
                    const int code = (qs[(j / 2) * 32 + i] >> (4 * (j % 2))) & 15;
                    const float prod = a * (float)code;
                    w[r * cols + b * 256 + j * 32 + i] = prod - bm;
                }
            }
        }
}

/* ------------------------------------------------------------------------------------------------------------------
 * Q8_0 -> idol panel blob, bits 8, group 32: restates tools/gguf_to_decoder.py:16-40 (code = q + 128, scale = fp16 d,
 * min = fp16(-128 d), rejected unless exact) and tools/idolq.py:137-166 (16 output columns per panel; per group a 64-byte
 * header of 16 fp16 scales then 16 fp16 minimums, then 32 rows of k x 16 columns of codes). Returns 0, or -1 when a
 * minimum is not exact in fp16 (the converter's ValueError), or -2 for a shape the format cannot hold.
 * ---------------------------------------------------------------------------------------------------------------- */
int64_t orc_panel_blob_bytes(int out, int in) { return (int64_t)((out + 15) / 16) * (in / 32) * 576; }

int orc_q8_to_panels(const uint8_t* q8, int out, int in, uint8_t* blob) {
    if (out < 1 || in < 32 || in % 32) return -2;
    const int panels = (out + 15) / 16, ng = in / 32;
    memset(blob, 0, (size_t)orc_panel_blob_bytes(out, in));
    for (int p = 0; p < panels; ++p)
        for (int g = 0; g < ng; ++g) {
            uint8_t* dst = blob + ((int64_t)p * ng + g) * 576;
            for (int c = 0; c < 16; ++c) {
                const int n = p * 16 + c;
                uint16_t sh = 0, mh = 0;
                if (n < out) {
                    const uint8_t* blk = q8 + ((int64_t)n * ng + g) * 34;
                    sh = (uint16_t)(blk[0] | (blk[1] << 8));
                    const float d = orc_f16_to_f32(sh);
                    if (!isfinite(d)) return -1;
                    const float mn = -128.0f * d;
                    mh = orc_f32_to_f16(mn);
                    if (orc_f16_to_f32(mh) != mn) return -1;
                    for (int k = 0; k < 32; ++k) dst[64 + k * 16 + c] = (uint8_t)((int)(int8_t)blk[2 + k] + 128);
                }
                memcpy(dst + 2 * c, &sh, 2);
                memcpy(dst + 32 + 2 * c, &mh, 2);
            }
        }
    return 0;
}

/* ------------------------------------------------------------------------------------------------------------------
 * Epilogue activations.
 *   ORC_ACT_GELU_ERF : finish_tile's GELU, 0.5 x (1 + erf(x / sqrt 2)) with erf per Abramowitz-Stegun 7.1.26
 *                      (src/kernels.cpp:829-840 gelu_scalar)
 *   ORC_ACT_GELU_TANH: the decoders' MLP GELU, 0.5 x (1 + tanh(0.79788456 (x + 0.044715 x^3))) (src/decoders.cpp:55-71)
 *   ORC_ACT_SILU     : x / (1 + exp(-x)) (src/decoders.cpp:88)
 * ---------------------------------------------------------------------------------------------------------------- */
enum { ORC_ACT_NONE = 0, ORC_ACT_GELU_ERF = 1, ORC_ACT_GELU_TANH = 2, ORC_ACT_SILU = 3 };

float orc_gelu_erf(float x) {
    const float z = x * 0.70710678118654752f;
    const float az = fabsf(z);
    const float t = 1.0f / (1.0f + 0.3275911f * az);
    const float p = t * ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f);
    const float erf_abs = 1.0f - p * expf(-az * az);
    return 0.5f * x * (1.0f + (z < 0.0f ? -erf_abs : erf_abs));
}

float orc_gelu_tanh(float v) {
    const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(u));
}

float orc_silu(float x) { return x / (1.0f + expf(-x)); }

static float apply_act(float v, int act) {
    switch (act) {
        case ORC_ACT_GELU_ERF: return orc_gelu_erf(v);
        case ORC_ACT_GELU_TANH: return orc_gelu_tanh(v);
        case ORC_ACT_SILU: return orc_silu(v);
        default: return v;
    }
}

/* ------------------------------------------------------------------------------------------------------------------
 * C[m x n] = A[m x K] . W[n_offset : n_offset + n]^T + bias (+ residual) (-> act), with W given as Q8_0 blocks.
 * Summation order of the reference float kernel (src/kernels.cpp:246-296 gemm_quant with microkernel_6x16 :79-121):
 * per output, the depth runs in chunks of 32; inside a chunk a single fused multiply-add chain from zero over k; the
 * chunk partials are added to the running tile in k order. Then bias, then residual, then the activation (finish_tile
 * :212-241). The weights the kernel multiplies are fma(q + 128, d, -128 d) = q * d exactly (both products are exact
 * in fp32), which is what this function uses.
 * residual has row stride n and may alias c.
 * ---------------------------------------------------------------------------------------------------------------- */
void orc_gemm_q8(const float* a, int m, const uint8_t* q8, const float* bias, int N, int K, int n_offset, int n,
                 const float* residual, int act, float* c) {
    const int nb = K / 32;
    float* wrow = (float*)malloc(sizeof(float) * (size_t)K);
    float* out = (float*)malloc(sizeof(float) * (size_t)m);
    for (int j = 0; j < n; ++j) {
        const int col = n_offset + j;
        if (col >= N) break;
        orc_q8_dequantize(q8 + (int64_t)col * nb * 34, 1, K, wrow);
        /* Eight rows at a time: independent chains for the CPU, the same per-output order as one row at a time. */
        int i = 0;
        for (; i + 8 <= m; i += 8) {
            float tile[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int k0 = 0; k0 < K; k0 += 32) {
                float part[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                for (int k = k0; k < k0 + 32; ++k)
                    for (int r = 0; r < 8; ++r) part[r] = fmaf(a[(int64_t)(i + r) * K + k], wrow[k], part[r]);
                for (int r = 0; r < 8; ++r) tile[r] = k0 == 0 ? part[r] : tile[r] + part[r];
            }
            for (int r = 0; r < 8; ++r) out[i + r] = tile[r];
        }
        for (; i < m; ++i) {
            const float* ar = a + (int64_t)i * K;
            float tile = 0.0f;
            for (int k0 = 0; k0 < K; k0 += 32) {
                float part = 0.0f;
                for (int k = k0; k < k0 + 32; ++k) part = fmaf(ar[k], wrow[k], part);
                tile = k0 == 0 ? part : tile + part;
            }
            out[i] = tile;
        }
        for (int i = 0; i < m; ++i) {
            float v = out[i] + (bias ? bias[col] : 0.0f);
            if (residual) v += residual[(int64_t)i * n + j];
            c[(int64_t)i * n + j] = apply_act(v, act);
        }
    }
    free(wrow);
    free(out);
}

/* ------------------------------------------------------------------------------------------------------------------
 * The same linear on integer activations: the reference's second CPU kernel (src/kernels.cpp:368-479,
 * quantize_activations + vnni_task + gemm_quant_int8, chosen there by set_quant_kernel(1)), for Q8_0-derived 8-bit
 * panels (stored code u = q + 128, minimum -128 d). Activations per (row, 32-group): amax = max |x|, sa = amax / 127,
 * qa = rint(x * (127 / amax)) (round to nearest even; 0 when amax is 0), qsum = sum qa. Per output the float tile
 * starts at 0 and takes, group by group in k order, t = fma(float(sum u qa), d * sa, fma(-128 d, sa * float(qsum), t))
 * (each product rounded, as the reference's vector multiplies are); then bias, residual and the activation as above.
 * ---------------------------------------------------------------------------------------------------------------- */
void orc_quantize_activations(const float* a, int m, int K, int8_t* qa, float* scale, int32_t* qsum) {
    const int ng = K / 32;
    for (int r = 0; r < m; ++r)
        for (int g = 0; g < ng; ++g) {
            const float* x = a + (int64_t)r * K + g * 32;
            float amax = 0.0f;
            for (int k = 0; k < 32; ++k) amax = fmaxf(amax, fabsf(x[k]));
            const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
            int32_t sum = 0;
            for (int k = 0; k < 32; ++k) {
                const int32_t q = (int32_t)lrintf(x[k] * inv);
                qa[(int64_t)r * K + g * 32 + k] = (int8_t)q;
                sum += q;
            }
            scale[(int64_t)r * ng + g] = amax / 127.0f;
            qsum[(int64_t)r * ng + g] = sum;
        }
}

void orc_gemm_q8_int8act(const float* a, int m, const uint8_t* q8, const float* bias, int N, int K, int n_offset,
                         int n, const float* residual, int act, float* c) {
    const int ng = K / 32;
    int8_t* qa = (int8_t*)malloc((size_t)m * K);
    float* sa = (float*)malloc(sizeof(float) * (size_t)m * ng);
    int32_t* qs = (int32_t*)malloc(sizeof(int32_t) * (size_t)m * ng);
    orc_quantize_activations(a, m, K, qa, sa, qs);
    for (int j = 0; j < n; ++j) {
        const int col = n_offset + j;
        if (col >= N) break;
        for (int i = 0; i < m; ++i) {
            float t = 0.0f;
            for (int g = 0; g < ng; ++g) {
                const uint8_t* blk = q8 + ((int64_t)col * ng + g) * 34;
                const float d = orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
                int32_t acc = 0;
                for (int k = 0; k < 32; ++k) acc += ((int32_t)(int8_t)blk[2 + k] + 128) * qa[(int64_t)i * K + g * 32 + k];
                const float s = sa[(int64_t)i * ng + g];
                const float sq = s * (float)qs[(int64_t)i * ng + g];
                t = fmaf((float)acc, d * s, fmaf(-128.0f * d, sq, t));
            }
            float v = t + (bias ? bias[col] : 0.0f);
            if (residual) v += residual[(int64_t)i * n + j];
            c[(int64_t)i * n + j] = apply_act(v, act);
        }
    }
    free(qa);
    free(sa);
    free(qs);
}

/* Elementwise activation in place (the decoders run gelu_tanh / silu as separate passes). */
void orc_activate(float* x, int64_t count, int act) {
    for (int64_t i = 0; i < count; ++i) x[i] = apply_act(x[i], act);
}

/* ------------------------------------------------------------------------------------------------------------------
 * Row LayerNorm as the decoders run it (src/decoders.cpp:23-42 norm_rows): fp64 sums for mean and variance, fp32
 * normalisation, optional affine gamma/beta, optional adaLN (1 + scale) and shift. y may alias x.
 * ---------------------------------------------------------------------------------------------------------------- */
void orc_norm_rows(const float* x, float* y, int rows, int dim, float eps, const float* gamma, const float* beta,
                   const float* shift, const float* scale) {
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (int64_t)r * dim;
        float* yr = y + (int64_t)r * dim;
        double sum = 0.0;
        for (int c = 0; c < dim; ++c) sum += xr[c];
        const float mean = (float)(sum / dim);
        double sq = 0.0;
        for (int c = 0; c < dim; ++c) sq += (double)(xr[c] - mean) * (xr[c] - mean);
        const float inv = 1.0f / sqrtf((float)(sq / dim) + eps);
        for (int c = 0; c < dim; ++c) {
            float v = (xr[c] - mean) * inv;
            if (gamma) v = v * gamma[c] + beta[c];
            if (scale) v = v * (1.0f + scale[c]) + shift[c];
            yr[c] = v;
        }
    }
}

/* ------------------------------------------------------------------------------------------------------------------
 * Per-head L2 norm of q or k (src/decoders.cpp:74-86 rms_heads): x * sqrt(hd) / max(|x|, 1e-12) * gamma, rows ld apart.
 * ---------------------------------------------------------------------------------------------------------------- */
void orc_rms_heads(float* x, int rows, int ld, int heads, int hd, const float* gamma) {
    const float root = sqrtf((float)hd);
    for (int r = 0; r < rows; ++r)
        for (int h = 0; h < heads; ++h) {
            float* p = x + (int64_t)r * ld + (int64_t)h * hd;
            const float* g = gamma + (int64_t)h * hd;
            float ss = 0.0f;
            for (int d = 0; d < hd; ++d) ss += p[d] * p[d];
            const float nrm = sqrtf(ss);
            const float mult = root / (nrm > 1e-12f ? nrm : 1e-12f);
            for (int d = 0; d < hd; ++d) p[d] = p[d] * mult * g[d];
        }
}

/* ------------------------------------------------------------------------------------------------------------------
 * Multi-head attention over projected rows (src/kernels.cpp:629-746 attention / attention_blocked): per head, scores
 * s_j = q . k_j (fp32 chain over the head dims), p_j = exp((s_j - max) / sqrt(hd)), normalised by their sum, and
 * out = sum_j p_j v_j. q rows are ldq apart, k and v rows ldkv apart, out rows dim apart. Head h uses columns
 * [h hd, (h + 1) hd).
 * ---------------------------------------------------------------------------------------------------------------- */
void orc_attention(const float* q, int lq, int ldq, const float* k, const float* v, int lk, int ldkv, int heads,
                   int head_dim, float* out, int dim) {
    const float scale = 1.0f / sqrtf((float)head_dim);
    float* s = (float*)malloc(sizeof(float) * (size_t)lk);
    for (int h = 0; h < heads; ++h)
        for (int i = 0; i < lq; ++i) {
            const float* qr = q + (int64_t)i * ldq + (int64_t)h * head_dim;
            float mx = -INFINITY;
            for (int j = 0; j < lk; ++j) {
                const float* kr = k + (int64_t)j * ldkv + (int64_t)h * head_dim;
                float acc = 0.0f;
                for (int d = 0; d < head_dim; ++d) acc = fmaf(qr[d], kr[d], acc);
                s[j] = acc;
                if (acc > mx) mx = acc;
            }
            float total = 0.0f;
            for (int j = 0; j < lk; ++j) {
                s[j] = expf((s[j] - mx) * scale);
                total += s[j];
            }
            const float inv = 1.0f / total;
            for (int j = 0; j < lk; ++j) s[j] *= inv;
            float* o = out + (int64_t)i * dim + (int64_t)h * head_dim;
            for (int d = 0; d < head_dim; ++d) o[d] = 0.0f;
            for (int j = 0; j < lk; ++j) {
                const float* vr = v + (int64_t)j * ldkv + (int64_t)h * head_dim;
                for (int d = 0; d < head_dim; ++d) o[d] = fmaf(s[j], vr[d], o[d]);
            }
        }
    free(s);
}

/* ------------------------------------------------------------------------------------------------------------------
 * Output heads of the synthetic Gaussian MLP (14 raw values per point -> 14 activated values, same order):
 *   pos 0..2 identity; scale 3..5 exp; rot 6..9 as src/decoders.cpp:422-428: r = f * lr_rotation + (1, 0, 0, 0)
 *   with the default lr_rotation 0.1 (src/weights.hpp:27), divided by max(|r|, 1e-12); color 10..12 sigmoid;
 *   opacity 13 sigmoid (src/decoders.cpp:429).
 * ---------------------------------------------------------------------------------------------------------------- */
/* ------------------------------------------------------------------------------------------------------------------
 * The Gaussian decoder's position embedding (src/decoders.cpp:215-230 pos_embed): per row, for each of the 3
 * coordinates v and each of the fd frequencies f, sin((v f) pi) then, fd columns later, cos((v f) pi); columns from
 * 6 fd on are zero. out: [rows, dim].
 * ---------------------------------------------------------------------------------------------------------------- */
void orc_pos_embed(const float* x, int64_t rows, const float* freqs, int fd, int dim, float* out) {
    const float pi = 3.14159265358979323846f;
    for (int64_t r = 0; r < rows; ++r) {
        float* o = out + r * dim;
        for (int c = 0; c < 3; ++c) {
            const float v = x[r * 3 + c];
            for (int j = 0; j < fd; ++j) {
                const float ang = (v * freqs[j]) * pi;
                o[c * 2 * fd + j] = sinf(ang);
                o[c * 2 * fd + fd + j] = cosf(ang);
            }
        }
        for (int j = 6 * fd; j < dim; ++j) o[j] = 0.0f;
    }
}

/* ------------------------------------------------------------------------------------------------------------------
 * The octree decoder's level embedding (src/decoders.cpp:254-259): for the 128 level frequencies f,
 * cos(((resolution f) 2) pi) then sin(((resolution f) 2) pi). out: 256 floats.
 * ---------------------------------------------------------------------------------------------------------------- */
void orc_level_embed(float resolution, const float* freqs, float* out) {
    const float pi = 3.14159265358979323846f;
    for (int i = 0; i < 128; ++i) {
        const float ang = ((resolution * freqs[i]) * 2.0f) * pi;
        out[i] = cosf(ang);
        out[128 + i] = sinf(ang);
    }
}

/* ------------------------------------------------------------------------------------------------------------------
 * Decoders::to_gaussians (src/decoders.cpp:393-433): per anchor a (xyz anchors[a]) and Gaussian g of per_anchor G,
 * from the anchor's 15 G features (xyz offsets at 0, colour at 3G, scale at 6G, rotation at 9G, opacity at 13G,
 * offset scale at 14G):
 *   offset_scale = softplus(f_os + base_offset_scale)
 *   xyz = (tanh(f_xyz lr_xyz + perturbation[g]) * 0.5 perturbe offset_scale + anchor) - 0.5
 *   f_dc = f_dc lr_dc; scale = sqrt(softplus(f_sc lr_scaling + scale_offset)^2 + kernel^2) with
 *   scale_offset = sb + log(-expm1(-sb)) in double (inverse softplus of sb = scaling_bias)
 *   rotation = (f_rot lr_rotation + (1, 0, 0, 0)) / max(|.|, 1e-12)
 *   opacity = 1 / (1 + exp(-(f_op lr_opacity + log(ob / (1 - ob))))) with ob = opacity_bias
 * softplus(x) = x above 20, else log1p(exp(x)) (src/decoders.cpp:90). rep = [perturbe, kernel, scaling_bias,
 * opacity_bias, lr_xyz, lr_dc, lr_opacity, lr_scaling, lr_rotation] (src/weights.hpp:25-28). Outputs: xyz, f_dc,
 * scale [anchors G, 3], rotation [anchors G, 4], opacity [anchors G].
 * ---------------------------------------------------------------------------------------------------------------- */
static float orc_softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

void orc_to_gaussians(const float* anchors, int64_t rows, const float* features, int G, const float* perturbation,
                      float base_offset_scale, const float* rep, float* xyz, float* f_dc, float* scale,
                      float* rotation, float* opacity) {
    const float perturbe = rep[0], kernel = rep[1];
    const double sb = rep[2], ob = rep[3];
    const float lr_xyz = rep[4], lr_dc = rep[5], lr_opacity = rep[6], lr_scaling = rep[7], lr_rotation = rep[8];
    const float scale_offset = (float)(sb + log(-expm1(-sb)));
    const float opacity_offset = (float)log(ob / (1.0 - ob));
    const int stride = G * 15, xyz0 = 0, dc0 = G * 3, sc0 = G * 6, rot0 = G * 9, op0 = G * 13, os0 = G * 14;
    for (int64_t a = 0; a < rows; ++a) {
        const float* f = features + a * stride;
        for (int g = 0; g < G; ++g) {
            const int64_t i = a * G + g;
            const float offset_scale = orc_softplus(f[os0 + g] + base_offset_scale);
            for (int c = 0; c < 3; ++c) {
                const float o = tanhf(f[xyz0 + g * 3 + c] * lr_xyz + perturbation[g * 3 + c]) * 0.5f * perturbe *
                                offset_scale;
                xyz[i * 3 + c] = (o + anchors[a * 3 + c]) - 0.5f;
                f_dc[i * 3 + c] = f[dc0 + g * 3 + c] * lr_dc;
                const float s = orc_softplus(f[sc0 + g * 3 + c] * lr_scaling + scale_offset);
                scale[i * 3 + c] = sqrtf(s * s + kernel * kernel);
            }
            float q[4], norm = 0.0f;
            for (int c = 0; c < 4; ++c) {
                q[c] = f[rot0 + g * 4 + c] * lr_rotation + (c == 0 ? 1.0f : 0.0f);
                norm += q[c] * q[c];
            }
            norm = sqrtf(norm);
            if (norm < 1e-12f) norm = 1e-12f;
            for (int c = 0; c < 4; ++c) rotation[i * 4 + c] = q[c] / norm;
            opacity[i] = 1.0f / (1.0f + expf(-(f[op0 + g] * lr_opacity + opacity_offset)));
        }
    }
}

void orc_gaussian_heads(const float* raw, int64_t points, float* out) {
    for (int64_t p = 0; p < points; ++p) {
        const float* f = raw + p * 14;
        float* o = out + p * 14;
        for (int c = 0; c < 3; ++c) o[c] = f[c];
        for (int c = 3; c < 6; ++c) o[c] = expf(f[c]);
        float r[4], nrm = 0.0f;
        for (int c = 0; c < 4; ++c) {
            r[c] = f[6 + c] * 0.1f + (c == 0 ? 1.0f : 0.0f);
            nrm += r[c] * r[c];
        }
        nrm = sqrtf(nrm);
        if (nrm < 1e-12f) nrm = 1e-12f;
        for (int c = 0; c < 4; ++c) o[6 + c] = r[c] / nrm;
        for (int c = 10; c < 14; ++c) o[c] = 1.0f / (1.0f + expf(-f[c]));
    }
}
