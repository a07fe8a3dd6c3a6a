// q8_common.cuh - pieces shared by the Q8_0 GEMM kernels (q8_gemm.cu: tcgen05 path for M > 16; q8_gemv.cu: the
// streaming path for M <= 16): the launch parameters, the output epilogue (bias, residual, activation, rounding) and
// the exact in-register dequantisation of sixteen codes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "internal.h"
#include "ptx.cuh"

namespace idol {
namespace q8 {

struct Params {
    const uint8_t* tiles;
    const float* bias;
    const void* residual;
    void* y;
    int m, n, k, kb;
    int row_tiles, layout_stages;  // chunk grid of the tiled layout
    int row_begin;            // first weight row of tile 0 (the window start rounded down to 128)
    int n_offset, n_count;    // output columns [n_offset, n_offset + n_count)
    long long ldy, ldr;
    int act;
    int bias_after_round;
    int stages_per_split, stages_total;
    int y_tma;                // the output tensor map may be used for TMA stores (2-byte output, aligned rows)
    // Per-head norm of the stored output (src/decoders.cpp:74-86 rms_heads, head dim 64) applied in the staged
    // epilogue: columns [0, hn_split) with hn_gamma_a, [hn_split, hn_cols) with hn_gamma_b; hn_cols = 0: none.
    const float* hn_gamma_a;
    const float* hn_gamma_b;
    int hn_cols, hn_split;
};

template <typename OutT>
__device__ __forceinline__ float out_round(float v) {
    if constexpr (sizeof(OutT) == 4) return v;
    else if constexpr (std::is_same<OutT, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(v));
    else return __half2float(__float2half_rn(v));
}
template <typename OutT>
__device__ __forceinline__ OutT to_out(float v) {
    if constexpr (sizeof(OutT) == 4) return v;
    else if constexpr (std::is_same<OutT, __nv_bfloat16>::value) return __float2bfloat16_rn(v);
    else return __float2half_rn(v);
}
template <typename OutT>
__device__ __forceinline__ float from_out(OutT v) {
    if constexpr (sizeof(OutT) == 4) return v;
    else if constexpr (std::is_same<OutT, __nv_bfloat16>::value) return __bfloat162float(v);
    else return __half2float(v);
}

// Activations of the epilogue. SiLU is v sigmoid(v) = v / (1 + e^-v), on the fast base-2 exponential and approximate
// division intrinsics (relative error near 2^-21; e^-v overflowing to +inf gives -0, the correct limit). GELU-tanh is
// 0.5 v (1 + tanh u) with u = sqrt(2/pi) v (1 + 0.044715 v^2), the tanh from the special-function unit's tanh.approx
// (one instruction; absolute error near 2^-11 |tanh u|, so the output's absolute error stays below 2^-12 |v|, far
// under the tolerance of the layers that consume it). GELU-erf keeps erff.
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int kAct>
__device__ __forceinline__ float activate_t(float v) {
    if constexpr (kAct == IDOL_ACT_GELU_ERF) {
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    } else if constexpr (kAct == IDOL_ACT_GELU_TANH) {
        const float u = (0.7978845608028654f * v) * fmaf(0.044715f, v * v, 1.0f);
        const float h = 0.5f * v;
        return fmaf(h, tanh_approx(u), h);
    } else if constexpr (kAct == IDOL_ACT_SILU) {
        return __fdividef(v, 1.0f + __expf(-v));
    } else {
        return v;
    }
}

__device__ __forceinline__ float activate(float v, int act) {
    switch (act) {
        case IDOL_ACT_GELU_ERF: return activate_t<IDOL_ACT_GELU_ERF>(v);
        case IDOL_ACT_GELU_TANH: return activate_t<IDOL_ACT_GELU_TANH>(v);
        case IDOL_ACT_SILU: return activate_t<IDOL_ACT_SILU>(v);
        default: return v;
    }
}

// Epilogue for one accumulator value: output (token m, weight row `row`).
template <typename OutT>
__device__ __forceinline__ void finish(const Params& p, int m, int row, float acc) {
    if (m >= p.m || row >= p.n || row < p.n_offset || row >= p.n_offset + p.n_count) return;
    const float b = p.bias ? p.bias[row] : 0.0f;
    float v = p.bias_after_round ? out_round<OutT>(acc) + b : acc + b;
    const int col = row - p.n_offset;
    if (p.residual) v += from_out<OutT>(static_cast<const OutT*>(p.residual)[(long long)m * p.ldr + col]);
    v = activate(v, p.act);
    static_cast<OutT*>(p.y)[(long long)m * p.ldy + col] = to_out<OutT>(v);
}

// 16 signed codes (one uint4) times d, as 8 packed 2-element registers of the operand type.
// Exact dequantisation in three steps: PRMT places the byte u = q + 128 into the mantissa of 32768, giving
// f = 32896 + q exactly; one packed FMA forms f d - 32896 d = q d with a single rounding, which is exact because q d
// has at most 19 significant bits and 32896 d = 2^7 (2^8 + 1) d at most 20; the pair is then rounded to the operand
// type (round to nearest even), which is what tools/idol_triton.py:62,83 does to the fp32 product d * q.
template <bool kBF16>
__device__ __forceinline__ void dequant16(uint4 c, float2 dd, float2 ncd, uint32_t* out) {
    const uint32_t w[4] = {c.x ^ 0x80808080u, c.y ^ 0x80808080u, c.z ^ 0x80808080u, c.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float f0 = __uint_as_float(__byte_perm(w[i], 0x47000000u, 0x7504));
        const float f1 = __uint_as_float(__byte_perm(w[i], 0x47000000u, 0x7514));
        const float f2 = __uint_as_float(__byte_perm(w[i], 0x47000000u, 0x7524));
        const float f3 = __uint_as_float(__byte_perm(w[i], 0x47000000u, 0x7534));
        const float2 p01 = __ffma2_rn(make_float2(f0, f1), dd, ncd);
        const float2 p23 = __ffma2_rn(make_float2(f2, f3), dd, ncd);
        if constexpr (kBF16) {
            out[2 * i] = pack_bf16x2(p01.x, p01.y);
            out[2 * i + 1] = pack_bf16x2(p23.x, p23.y);
        } else {
            out[2 * i] = pack_f16x2(p01.x, p01.y);
            out[2 * i + 1] = pack_f16x2(p23.x, p23.y);
        }
    }
}

// The 32 codes of one Q4_K sub-block (one uint4; byte i holds the codes of k = 2i and 2i + 1 in its low and high
// nibble) with fp32 a = d sc and b = dmin m, as 16 packed registers of the operand type in k order. PRMT places a code
// u in the mantissa of 32768 (f = 32768 + u exactly); one packed FMA forms f a - 32768 a = u a, exact because u a has
// at most 21 significant bits; one packed add rounds u a - b once to fp32 - the reference's weight
// (tools/idol_packed.py:41-54, tools/idol_triton.py:80) - and the pair is rounded to the operand type.
template <bool kBF16>
__device__ __forceinline__ void dequant32_q4k(uint4 c, float a, float b, uint32_t* out) {
    const float2 aa = make_float2(a, a);
    const float2 na = make_float2(-32768.0f * a, -32768.0f * a);
    const float2 nb = make_float2(-b, -b);
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t sel = 0x7504u | ((uint32_t)j << 4);
            const float f0 = __uint_as_float(__byte_perm(lo, 0x47000000u, sel));
            const float f1 = __uint_as_float(__byte_perm(hi, 0x47000000u, sel));
            const float2 v = __fadd2_rn(__ffma2_rn(make_float2(f0, f1), aa, na), nb);
            out[4 * i + j] = kBF16 ? pack_bf16x2(v.x, v.y) : pack_f16x2(v.x, v.y);
        }
    }
}

}  // namespace q8

// The streaming kernel for M <= 16 (q8_gemv.cu): the number of K splits it would use for `groups` 32-row groups and
// `stages_total` k stages (0 when K is too long for it), and the launch.
int q8_gemv_splits(int device, int groups, int stages_total);
int q8_gemv(const GemmCall& c, const q8::Params& p, int splits);

}  // namespace idol
