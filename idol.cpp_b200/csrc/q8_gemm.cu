// q8_gemm.cu - Y[m, n] = X[m, K] . dequant(W)[n, K]^T + bias (+ residual) (-> act) on sm_100a tensor cores.
//
// Replaces the reference's src/kernels.cpp:246-296 gemm_quant (CPU) and tools/idol_triton.py:36-126 fused_linear
// (GPU). The problem is computed transposed, Y^T = W . X^T, so that the dequantized weights are the tcgen05 A operand
// and can be written straight from registers into tensor memory (TMEM), never touching shared memory as bf16:
//
//   producer warp (1 thread) : TMA loads of the X tile [BN tokens x 64 k] (128-byte swizzle) plus bulk copies of the
//                              tiled int8 codes [128 rows x 64 k] and their fp16 scales, one mbarrier per stage;
//   dequant warps (4 x 32)   : lane r of warp q owns weight row 32 q + r (= TMEM lane): reads its 64 codes and two
//                              scales from shared memory, forms bf16(d * q) exactly as the reference GPU path does
//                              (tools/idol_triton.py:62,83: fp32 product rounded to the activation dtype), and stores
//                              32 packed columns into the stage's TMEM A buffer with tcgen05.st;
//   MMA warp (1 thread)      : tcgen05.mma.kind::f16 D[128 x BN] (fp32, TMEM) += A[128 x 16] (TMEM) x B[16 x BN]
//                              (shared memory descriptor), four per stage, then tcgen05.commit frees the stage;
//   epilogue (dequant warps) : tcgen05.ld of the accumulator, bias, residual, activation, store.
//
// Split-K: with `splits` > 1 the CTAs that share an output tile form a thread-block cluster along z; each reduces its
// K range into TMEM, parks the partial tile in its own shared memory, and after a cluster barrier every CTA sums a
// share of the tile's tokens over the cluster through distributed shared memory. No global scratch is used.
//
// Large M (from 1024 tokens, when the tiles fill the GPU) takes the dense path instead: q8_dense_tiles_kernel
// dequantises the window's weights into a per-(device, stream) scratch laid out as pre-swizzled bf16/f16 tiles, and
// the persistent kernel in dense mode runs on CTA pairs (256 x 256 tiles) with both MMA operands fed by TMA into shared
// memory, its MMA thread free of the dequantising warps' per-stage hand-offs (see q8_gemm_impl for the measurements).
//
// Every spin-wait is bounded (ptx.cuh mbar_wait); a timeout raises a sticky device error bit and the kernel winds
// down instead of hanging.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "internal.h"
#include "ptx.cuh"
#include "q8_common.cuh"

namespace idol {

IDOL_DEVICE_ERROR_READER(take_device_error_gemm)

namespace {

using namespace q8;

constexpr int kRowsPerTile = 128;   // weight rows (output features) per CTA = TMEM lanes
constexpr int kStageK = 64;         // k per pipeline stage: two Q8 blocks, one 128-byte swizzle row of bf16
constexpr int kDequantWarps = 8;    // two per TMEM lane quarter: one per Q8 block of a stage
constexpr int kThreads = 64 + 32 * kDequantWarps;  // warp 0 producer, warp 1 MMA / TMEM owner, warps 2-9 dequant
// One stage of weights = one chunk of the tiled layout: 8192 code bytes + 512 scale bytes, one bulk copy.
static_assert(kTileRows == kRowsPerTile && kTileK == kStageK, "the GEMM stage is the layout's chunk");

template <int BN, int S, int kFmt = kFmtQ8>
struct Config {
    static constexpr int kXBytes = BN * 128;                         // BN rows of 64 bf16
    static constexpr int kChunk = chunk_bytes<kFmt>();                // one stage of weights: 8704 (Q8) / 6144 (Q4_K)
    static constexpr int kStageBytes = kXBytes + kChunk;
    static constexpr int kACol0 = BN < 32 ? 32 : BN;                 // TMEM column of A stage 0 (D at column 0)
    static constexpr int kColsNeeded = kACol0 + S * 32;
    static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64 : kColsNeeded <= 128 ? 128
                                     : kColsNeeded <= 256 ? 256 : 512;
    static constexpr int kBarBytes = 8 * (3 * S + 1) + 16;
    // At least 80 KB so that no more than two CTAs share an SM: two TMEM allocations of <= 256 columns always fit,
    // and a CTA never waits in tcgen05.alloc on a neighbour that is itself waiting for its cluster.
    static constexpr int kSmemUsed = 1024 + S * kStageBytes + kBarBytes;
    static constexpr int kSmemBytes = kSmemUsed < 80 * 1024 ? 80 * 1024 : kSmemUsed;
    static_assert(kColsNeeded <= 512, "TMEM budget");
    static_assert(S * kXBytes >= BN * kRowsPerTile * 4, "split-K partial tile must fit in the X ring");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
};

// One warp's share of a stage: rows 32 q .. 32 q + 31 of the weight chunk at `chunk` (both 32-deep Q8 blocks, or the
// first `blocks` of them), dequantised into TMEM columns col .. col + 31 of those lanes (lane_base folded into col).
// Blocks past K are written as zeros.
template <bool kBF16>
__device__ __forceinline__ void dequant_stage(const uint8_t* chunk, int q, int lane, int blocks, uint32_t col) {
    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(chunk + kChunkCodeBytes + q * 128);
    uint32_t regs[32];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        if (b < blocks) {
            const uint8_t* cbase = chunk + q * 2048 + b * 1024 + lane * 16;
            const float d = __half2float(__ushort_as_half(sbase[b * 32 + lane]));
            const float2 dd = make_float2(d, d);
            const float2 ncd = make_float2(-32896.0f * d, -32896.0f * d);
            dequant16<kBF16>(*reinterpret_cast<const uint4*>(cbase), dd, ncd, regs + 16 * b);
            dequant16<kBF16>(*reinterpret_cast<const uint4*>(cbase + 512), dd, ncd, regs + 16 * b + 8);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) regs[16 * b + j] = 0u;
        }
    }
    tmem_st16(col, *reinterpret_cast<const uint32_t(*)[16]>(regs));
    tmem_st16(col + 16, *reinterpret_cast<const uint32_t(*)[16]>(regs + 16));
    tmem_st_wait();
}

// The same for a Q4_K chunk: rows 32 q .. 32 q + 31, both 32-deep sub-blocks (codes two per byte, fp32 A and B of
// the row), weights fl(A code - B) rounded to the operand type, into TMEM columns col .. col + 31.
template <bool kBF16>
__device__ __forceinline__ void dequant_stage_q4k(const uint8_t* chunk, int q, int lane, int blocks, uint32_t col) {
    const float4 prm = *reinterpret_cast<const float4*>(chunk + kQ4KCodeBytes + (q * 32 + lane) * 16);
    uint32_t regs[32];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        if (b < blocks) {
            const uint4 c = *reinterpret_cast<const uint4*>(chunk + q * 1024 + b * 512 + lane * 16);
            dequant32_q4k<kBF16>(c, b ? prm.y : prm.x, b ? prm.w : prm.z, regs + 16 * b);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) regs[16 * b + j] = 0u;
        }
    }
    tmem_st16(col, *reinterpret_cast<const uint32_t(*)[16]>(regs));
    tmem_st16(col + 16, *reinterpret_cast<const uint32_t(*)[16]>(regs + 16));
    tmem_st_wait();
}

// Epilogue over `cols` consecutive accumulator columns (tokens m .. m + cols - 1) of one weight row, with the
// activation fixed at compile time so the per-element loop carries no dispatch.
// kRv: the residual values of these columns are in `rv`, loaded ahead by the caller. A chunk wholly inside M (m is
// warp-uniform, so every lane takes the same path) then runs as straight-line code with no per-element bounds test:
// those tests were branches per element that tripled the residual epilogue's branch count and stalled its warps on
// instruction fetch (ncu: a 16384 x 1024 x 1024 fp32-residual launch took 2.0x the time of the same launch without
// a residual). The arithmetic and its order are the same on every path.
template <typename OutT, int kCols, int kAct, bool kRv>
__device__ __forceinline__ void finish_cols_act(const Params& p, int m, int row, const uint32_t* v, float bias,
                                                const float* rv) {
    const int col = row - p.n_offset;
    OutT* y = static_cast<OutT*>(p.y) + col;
    if constexpr (kRv) {
        const bool round_first = p.bias_after_round != 0;
        if (m + kCols <= p.m) {
#pragma unroll
            for (int j = 0; j < kCols; ++j) {
                const float a = __uint_as_float(v[j]);
                const float x = ((round_first ? out_round<OutT>(a) : a) + bias) + rv[j];
                y[(long long)(m + j) * p.ldy] = to_out<OutT>(activate_t<kAct>(x));
            }
            return;
        }
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
            if (m + j >= p.m) break;
            const float a = __uint_as_float(v[j]);
            const float x = ((round_first ? out_round<OutT>(a) : a) + bias) + rv[j];
            y[(long long)(m + j) * p.ldy] = to_out<OutT>(activate_t<kAct>(x));
        }
    } else {
        const OutT* res = static_cast<const OutT*>(p.residual);
        if (!res && !p.bias_after_round && m + kCols <= p.m) {
#pragma unroll
            for (int j = 0; j < kCols; ++j)
                y[(long long)(m + j) * p.ldy] = to_out<OutT>(activate_t<kAct>(__uint_as_float(v[j]) + bias));
            return;
        }
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
            if (m + j >= p.m) break;
            const float acc = __uint_as_float(v[j]);
            float x = p.bias_after_round ? out_round<OutT>(acc) + bias : acc + bias;
            if (res) x += from_out<OutT>(res[(long long)(m + j) * p.ldr + col]);
            y[(long long)(m + j) * p.ldy] = to_out<OutT>(activate_t<kAct>(x));
        }
    }
}

template <typename OutT, int kCols, bool kRv = false>
__device__ __forceinline__ void finish_cols(const Params& p, int m, int row, const uint32_t* v, float bias,
                                            bool row_ok, const float* rv = nullptr) {
    if (!row_ok) return;
    switch (p.act) {
        case IDOL_ACT_GELU_ERF: finish_cols_act<OutT, kCols, IDOL_ACT_GELU_ERF, kRv>(p, m, row, v, bias, rv); break;
        case IDOL_ACT_GELU_TANH: finish_cols_act<OutT, kCols, IDOL_ACT_GELU_TANH, kRv>(p, m, row, v, bias, rv); break;
        case IDOL_ACT_SILU: finish_cols_act<OutT, kCols, IDOL_ACT_SILU, kRv>(p, m, row, v, bias, rv); break;
        default: finish_cols_act<OutT, kCols, IDOL_ACT_NONE, kRv>(p, m, row, v, bias, rv); break;
    }
}

// L2 prefetch of the residual that the epilogue of an output tile will read: token `token`'s values of the tile's
// features [row0, row0 + 128) inside the window, one bulk prefetch of the 16-byte aligned part of that row segment
// (512 bytes for a full fp32 tile). Issued while the tile's main loop runs, so that the epilogue's residual loads,
// one per token and feature, find their lines in L2 instead of waiting for HBM. Nothing outside the residual rows
// the epilogue reads is touched.
template <typename OutT>
__device__ __forceinline__ void prefetch_residual_row(const Params& p, int row0, int token) {
    if (p.residual == nullptr || token < 0 || token >= p.m) return;
    const int c0 = max(row0, p.n_offset) - p.n_offset;
    const int c1 = min(row0 + kRowsPerTile, p.n_offset + p.n_count) - p.n_offset;
    if (c1 <= c0) return;
    const OutT* r = static_cast<const OutT*>(p.residual) + (long long)token * p.ldr;
    const uintptr_t a = (reinterpret_cast<uintptr_t>(r + c0) + 15) & ~static_cast<uintptr_t>(15);
    const uintptr_t b = reinterpret_cast<uintptr_t>(r + c1) & ~static_cast<uintptr_t>(15);
    if (b > a) prefetch_l2_bulk(reinterpret_cast<const void*>(a), (uint32_t)(b - a));
}

// Epilogue of one weight row (TMEM lane) over kSpan accumulator columns from TMEM address `acc` (tokens m0 ...),
// 16 (or 8) columns per tcgen05.ld. With a residual, its values are loaded kMaxGroup tokens at a time before the
// columns they meet, so a row waits one memory latency per kMaxGroup tokens instead of one per 16 (as many as the
// kernel's register budget holds: 16 in the fused persistent kernels, whose 576 threads have 113 registers each and
// whose residual rows are prefetched to L2 one tile ahead; 32 in their dense form, which has no dequantisation code
// competing for registers (the block's out projection 99.9 -> 91.2 us at 32768 tokens); 64 in the 320-thread
// kernel). Control flow around the warp-collective tcgen05.ld depends only on
// warp-uniform values; row_ok gates the per-lane memory accesses.
template <typename OutT, int kSpan, int kMaxGroup = 32>
__device__ __forceinline__ void epilogue_span(const Params& p, int m0, int row, uint32_t acc, float bias,
                                              bool row_ok) {
    constexpr int kChunk = kSpan >= 16 ? 16 : 8;
    constexpr int kGroup = kSpan >= kMaxGroup ? kMaxGroup : kSpan;
    if constexpr (kGroup % 16 == 0) {
        if (p.residual != nullptr) {
            // Unconditional loads from clamped addresses (a lane outside the window reads the window's first column,
            // a token past M the last token): per-element conditions made predicated or branching loads that cost
            // more than the loads. Values read for such positions are never used.
            const OutT* res = static_cast<const OutT*>(p.residual) + (row_ok ? row - p.n_offset : 0);
            for (int g0 = 0; g0 < kSpan && m0 + g0 < p.m; g0 += kGroup) {
                float rv[kGroup];
#pragma unroll
                for (int j = 0; j < kGroup; ++j)
                    rv[j] = from_out<OutT>(res[(long long)min(m0 + g0 + j, p.m - 1) * p.ldr]);
#pragma unroll
                for (int c0 = 0; c0 < kGroup; c0 += 16) {
                    if (m0 + g0 + c0 >= p.m) break;
                    uint32_t v[16];
                    tmem_ld16(acc + g0 + c0, v);
                    tmem_ld_wait();
                    finish_cols<OutT, 16, true>(p, m0 + g0 + c0, row, v, bias, row_ok, rv + c0);
                }
            }
            return;
        }
    }
    for (int c0 = 0; c0 < kSpan && m0 + c0 < p.m; c0 += kChunk) {
        uint32_t v[kChunk];
        if constexpr (kChunk == 16) tmem_ld16(acc + c0, v);
        else tmem_ld8(acc + c0, v);
        tmem_ld_wait();
        finish_cols<OutT, kChunk>(p, m0 + c0, row, v, bias, row_ok);
    }
}

// epilogue_span for an fp32 output with an fp32 residual, the residual streamed through this warp's ring in shared
// memory (`ring`: two buffers of kResGroup tokens x 32 lanes of floats, token-major: the warp's 32 features of a token
// are 128 contiguous bytes) while the current group is finished, so the bytes in flight are not bounded by the
// registers a thread can hold (the residual loads bounded the out projection: 0.45 of the tensor peak). When the
// warp's 32 features all lie in the window and start on a 16-byte boundary, each 16-byte cp.async copies four
// features of one token (eight lanes per token, four tokens per instruction): a quarter of the copy instructions and
// address arithmetic of one 4-byte copy per lane and token, which took issue slots from the MMA thread on the same
// scheduler (tensor pipe 60% -> 43% active with the residual at 32768 x 1024 x 1024). Lanes then read words that
// other lanes copied, so each group's wait is followed by a warp barrier, and a warp barrier before each issue keeps
// a buffer from being refilled while a lane still reads it. Otherwise each lane copies its own feature's values with
// 4-byte copies. Addresses are clamped as in epilogue_span; values read for positions outside the window or past M
// are never used.
constexpr int kResGroup = 32;
template <int kSpan>
__device__ __forceinline__ void epilogue_span_res_ring(const Params& p, int m0, int row, uint32_t acc, float bias,
                                                       bool row_ok, uint32_t ring, int lane) {
    static_assert(kSpan % kResGroup == 0 && kResGroup % 4 == 0, "whole groups");
    const int col0 = row - lane - p.n_offset;  // the window column of the warp's first feature
    const bool vec = __all_sync(0xffffffffu, row_ok) && col0 % 4 == 0 && p.ldr % 4 == 0 &&
                     reinterpret_cast<uintptr_t>(p.residual) % 16 == 0;
    const float* res = static_cast<const float*>(p.residual) + (vec ? col0 + (lane % 8) * 4 : (row_ok ? row - p.n_offset : 0));
    const int groups = min(kSpan, p.m - m0 + kResGroup - 1) / kResGroup;  // groups with at least one token below M
    // The outputs leave the same way when the output rows allow 16-byte stores and no activation follows.
    const bool vst = vec && p.act == IDOL_ACT_NONE && p.ldy % 4 == 0 && reinterpret_cast<uintptr_t>(p.y) % 16 == 0;
    float* yv = static_cast<float*>(p.y) + col0 + (lane % 8) * 4;
    auto issue = [&](int g) {
        if (vec) {
            const uint32_t dst = ring + (uint32_t)(((g & 1) * kResGroup * 32 + (lane / 8) * 32 + (lane % 8) * 4) * 4);
#pragma unroll
            for (int j = 0; j < kResGroup; j += 4)
                cp_async16(dst + (uint32_t)(j * 32 * 4),
                           res + (long long)min(m0 + g * kResGroup + j + lane / 8, p.m - 1) * p.ldr);
        } else {
            const uint32_t dst = ring + (uint32_t)(((g & 1) * kResGroup * 32 + lane) * 4);
#pragma unroll 8
            for (int j = 0; j < kResGroup; ++j)
                cp_async4(dst + (uint32_t)(j * 32 * 4), res + (long long)min(m0 + g * kResGroup + j, p.m - 1) * p.ldr);
        }
        cp_async_commit();
    };
    if (groups > 0) issue(0);
    for (int g = 0; g < groups; ++g) {
        __syncwarp();  // every lane has finished reading group g - 1, whose buffer group g + 1 refills
        if (g + 1 < groups) issue(g + 1);
        else cp_async_commit();  // an empty group keeps "all but the newest group" meaning group g
        cp_async_wait<1>();
        __syncwarp();  // group g's copies of every lane have landed
        const uint32_t src = ring + (uint32_t)(((g & 1) * kResGroup * 32 + lane) * 4);
#pragma unroll
        for (int c0 = 0; c0 < kResGroup; c0 += 16) {
            float rv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float v;
                asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(src + (uint32_t)((c0 + j) * 32 * 4)));
                rv[j] = v;
            }
            uint32_t v[16];
            tmem_ld16(acc + g * kResGroup + c0, v);
            tmem_ld_wait();
            if (vst) {
                // The finished values go back into this lane's words of the ring.
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float a = __uint_as_float(v[j]);
                    const float x = ((p.bias_after_round ? out_round<float>(a) : a) + bias) + rv[j];
                    asm volatile("st.shared.f32 [%0], %1;" ::"r"(src + (uint32_t)((c0 + j) * 32 * 4)), "f"(x));
                }
            } else {
                finish_cols<float, 16, true>(p, m0 + g * kResGroup + c0, row, v, bias, row_ok, rv);
            }
        }
        if (vst) {
            // Each 16-byte store writes four features of one token (eight lanes per token, four tokens per
            // instruction) from the ring.
            __syncwarp();
            const uint32_t vsrc = ring + (uint32_t)(((g & 1) * kResGroup * 32 + (lane / 8) * 32 + (lane % 8) * 4) * 4);
#pragma unroll
            for (int j = 0; j < kResGroup; j += 4) {
                const int m = m0 + g * kResGroup + j + lane / 8;
                uint4 w;
                asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                             : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                             : "r"(vsrc + (uint32_t)(j * 32 * 4)));
                if (m < p.m) *reinterpret_cast<uint4*>(yv + (long long)m * p.ldy) = w;
            }
        }
    }
    cp_async_wait<0>();
}

// The staged form of epilogue_span for the TMA-store path: the finished value of token m0 + j goes to shared address
// st + 256 j of the staging tile (token-major, 128 features of 2 bytes per token; this lane's feature folded into st),
// and a single TMA store later writes the tile. Features outside the output window and tokens past M are written
// too: the store clips them. The 32 lanes of a warp store 64 contiguous bytes per token (no bank conflict).
// GELU-erf takes 8 columns per tcgen05.ld: erff on 16 values at once needs more than the 96 registers a thread has.
template <typename OutT, int kSpan, int kAct, bool kRes>
__device__ __forceinline__ void epilogue_span_staged(const Params& p, int m0, int row, uint32_t acc, float bias,
                                                     bool row_ok, uint32_t st) {
    constexpr int kC = kAct == IDOL_ACT_GELU_ERF ? 8 : 16;
    static_assert(kSpan % kC == 0 && sizeof(OutT) == 2, "whole chunks of a 2-byte output");
    // kRes: residual loads are unconditional, from clamped addresses, as in epilogue_span (per-element conditions
    // on 2-byte loads made this path 5x slower than the one without a residual). The path without a residual is
    // a separate instantiation, so that its code and registers carry nothing of the residual's.
    const OutT* res = kRes ? static_cast<const OutT*>(p.residual) + (row_ok ? row - p.n_offset : 0) : nullptr;
    for (int c0 = 0; c0 < kSpan && m0 + c0 < p.m; c0 += kC) {
        float rv[kC];
        if constexpr (kRes) {
#pragma unroll
            for (int j = 0; j < kC; ++j) rv[j] = from_out<OutT>(res[(long long)min(m0 + c0 + j, p.m - 1) * p.ldr]);
        }
        uint32_t v[kC];
        if constexpr (kC == 16) tmem_ld16(acc + c0, v);
        else tmem_ld8(acc + c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < kC; ++j) {
            const float a = __uint_as_float(v[j]);
            float x = p.bias_after_round ? out_round<OutT>(a) + bias : a + bias;
            if constexpr (kRes) x += rv[j];
            const OutT o = to_out<OutT>(activate_t<kAct>(x));
            st_shared_u16(st + (uint32_t)(c0 + j) * (kRowsPerTile * 2),
                          *reinterpret_cast<const uint16_t*>(&o));
        }
    }
}

// epilogue_span_staged with the residual choice made once per span.
template <typename OutT, int kSpan, int kAct>
__device__ __forceinline__ void epilogue_span_staged_any(const Params& p, int m0, int row, uint32_t acc, float bias,
                                                         bool row_ok, uint32_t st) {
    if (p.residual != nullptr) epilogue_span_staged<OutT, kSpan, kAct, true>(p, m0, row, acc, bias, row_ok, st);
    else epilogue_span_staged<OutT, kSpan, kAct, false>(p, m0, row, acc, bias, row_ok, st);
}

template <int BN, int S, bool kBF16, typename OutT, int kFmt>
__global__ void __launch_bounds__(kThreads, 1) q8_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const Params p) {
    using C = Config<BN, S, kFmt>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // The 128-byte swizzle needs 1024-aligned tiles in the shared address space.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* xs = smem;                                        // S x kXBytes, each 1024-aligned
    uint8_t* ws = xs + S * C::kXBytes;                         // S x 8704: codes then scales of the stage
    uint64_t* full = reinterpret_cast<uint64_t*>(ws + S * C::kChunk);
    uint64_t* empty = full + S;
    uint64_t* afull = empty + S;
    uint64_t* accfull = afull + S;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accfull + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int row0 = p.row_begin + blockIdx.x * kRowsPerTile;
    const int t128 = row0 / kRowsPerTile;  // row tile of the layout (always < row_tiles)
    const int m0 = blockIdx.y * BN;
    const int split = blockIdx.z;
    const int ks_begin = split * p.stages_per_split;
    const int ks_end = min(ks_begin + p.stages_per_split, p.stages_total);
    const int nks = ks_end - ks_begin;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&afull[s], kDequantWarps / 2);  // one arrival per dequant warp of the stage's group
        }
        mbar_init(accfull, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&xmap);
            int issued = 0;  // stages loaded so far
            for (int i = 0; i < nks; ++i) {
                const int s = i % S, u = i / S;
                if (i >= S && !mbar_wait(&empty[s], (u - 1) & 1, abort_flag)) break;
                ++issued;
                const int ks = ks_begin + i;
                const int b0 = ks * 2;
                const int nb = min(2, p.kb - b0);
                (void)nb;
                mbar_arrive_expect_tx(&full[s], C::kXBytes + C::kChunk);
                tma_load_2d(xs + s * C::kXBytes, &xmap, ks * kStageK, m0, &full[s]);
                bulk_load(ws + s * C::kChunk, p.tiles + ((long long)t128 * p.layout_stages + ks) * C::kChunk,
                          C::kChunk, &full[s]);
            }
            // The last load into each stage has landed before the CTA can leave (see mbar_drain).
            for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i) mbar_drain(&full[i % S], (i / S) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // One wait per stage: every dequant warp waited for the stage's bytes (full) before it reported its A
            // stage (afull), so afull completing implies the token tile has landed too.
            const uint32_t idesc = make_idesc_f16(kRowsPerTile, BN, kBF16);
            for (int i = 0; i < nks; ++i) {
                const int s = i % S, u = i / S;
                if (!mbar_wait(&afull[s], u & 1, abort_flag)) break;
                tc_fence_after();
                const int ks = ks_begin + i;
                const bool two_blocks = (p.kb - ks * 2) >= 2;
                const uint32_t xaddr = smem_u32(xs + s * C::kXBytes);
                const uint32_t a0 = tmem + C::kACol0 + s * 32;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < 2 || two_blocks)
                        mma_ts(tmem, a0 + j * 8, make_sdesc_sw128(xaddr + j * 32), idesc, (i > 0 || j > 0) ? 1u : 0u);
                mma_commit(&empty[s]);
            }
            mma_commit(accfull);
        }
    } else {
        // Dequant warps: warp w may only touch TMEM lanes [32 (w % 4), 32 (w % 4) + 32). Warps 2-5 take the even
        // stages, warps 6-9 the odd ones, each dequantising both Q8 blocks of its stage for its 32 weight rows: the
        // same work per warp as one block per stage, with half the barrier traffic per stage (waits, arrivals and
        // tcgen05 fences of other warps slow the MMA issuer down).
        const int q = warp % 4;
        const int half = (warp - 2) / 4;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        // The tile's residual rows go to L2 while the main loop runs (one token per dequant thread, BN <= 256).
        if (gridDim.z == 1 && (warp - 2) * 32 + lane < BN)
            prefetch_residual_row<OutT>(p, row0, m0 + (warp - 2) * 32 + lane);
        // The A buffer of slot s was last read by stage i - S. Its MMA has completed once full[s] completes for stage
        // i: the producer issues stage i's copies only after that MMA's commit (empty[s]), so one wait covers both.
        // With an odd S the two groups alternate on a slot: stage i and stage i - S of slot s belong to different
        // groups, and a parity wait cannot tell phase u of full[s] from phase u - 2. So the group first waits for the
        // commit of stage i - S (empty[s]; commits complete in order, and the group has seen the commit of its own
        // previous stage's predecessor, so that wait is exact): stage i - S had landed before its MMA, so full[s]
        // is then in phase u and the parity wait below is exact too.
        for (int i = half; i < nks; i += 2) {
            const int s = i % S, u = i / S;
            bool got = true;
            if constexpr (S % 2 == 1) {
                if (i >= S) got = mbar_wait(&empty[s], (u - 1) & 1, abort_flag);
            }
            if (got) got = mbar_wait(&full[s], u & 1, abort_flag);
            if (!__all_sync(0xffffffffu, got)) break;  // tcgen05.st below is warp-collective
            tc_fence_after();
            if constexpr (kFmt == kFmtQ4K)
                dequant_stage_q4k<kBF16>(ws + s * C::kChunk, q, lane, min(2, p.kb - (ks_begin + i) * 2),
                                         tmem + lane_base + C::kACol0 + s * 32);
            else
                dequant_stage<kBF16>(ws + s * C::kChunk, q, lane, min(2, p.kb - (ks_begin + i) * 2),
                                     tmem + lane_base + C::kACol0 + s * 32);
            tc_fence_before();
            __syncwarp();  // every lane's stores are complete and fenced before lane 0 reports the warp
            if (lane == 0) mbar_arrive(&afull[s]);
        }

        // Epilogue: the accumulator is ready once the last commit lands. Warp half h covers tokens
        // [h BN / 2, (h + 1) BN / 2) of its 32 rows.
        const bool ok = __all_sync(0xffffffffu, mbar_wait(accfull, 0, abort_flag));
        tc_fence_after();
        const int row = row0 + 32 * q + lane;
        constexpr int kHalf = BN / 2;
        constexpr int kChunk = kHalf >= 16 ? 16 : 8;
        const int c_begin = half * kHalf;
        if (gridDim.z == 1) {
            const bool row_ok = ok && row < p.n && row >= p.n_offset && row < p.n_offset + p.n_count;
            const float bias = (row_ok && p.bias) ? p.bias[row] : 0.0f;
            epilogue_span<OutT, kHalf, 64>(p, m0 + c_begin, row, tmem + lane_base + c_begin, bias, row_ok);
        } else {
            // Park the partial tile [token][row] in this CTA's X ring (all loads into it have landed).
            float* red = reinterpret_cast<float*>(xs);
            for (int c0 = c_begin; c0 < c_begin + kHalf; c0 += kChunk) {
                uint32_t v[kChunk];
                if constexpr (kChunk == 16) tmem_ld16(tmem + lane_base + c0, v);
                else tmem_ld8(tmem + lane_base + c0, v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < kChunk; ++j)
                    red[(c0 + j) * kRowsPerTile + 32 * q + lane] = ok ? __uint_as_float(v[j]) : 0.0f;
            }
        }
        tc_fence_before();
    }

    __syncthreads();
    if (gridDim.z > 1) {
        cluster_sync();
        if (warp >= 2) {
            const int q = warp % 4;
            const int half = (warp - 2) / 4;
            const int row = row0 + 32 * q + lane;
            const int z = (int)cluster_ctarank();
            const int nz = (int)gridDim.z;  // <= 8 (a portable cluster)
            const uint32_t red_local = smem_u32(xs);
            const bool row_ok = row < p.n && row >= p.n_offset && row < p.n_offset + p.n_count;
            const float bias = (row_ok && p.bias) ? p.bias[row] : 0.0f;
            const OutT* res = static_cast<const OutT*>(p.residual);
            OutT* y = static_cast<OutT*>(p.y);
            const int col = row - p.n_offset;
            // This thread finishes tokens t0, t0 + step, ... of its row. Eight tokens at a time, every rank's partial
            // and the residual are loaded before any is used (one latency per eight tokens); the partials are summed
            // in rank order (absent ranks add exact zeros), so the result does not depend on timing.
            const int t0 = z + half * nz, step = 2 * nz;
            const int count = t0 < BN ? (BN - t0 + step - 1) / step : 0;
            for (int i0 = 0; i0 < count; i0 += 8) {
                float acc[8], rv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int t = t0 + (i0 + u) * step;
                    acc[u] = 0.0f;
                    rv[u] = 0.0f;
                    if (i0 + u < count) {
                        const uint32_t off = (uint32_t)((t * kRowsPerTile + 32 * q + lane) * 4);
                        float v[8];
#pragma unroll
                        for (int rk = 0; rk < 8; ++rk)
                            v[rk] = rk < nz ? ld_cluster_f32(map_to_rank(red_local + off, (uint32_t)rk)) : 0.0f;
#pragma unroll
                        for (int rk = 0; rk < 8; ++rk) acc[u] += v[rk];
                        if (res && row_ok && m0 + t < p.m)
                            rv[u] = from_out<OutT>(res[(long long)(m0 + t) * p.ldr + col]);
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int t = t0 + (i0 + u) * step;
                    if (i0 + u < count && row_ok && m0 + t < p.m) {
                        float x = p.bias_after_round ? out_round<OutT>(acc[u]) + bias : acc[u] + bias;
                        if (res) x += rv[u];
                        y[(long long)(m0 + t) * p.ldy + col] = to_out<OutT>(activate(x, p.act));
                    }
                }
            }
        }
        cluster_sync();
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// ------------------------------------------------------------------------------------------------------------------
// Dense tile layout: the large-M path dequantises the tiled Q8_0 weights once per call into this layout and runs a
// GEMM whose weight operand comes from shared memory like the tokens (the reference's own large-M GPU strategy,
// tools/idol_triton.py:112-117, dequantises into a scratch and calls a dense GEMM). Per (row tile, k stage) one 16 KB
// tile: 128 rows of 64 operand-type values, 128 bytes per row, the 16-byte units of row r stored in the order of the
// 128-byte swizzle (unit c at position c ^ (r % 8)), so that one bulk copy puts the tile into shared memory exactly
// as a TMA load with that swizzle would and the MMA reads it with the same descriptor as the token tile. The values
// are those the fused kernel forms in registers (dequant16: bf16 or fp16 of the exact fp32 product d q); rows past N
// and blocks past K are zero because their codes and scales are.
constexpr int kDenseChunkBytes = kRowsPerTile * kStageK * 2;
// Smallest M that takes the dense path by default (measured on B200, see q8_gemm_impl).
constexpr int64_t kDenseMinM = 1024;

template <bool kBF16>
__global__ void __launch_bounds__(128) q8_dense_tiles_kernel(const uint8_t* __restrict__ tiles,
                                                             uint8_t* __restrict__ dense) {
    // The dense GEMM that follows is a programmatic dependent launch: it may start its set-up now and waits for this
    // grid to complete (griddepcontrol.wait) before it reads anything from global memory.
    asm volatile("griddepcontrol.launch_dependents;");
    const uint8_t* src = tiles + (long long)blockIdx.x * kChunkBytes;
    uint8_t* dst = dense + (long long)blockIdx.x * kDenseChunkBytes;
    const int r = threadIdx.x, q = r / 32, lane = r % 32;  // thread r: row r of the tile (lane r of quarter q)
    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(src + kChunkCodeBytes + q * 128);
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const float d = __half2float(__ushort_as_half(sbase[b * 32 + lane]));
        const float2 dd = make_float2(d, d);
        const float2 ncd = make_float2(-32896.0f * d, -32896.0f * d);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t w[8];
            dequant16<kBF16>(*reinterpret_cast<const uint4*>(src + q * 2048 + b * 1024 + h * 512 + lane * 16), dd, ncd,
                             w);
            const int c = 4 * b + 2 * h;  // 16-byte unit of k = 32 b + 16 h within the 128-byte row
            *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(dst + r * 128 + (((c + 1) ^ (r & 7)) * 16)) = make_uint4(w[4], w[5], w[6], w[7]);
        }
    }
}

// ------------------------------------------------------------------------------------------------------------------
// Persistent CTA-pair variant (cta_group::2) for large M.
//
// Two CTAs of a cluster share one MMA of M = 256 weight rows x N = BN tokens: each CTA dequantises its own 128 rows
// into its own TMEM but TMA-loads only its half of the token tile, so a CTA moves BN/2 x 64 x 2 bytes of activations
// per stage instead of BN x 64 x 2 (L2 -> SM traffic per tensor-pipe cycle ~48 instead of ~81 bytes per SM at
// BN = 256). The even CTA issues the MMAs; its barriers collect both CTAs' TMA bytes and both CTAs' dequantised
// stages, and its commits arrive on the stage and accumulator barriers of both CTAs. No TMA multicast: each CTA loads
// its own half.
//
// The grid holds one pair per two SMs and each pair walks the output tiles p, p + P, p + 2P, ... (P pairs). Three
// rings run continuously across tiles:
//   * S shared-memory stages (token half + weight chunk), filled by the producer, freed by the MMA commit (empty);
//   * SA TMEM A slots (32 columns: one stage of dequantised weights), filled by the dequant warps (afull) - fewer
//     than S, since TMEM also holds the accumulators. Slot i % SA is free again once stage i - SA is consumed, which
//     the same per-stage commit reports (empty[(i - SA) % S]), so the MMA thread commits once per stage;
//   * two TMEM accumulators of BN columns: the MMA warp fills accumulator lt % 2 for its lt-th tile and commits
//     accfull; eight separate epilogue warps drain it (bias, residual, activation, stores) and report accempty, so
//     the epilogue of one tile runs under the main loop of the next.
// TMEM budget: 2 BN + 32 SA <= 512 columns (BN = 192 with SA = 4, BN = 128 with SA = 8). With SA == S the
// dequant warps need no wait for their A slot: the codes of stage i land only after the commit of stage i - S.
constexpr int kEpilogueWarps = 8;   // two per TMEM lane quarter, half of the token columns each
constexpr int kPairThreads = 64 + 32 * kDequantWarps + 32 * kEpilogueWarps;

// kYStage: bytes of the shared staging tile the epilogue hands to TMA stores (0: the epilogue stores directly).
// kDense: the weights of a stage arrive already dequantised (a 16 KB tile of the dense layout, see
// q8_dense_tiles_kernel) and both MMA operands come from shared memory; no A slots in tensor memory.
template <int BN, int S, int SA, bool kPair, int kYStage = 0, bool kDense = false, bool kResRing = false>
struct ConfigPersistent {
    static constexpr int kHalf = kPair ? BN / 2 : BN;  // token rows this CTA loads per stage
    static constexpr int kXBytes = kHalf * 128;
    static constexpr int kWBytes = kDense ? kDenseChunkBytes : kChunkBytes;  // one stage of weights
    static constexpr int kStageBytes = kXBytes + kWBytes;
    static constexpr int kACol0 = 2 * BN;  // accumulators at columns 0 and BN, then the A slots
    static constexpr int kColsNeeded = kACol0 + (kDense ? 0 : SA * 32);
    static constexpr int kTmemCols = kColsNeeded <= 256 ? 256 : 512;
    static constexpr int kBarBytes = 8 * (3 * S + SA + 7) + 16;
    static_assert(SA <= S, "an A slot is released by the commit of a stage no later than the one reusing its buffer");
    // Dequant groups alternate by stage parity: an even SA keeps each A slot (afull) with one group; an odd S needs
    // the A-slot wait (SA < S) to order the parity waits on a stage slot the two groups share.
    static_assert(SA % 2 == 0 && (S % 2 == 0 || SA < S), "stage and A-slot counts");
    // kResRing: each epilogue warp's residual ring (epilogue_span_res_ring), 8 KB per warp.
    static constexpr int kRingBytes = kResRing ? kEpilogueWarps * 2 * kResGroup * 32 * 4 : 0;
    static constexpr int kSmemUsed = 1024 + S * kStageBytes + kYStage + kRingBytes + kBarBytes;
    // At least 120 KB: one CTA per SM, so a TMEM allocation of 512 columns never waits on a neighbour.
    static constexpr int kSmemBytes = kSmemUsed < 120 * 1024 ? 120 * 1024 : kSmemUsed;
    static_assert(kColsNeeded <= 512, "TMEM budget");
    static_assert(kSmemUsed <= 227 * 1024, "shared memory budget");
    static_assert(BN % (kPair ? 32 : 16) == 0 && BN >= 64 && BN <= 256, "MMA N");
    static_assert(kXBytes % 1024 == 0, "each token half must stay 1024-aligned for the 128-byte swizzle");
    static_assert(!kDense || kWBytes % 1024 == 0, "dense: 1024-aligned weight tiles");
    static constexpr int kYStageBytes = kYStage;
    static_assert(kYStage % 1024 == 0, "the staging tile keeps the weight chunks after it 16-byte aligned");
};

struct PersistentSchedule {
    int units_n;   // row units along the output features (256 rows for a pair, 128 for one CTA)
    int tiles_m;   // BN-token tiles along M
};

// kPair = false is the same pipeline on one CTA (cta_group::1, M = 128 rows, the whole token tile loaded locally, no
// cluster): X and the codes of a stage land on one barrier, so the dequant warps wait once per stage.
//
// kYStage > 0 (one CTA, 2-byte output, a window starting on a 128-row tile): every tile leaves through a shared
// staging tile and one TMA store (`ymap`: the output window [n_count features x M tokens]) instead of 96 global
// stores per lane; the store issuer (epilogue warp 0, lane 0) reports the staging tile free again on sfree once the
// store has read it.
// rms_heads (src/decoders.cpp:74-86, head dim 64) of a staged tile in place: BN token rows of 128 features (two heads,
// 256 bytes per token), features tile_row0 .. tile_row0 + 127 of the output. Eight lanes take one (token, head) row,
// eight features each, with the reduction of rms_heads_vec_kernel (norms.cu), so a head gets the same bits as that
// kernel gives the stored row. The epilogue warps share the BN x 2 rows round-robin (BN x 2 is a multiple of 128, so
// every lane of a warp runs the same iterations), four rows per thread at a time so that their loads, reductions and
// stores overlap (one row at a time, the norm was on the epilogue's critical path: QKV 188 us at 32768 tokens against
// 158 without the norm); rows past M hold stale values and are normalised too: the TMA store clips them.
template <int BN>
__device__ __forceinline__ void head_norm_staged(uint8_t* ys, int tile_row0, const Params& p, int ew, int lane) {
    constexpr int kStride = 4 * kEpilogueWarps;  // (token, head) rows per round of all epilogue warps
    constexpr int kBatch = 4;                     // rows a thread carries at once (independent chains)
    static_assert((BN * 2) % (kStride * kBatch) == 0, "whole batches of (token, head) rows");
    const int l8 = lane % 8;
    // A thread's rows all fall in the same head of the 128-feature tile (task parity is fixed: kStride is even), so
    // its eight gammas are loaded once.
    const int hh = (ew * 4 + lane / 8) % 2;
    const int f0 = tile_row0 + hh * 64 + l8 * 8;
    const float* g = f0 < p.hn_split ? p.hn_gamma_a + f0 : p.hn_gamma_b + (f0 - p.hn_split);
    const float4 g0 = *reinterpret_cast<const float4*>(g), g1 = *reinterpret_cast<const float4*>(g + 4);
    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    for (int t0 = ew * 4 + lane / 8; t0 < BN * 2; t0 += kStride * kBatch) {
        uint4 raw[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
            raw[u] = *reinterpret_cast<const uint4*>(ys + ((t0 + u * kStride) / 2) * 256 + hh * 128 + l8 * 16);
        float v[kBatch][8], ss[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const __nv_bfloat162* pr = reinterpret_cast<const __nv_bfloat162*>(&raw[u]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __bfloat1622float2(pr[i]);
                v[u][2 * i] = f.x;
                v[u][2 * i + 1] = f.y;
            }
            ss[u] = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) ss[u] = fmaf(v[u][i], v[u][i], ss[u]);
        }
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1)
#pragma unroll
            for (int u = 0; u < kBatch; ++u) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const float mult = 8.0f / fmaxf(sqrtf(ss[u]), 1e-12f);  // sqrt(64) = 8
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __nv_bfloat162 o2 = __floats2bfloat162_rn(v[u][2 * i] * mult * gg[2 * i],
                                                                v[u][2 * i + 1] * mult * gg[2 * i + 1]);
                o[i] = *reinterpret_cast<const uint32_t*>(&o2);
            }
            *reinterpret_cast<uint4*>(ys + ((t0 + u * kStride) / 2) * 256 + hh * 128 + l8 * 16) =
                make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

template <int BN, int S, int SA, bool kPair, bool kBF16, typename OutT, int kYStage, bool kDense, bool kResRing>
__global__ void __launch_bounds__(kPairThreads, 1) q8_gemm_persistent_kernel(
    const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
    const __grid_constant__ CUtensorMap wmap, const Params p, const PersistentSchedule sched) {
    using C = ConfigPersistent<BN, S, SA, kPair, kYStage, kDense, kResRing>;
    static_assert(!kResRing || (kYStage == 0 && sizeof(OutT) == 4), "the residual ring serves the fp32 direct path");
    static_assert(kYStage == 0 || ((!kPair || kDense) && sizeof(OutT) == 2 && kYStage >= BN * kRowsPerTile * 2),
                  "staging: one CTA (or a dense pair), a 2-byte output and room for the whole tile");
    constexpr int kRowsPerUnit = kPair ? 2 * kRowsPerTile : kRowsPerTile;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* xs = smem;
    uint8_t* ys = xs + S * C::kXBytes;                                              // output staging (1024-aligned)
    uint8_t* ws = ys + C::kYStageBytes;                                             // S weight stages
    uint8_t* rs = ws + S * C::kWBytes;                                              // residual rings (kResRing)
    uint64_t* xfull = reinterpret_cast<uint64_t*>(rs + C::kRingBytes);              // even CTA: both halves landed
    uint64_t* cfull = xfull + S;                                                    // this CTA's codes landed
    uint64_t* empty = cfull + S;                                                    // both: stage s consumed
    uint64_t* afull = empty + S;                                                    // even CTA: A slot written (both)
    uint64_t* accfull = afull + SA;                                                 // both: accumulator b ready
    uint64_t* accempty = accfull + 2;                                               // even CTA: accumulator b drained
    uint64_t* sfull = accempty + 2;                                                 // staging tile written
    uint64_t* sfree = sfull + 1;                                                    // staging tile read by TMA
    uint64_t* snorm = sfree + 1;                                                    // staged heads normalised
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(snorm + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const uint32_t rank = kPair ? cluster_ctarank() : 0u;
    const int pair_id = kPair ? blockIdx.x / 2 : blockIdx.x;   // the unit (pair or single CTA) this CTA belongs to
    const int num_pairs = kPair ? gridDim.x / 2 : gridDim.x;
    const int total_tiles = sched.units_n * sched.tiles_m;
    const int nks = p.stages_total;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&cfull[s], 1);
            mbar_init(&empty[s], 1);
        }
        // One arrival per dequant warp of the stage's group (four per CTA), and per epilogue warp, of every CTA.
        for (int a = 0; a < SA; ++a) mbar_init(&afull[a], (kPair ? 2 : 1) * (kDequantWarps / 2));
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accfull[b], 1);
            mbar_init(&accempty[b], (kPair ? 2 : 1) * kEpilogueWarps);
        }
        mbar_init(sfull, kEpilogueWarps);  // one arrival per epilogue warp once its share of the staging tile is in
        mbar_init(sfree, 1);               // the store issuer, once the TMA store has read the staging tile
        mbar_init(snorm, kEpilogueWarps);  // one arrival per epilogue warp once its share of the heads is normalised
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        if constexpr (kPair) {
            tmem_alloc_pair(tmem_holder, C::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_holder, C::kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync();  // the peer's barriers exist before anything arrives on them
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    // Dense: launched as a programmatic dependent of the dequantisation kernel, so the set-up above overlapped it;
    // nothing global (weights, tokens, bias, residual, output) is touched before that grid has completed. A no-op for
    // an ordinary launch.
    if constexpr (kDense) asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&xmap);
            int i = 0;  // stage counter across tiles (= stages loaded so far)
            bool ok = true;
            for (int t = pair_id; t < total_tiles && ok; t += num_pairs) {
                const int row0 = p.row_begin + (t % sched.units_n) * kRowsPerUnit + (int)rank * kRowsPerTile;
                const int t128 = row0 / kRowsPerTile;
                const bool valid = t128 < p.row_tiles;  // the pair's second tile can fall past N
                const int m0 = (t / sched.units_n) * BN;
                for (int ks = 0; ks < nks; ++ks, ++i) {
                    const int s = i % S, u = i / S;
                    if (i >= S && !mbar_wait(&empty[s], (u - 1) & 1, abort_flag)) { ok = false; break; }
                    const uint8_t* chunk = p.tiles + ((long long)t128 * p.layout_stages + ks) * C::kWBytes;
                    if constexpr (kPair && kDense) {
                        // Both CTAs' token halves and weight tiles land on the even CTA's barrier (the MMA waits
                        // there only). The weight tile comes by TMA without swizzle, as the dense layout already
                        // holds it swizzled; a pair's second tile past N reads zeros.
                        if (rank == 0) mbar_arrive_expect_tx(&xfull[s], 2 * (C::kXBytes + C::kWBytes));
                        tma_load_2d_pair(xs + s * C::kXBytes, &xmap, ks * kStageK, m0 + (int)rank * C::kHalf,
                                         map_to_rank(smem_u32(&xfull[s]), 0));
                        tma_load_2d_pair(ws + s * C::kWBytes, &wmap, 0, (t128 * p.layout_stages + ks) * kRowsPerTile,
                                         map_to_rank(smem_u32(&xfull[s]), 0));
                    } else if constexpr (kPair) {
                        if (rank == 0) mbar_arrive_expect_tx(&xfull[s], 2 * C::kXBytes);
                        tma_load_2d_pair(xs + s * C::kXBytes, &xmap, ks * kStageK, m0 + (int)rank * C::kHalf,
                                         map_to_rank(smem_u32(&xfull[s]), 0));
                        mbar_arrive_expect_tx(&cfull[s], valid ? kChunkBytes : 0);
                        if (valid) bulk_load(ws + s * kChunkBytes, chunk, kChunkBytes, &cfull[s]);
                    } else {
                        mbar_arrive_expect_tx(&xfull[s], C::kXBytes + C::kWBytes);
                        tma_load_2d(xs + s * C::kXBytes, &xmap, ks * kStageK, m0, &xfull[s]);
                        bulk_load(ws + s * C::kWBytes, chunk, C::kWBytes, &xfull[s]);
                    }
                }
            }
            // The last loads into each stage have landed before the CTA can leave (see mbar_drain): this CTA's codes
            // on cfull; both CTAs' token halves on the even CTA's xfull (the odd CTA's copies count there too, and
            // the final cluster barrier keeps the odd CTA until the even one has drained).
            for (int j = i - S > 0 ? i - S : 0; j < i; ++j) {
                if constexpr (kPair && !kDense) mbar_drain(&cfull[j % S], (j / S) & 1);
                if (rank == 0) mbar_drain(&xfull[j % S], (j / S) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = make_idesc_f16(kPair ? 2 * kRowsPerTile : kRowsPerTile, BN, kBF16);
            int i = 0, lt = 0;
            bool ok = true;
            for (int t = pair_id; t < total_tiles && ok; t += num_pairs, ++lt) {
                // The epilogue warps of both CTAs must have read this accumulator's previous tile (two tiles ago).
                const int b = lt & 1;
                if (lt >= 2 && !mbar_wait(&accempty[b], ((lt >> 1) - 1) & 1, abort_flag)) break;
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * BN);
                for (int ks = 0; ks < nks; ++ks, ++i) {
                    // One wait per stage: the even CTA's dequant warps waited for both token halves (xfull) before
                    // they reported the A slot, so afull completing implies the stage's tokens have landed.
                    const int s = i % S;
                    const int a = i % SA, ua = i / SA;
                    // Dense: the stage's weights and tokens land on xfull; otherwise the A slot's barrier implies both.
                    if (!(kDense ? mbar_wait(&xfull[s], (i / S) & 1, abort_flag)
                                 : mbar_wait(&afull[a], ua & 1, abort_flag))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const bool two_blocks = (p.kb - ks * 2) >= 2;
                    const uint32_t xaddr = smem_u32(xs + s * C::kXBytes);
                    const uint32_t waddr = smem_u32(ws + s * C::kWBytes);
                    const uint32_t a0 = tmem + C::kACol0 + a * 32;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (j < 2 || two_blocks) {
                            if constexpr (kDense && kPair)
                                mma_ss_pair(acc, make_sdesc_sw128(waddr + j * 32), make_sdesc_sw128(xaddr + j * 32),
                                            idesc, (ks > 0 || j > 0) ? 1u : 0u);
                            else if constexpr (kDense)
                                mma_ss(acc, make_sdesc_sw128(waddr + j * 32), make_sdesc_sw128(xaddr + j * 32), idesc,
                                       (ks > 0 || j > 0) ? 1u : 0u);
                            else if constexpr (kPair)
                                mma_ts_pair(acc, a0 + j * 8, make_sdesc_sw128(xaddr + j * 32), idesc,
                                            (ks > 0 || j > 0) ? 1u : 0u);
                            else
                                mma_ts(acc, a0 + j * 8, make_sdesc_sw128(xaddr + j * 32), idesc,
                                       (ks > 0 || j > 0) ? 1u : 0u);
                        }
                    }
                    if constexpr (kPair) mma_commit_pair(&empty[s], 0x3);
                    else mma_commit(&empty[s]);
                }
                if constexpr (kPair) mma_commit_pair(&accfull[b], 0x3);
                else mma_commit(&accfull[b]);
            }
        }
    } else if (warp < 2 + kDequantWarps) {
      if constexpr (!kDense) {  // dense: the weights arrive dequantised and these warps wait at the final barrier
        // As in the single-CTA kernel: warps 2-5 take the even stages, warps 6-9 the odd ones, both Q8 blocks each.
        const int q = warp % 4;
        const int half = (warp - 2) / 4;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        int i = 0;
        bool ok = true;
        for (int t = pair_id; t < total_tiles && ok; t += num_pairs) {
            const int row0 = p.row_begin + (t % sched.units_n) * kRowsPerUnit + (int)rank * kRowsPerTile;
            const bool valid = row0 / kRowsPerTile < p.row_tiles;
            for (int ks = 0; ks < nks; ++ks, ++i) {
                if ((i & 1) != half) continue;
                const int s = i % S, u = i / S;
                const int a = i % SA;
                // A pair: this CTA's codes (cfull), and on the even CTA both token halves (xfull, see the MMA loop).
                // One CTA: codes and tokens land together on xfull.
                // The A-slot wait comes first: A slot a was last read by stage i - SA, and its commit (commits
                // complete in order) implies that of stage i - S, so stage i - S has landed and the parity waits on
                // xfull[s] / cfull[s] below cannot mistake phase u - 2 for phase u when the two groups alternate on a
                // slot (odd S). With SA == S (S even: one group per slot, which sees its slot's phases in order),
                // cfull[s] of stage i implies the commit of stage i - S (the producer waited for it).
                bool got = true;
                if constexpr (SA < S) {
                    if (i >= SA) {
                        const int r = i - SA;
                        got = mbar_wait(&empty[r % S], (r / S) & 1, abort_flag);
                    }
                }
                if (got && kPair) got = mbar_wait(&cfull[s], u & 1, abort_flag);
                if (got && rank == 0) got = mbar_wait(&xfull[s], u & 1, abort_flag);
                if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                tc_fence_after();
                dequant_stage<kBF16>(ws + s * kChunkBytes, q, lane, valid ? min(2, p.kb - ks * 2) : 0,
                                     tmem + lane_base + C::kACol0 + a * 32);
                tc_fence_before();
                __syncwarp();  // every lane's stores are complete and fenced before lane 0 reports the warp
                if (lane == 0) {
                    if (rank == 0) mbar_arrive(&afull[a]);
                    else mbar_arrive_remote(map_to_rank(smem_u32(&afull[a]), 0));
                }
            }
        }
      }
    } else {
        // Epilogue warps: warp w reads TMEM lanes of quarter w % 4; the two warps of a quarter split the columns.
        const int ew = warp - 2 - kDequantWarps;
        const int q = warp % 4;
        const int half = ew / 4;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        constexpr int kHalfCols = BN / 2;
        int lt = 0;
        int ns = 0;  // TMA stores issued so far (staged tiles)
        int nh = 0;  // staged tiles whose heads were normalised
        // The residual rows of a tile go to L2 one tile ahead of its epilogue (while its main loop runs): one token
        // per epilogue thread (BN <= 256).
        auto prefetch_tile = [&](int t) {
            const int e = ew * 32 + lane;
            if (t < total_tiles && e < BN)
                prefetch_residual_row<OutT>(p, p.row_begin + (t % sched.units_n) * kRowsPerUnit +
                                                   (int)rank * kRowsPerTile, (t / sched.units_n) * BN + e);
        };
        prefetch_tile(pair_id);
        for (int t = pair_id; t < total_tiles; t += num_pairs, ++lt) {
            const int b = lt & 1;
            prefetch_tile(t + num_pairs);
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&accfull[b], (lt >> 1) & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            const int tile_row0 = p.row_begin + (t % sched.units_n) * kRowsPerUnit + (int)rank * kRowsPerTile;
            const int row = tile_row0 + 32 * q + lane;
            const int m0 = (t / sched.units_n) * BN;
            const bool row_ok = row < p.n && row >= p.n_offset && row < p.n_offset + p.n_count;
            const float bias = (row_ok && p.bias) ? p.bias[row] : 0.0f;
            const int c_begin = half * kHalfCols;
            const uint32_t acc = tmem + lane_base + (uint32_t)(b * BN);
            if constexpr (C::kYStageBytes > 0) {
                // Staged: every tile leaves through the staging tile and one TMA store at column tile_row0 - n_offset
                // (>= 0 and a multiple of 8: the host stages only windows with n_offset % 128 == 0).
                if (ns > 0 && !__all_sync(0xffffffffu, mbar_wait(sfree, (ns - 1) & 1, abort_flag))) break;
                const uint32_t st = smem_u32(ys) + 2u * (uint32_t)(c_begin * kRowsPerTile + 32 * q + lane);
                const int ms = m0 + c_begin;
                const uint32_t ac = acc + c_begin;
                switch (p.act) {
                    case IDOL_ACT_GELU_ERF:
                        epilogue_span_staged_any<OutT, kHalfCols, IDOL_ACT_GELU_ERF>(p, ms, row, ac, bias, row_ok, st);
                        break;
                    case IDOL_ACT_GELU_TANH:
                        epilogue_span_staged_any<OutT, kHalfCols, IDOL_ACT_GELU_TANH>(p, ms, row, ac, bias, row_ok, st);
                        break;
                    case IDOL_ACT_SILU:
                        epilogue_span_staged_any<OutT, kHalfCols, IDOL_ACT_SILU>(p, ms, row, ac, bias, row_ok, st);
                        break;
                    default:
                        epilogue_span_staged_any<OutT, kHalfCols, IDOL_ACT_NONE>(p, ms, row, ac, bias, row_ok, st);
                        break;
                }
                tc_fence_before();
                fence_proxy_async_shared();  // this lane's staging writes, before the TMA store reads them
                __syncwarp();
                if (lane == 0) {
                    if (rank == 0) mbar_arrive(&accempty[b]);
                    else mbar_arrive_remote(map_to_rank(smem_u32(&accempty[b]), 0));
                    mbar_arrive(sfull);
                }
                // rms_heads of the staged tile (tiles lie wholly inside or outside [0, hn_cols): hn_cols is a
                // multiple of 128): every epilogue warp waits for the whole tile, normalises its share of the
                // (token, head) rows in place and reports on snorm, which the store then waits for instead of sfull.
                const bool hn = tile_row0 < p.hn_cols;
                if (hn) {
                    if (!__all_sync(0xffffffffu, mbar_wait(sfull, ns & 1, abort_flag))) break;
                    head_norm_staged<BN>(ys, tile_row0, p, ew, lane);
                    fence_proxy_async_shared();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(snorm);
                }
                if (ew == 0) {
                    bool stored = true;
                    if (lane == 0) {
                        stored = mbar_wait(hn ? snorm : sfull, (hn ? nh : ns) & 1, abort_flag);
                        if (stored) {
                            tma_store_2d(&ymap, ys, tile_row0 - p.n_offset, m0);
                            bulk_commit_group();
                            bulk_wait_group_read0();
                        }
                        mbar_arrive(sfree);
                    }
                    __syncwarp();
                    if (!__shfl_sync(0xffffffffu, stored ? 1 : 0, 0)) break;
                }
                ++ns;
                nh += hn ? 1 : 0;
            } else {
                if constexpr (kResRing) {
                    if (p.residual != nullptr)
                        epilogue_span_res_ring<kHalfCols>(p, m0 + c_begin, row, acc + c_begin, bias, row_ok,
                                                          smem_u32(rs) + (uint32_t)(ew * 2 * kResGroup * 32 * 4), lane);
                    else
                        epilogue_span<OutT, kHalfCols, 32>(p, m0 + c_begin, row, acc + c_begin, bias, row_ok);
                } else {
                    epilogue_span<OutT, kHalfCols, kDense ? 32 : 16>(p, m0 + c_begin, row, acc + c_begin, bias,
                                                                     row_ok);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (rank == 0) mbar_arrive(&accempty[b]);
                    else mbar_arrive_remote(map_to_rank(smem_u32(&accempty[b]), 0));
                }
            }
        }
        if constexpr (C::kYStageBytes > 0) {
            if (ew == 0 && lane == 0 && ns > 0) bulk_wait_group0();  // the stores have completed before the CTA exits
        }
    }

    __syncthreads();
    if constexpr (kPair) cluster_sync();  // no CTA leaves while its peer may still arrive on its barriers
    if (warp == 1) {
        tc_fence_after();
        if constexpr (kPair) tmem_dealloc_pair(tmem, C::kTmemCols);
        else tmem_dealloc(tmem, C::kTmemCols);
    }
}

template <int BN, int S, int SA, bool kPair, bool kBF16, typename OutT, int kYStage = 0, bool kDense = false,
          bool kResRing = false>
int launch_persistent(const CUtensorMap& xmap, const CUtensorMap& ymap, const CUtensorMap& wmap, const Params& p,
                      int units_n, int tiles_m, cudaStream_t stream) {
    using C = ConfigPersistent<BN, S, SA, kPair, kYStage, kDense, kResRing>;
    auto kern = q8_gemm_persistent_kernel<BN, S, SA, kPair, kBF16, OutT, kYStage, kDense, kResRing>;
    static unsigned long long configured = 0;
    int dev = 0;
    IDOL_CUDA(cudaGetDevice(&dev));
    if (!(configured >> (dev & 63) & 1ull)) {
        IDOL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
        configured |= 1ull << (dev & 63);
    }
    const int total = units_n * tiles_m;
    const int max_units = kPair ? num_sms(dev) / 2 : num_sms(dev);
    const int grid_units = total < max_units ? total : max_units;
    PersistentSchedule sched = {units_n, tiles_m};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((kPair ? 2 : 1) * grid_units, 1, 1);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if constexpr (kPair) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 2;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if constexpr (kDense) {  // right after its dequantisation launch on the same stream (q8_gemm_impl)
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    IDOL_CUDA(cudaLaunchKernelEx(&cfg, kern, xmap, ymap, wmap, p, sched));
    return IDOL_OK;
}

// kind 0: CTA pair, 128- or 192-token tiles; kind 1: one CTA, 192-token tiles (with p.y_tma through the 48 KB
// staging tile and TMA stores, with five stages; otherwise six stages and direct stores); kind 2: the dense form of
// kind 1 (p.tiles is the dequantised tile layout; 40 KB stages: four beside the staging tile, five without); kind 3:
// the dense form on a CTA pair, 256 weight rows x 256 tokens per tile (each CTA loads its 128 weight rows and half of
// the tokens: 32 KB stages, five beside the 64 KB staging tile, six without), `wmap` the dense layout as rows of 64.
template <bool kBF16, typename OutT>
int dispatch_persistent(int kind, int bn, const CUtensorMap& xmap, const CUtensorMap& ymap, const CUtensorMap& wmap,
                        const Params& p, int units, int tiles_m, cudaStream_t stream) {
    if (kind == 3) {
        if constexpr (sizeof(OutT) == 2) {
            if (p.y_tma)
                return launch_persistent<256, 5, 4, true, kBF16, OutT, 256 * kRowsPerTile * 2, true>(
                    xmap, ymap, wmap, p, units, tiles_m, stream);
        }
        if constexpr (sizeof(OutT) == 4) {
            // Five stages beside the 64 KB residual rings: with 16-byte residual copies and stores the ring epilogue
            // takes few enough issue slots that it wins at every K (the blocks' out projection at 32768 tokens
            // 86.6 -> 79.0 us, ff2 220.8 -> 215.9 us against six stages and register-held residual groups).
            if (p.residual != nullptr)
                return launch_persistent<256, 5, 4, true, kBF16, OutT, 0, true, true>(xmap, ymap, wmap, p, units,
                                                                                    tiles_m, stream);
        }
        return launch_persistent<256, 6, 4, true, kBF16, OutT, 0, true>(xmap, ymap, wmap, p, units, tiles_m, stream);
    }
    if (kind == 2) {
        if constexpr (sizeof(OutT) == 2) {
            if (p.y_tma)
                return launch_persistent<192, 4, 4, false, kBF16, OutT, 192 * kRowsPerTile * 2, true>(
                    xmap, ymap, wmap, p, units, tiles_m, stream);
        }
        return launch_persistent<192, 5, 4, false, kBF16, OutT, 0, true>(xmap, ymap, wmap, p, units, tiles_m, stream);
    }
    if (kind == 1) {
        if constexpr (sizeof(OutT) == 2) {
            if (p.y_tma)
                return launch_persistent<192, 5, 4, false, kBF16, OutT, 192 * kRowsPerTile * 2>(xmap, ymap, wmap, p,
                                                                                              units, tiles_m, stream);
        }
        return launch_persistent<192, 6, 4, false, kBF16, OutT>(xmap, ymap, wmap, p, units, tiles_m, stream);
    }
    if (bn == 128) return launch_persistent<128, 8, 8, true, kBF16, OutT>(xmap, ymap, wmap, p, units, tiles_m, stream);
    return launch_persistent<192, 4, 4, true, kBF16, OutT>(xmap, ymap, wmap, p, units, tiles_m, stream);
}

template <int BN, int S, bool kBF16, typename OutT, int kFmt>
int launch(const CUtensorMap& xmap, const Params& p, int tiles_n, int tiles_m, int splits, cudaStream_t stream) {
    using C = Config<BN, S, kFmt>;
    auto kern = q8_gemm_kernel<BN, S, kBF16, OutT, kFmt>;
    static unsigned long long configured = 0;  // one bit per device: the shared-memory opt-in is set once
    int dev = 0;
    IDOL_CUDA(cudaGetDevice(&dev));
    if (!(configured >> (dev & 63) & 1ull)) {
        IDOL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
        configured |= 1ull << (dev & 63);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles_n, tiles_m, splits);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = splits;
    cfg.attrs = attr;
    cfg.numAttrs = splits > 1 ? 1 : 0;
    IDOL_CUDA(cudaLaunchKernelEx(&cfg, kern, xmap, p));
    return IDOL_OK;
}

template <bool kBF16, typename OutT, int kFmt>
int dispatch_fmt(int bn, const CUtensorMap& xmap, const Params& p, int tiles_n, int tiles_m, int splits,
                 cudaStream_t stream) {
    switch (bn) {
        case 16: return launch<16, 6, kBF16, OutT, kFmt>(xmap, p, tiles_n, tiles_m, splits, stream);
        case 32: return launch<32, 6, kBF16, OutT, kFmt>(xmap, p, tiles_n, tiles_m, splits, stream);
        case 64: return launch<64, 6, kBF16, OutT, kFmt>(xmap, p, tiles_n, tiles_m, splits, stream);
        case 128: return launch<128, 4, kBF16, OutT, kFmt>(xmap, p, tiles_n, tiles_m, splits, stream);
        // Five stages (204 KB): at M = 16384 the fifth stage hides the TMA latency that four leave exposed (measured
        // +6-16% on B200); six do not fit.
        default: return launch<256, 5, kBF16, OutT, kFmt>(xmap, p, tiles_n, tiles_m, splits, stream);
    }
}

template <bool kBF16, typename OutT>
int dispatch(int fmt, int bn, const CUtensorMap& xmap, const Params& p, int tiles_n, int tiles_m, int splits,
             cudaStream_t stream) {
    return fmt == kFmtQ4K ? dispatch_fmt<kBF16, OutT, kFmtQ4K>(bn, xmap, p, tiles_n, tiles_m, splits, stream)
                          : dispatch_fmt<kBF16, OutT, kFmtQ8>(bn, xmap, p, tiles_n, tiles_m, splits, stream);
}

int env_int(const char* name, int fallback) {
    const char* v = std::getenv(name);
    return v && *v ? std::atoi(v) : fallback;
}

}  // namespace

// Whether the output window can leave the one-CTA persistent kernel through TMA stores (see the kernel): a 2-byte
// output, a window starting on a 128-row tile, a 16-byte aligned base and row stride, and at least one full tile.
// IDOL_B200_GEMM_YTMA = 0 turns it off.
static bool staged_output_ok(const GemmCall& c) {
    return c.y_dtype != IDOL_F32 && c.n >= kRowsPerTile && c.m >= 192 && c.n_offset % kRowsPerTile == 0 &&
           (c.ldy * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(c.y) % 16 == 0 &&
           env_int("IDOL_B200_GEMM_YTMA", 1) != 0;
}

// ------------------------------------------------------------------------------------------------ dense path
// Scratch of the dense path, one buffer per (device, stream): a call dequantises its weights into it and the GEMM on
// the same stream reads them, so calls in stream order may share it and calls on different streams never do. Grown by
// allocating a larger buffer; the smaller one stays allocated until exit, because a CUDA graph captured earlier may
// still use it. Never allocated while the calling stream is being captured (the call then takes the fused kernel),
// nor while a NoScratchScope is active on the calling thread.
static std::mutex g_dense_mutex;
static std::map<std::pair<int, uintptr_t>, std::pair<void*, size_t>> g_dense_scratch;
static thread_local int g_no_scratch_depth = 0;

NoScratchScope::NoScratchScope() { ++g_no_scratch_depth; }
NoScratchScope::~NoScratchScope() { --g_no_scratch_depth; }

static void* dense_scratch(int device, cudaStream_t stream, size_t bytes) {
    if (g_no_scratch_depth > 0) return nullptr;
    std::lock_guard<std::mutex> lock(g_dense_mutex);
    auto& e = g_dense_scratch[{device, reinterpret_cast<uintptr_t>(stream)}];
    if (e.first && e.second >= bytes) return e.first;
    cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &status) != cudaSuccess || status != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;
    }
    size_t want = e.second ? 2 * e.second : (size_t)16 << 20;
    while (want < bytes) want *= 2;
    void* ptr = nullptr;
    if (cudaMalloc(&ptr, want) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    e = {ptr, want};
    return ptr;
}

// Token-tile width and split-K factor by M (the strategy choice). IDOL_B200_GEMM_BN and IDOL_B200_GEMM_SPLITS force
// them for tests and sweeps.
// Measured on B200 over the config-2 shapes: up to 64 tokens the launch is bound by streaming W, so K is split until
// the CTAs cover the SMs; above that a split pays only when K is long (>= 32 stages) and the tiles are few, since the
// cluster reduction costs about as much as a short main loop.
static void choose_tiles(int device, int64_t m, int tiles_n, int stages_total, int* bn, int* splits) {
    // 65-128 tokens: four 32-token tiles split K less deeply than two 64-token tiles for the same CTA count
    // (128 x 4096 x 1024: 17.9 -> 11.4 us; 128 x 1024 x 3072: 10.1 -> 9.7 us, measured on B200).
    int b = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 32 : 256;
    const int forced_bn = env_int("IDOL_B200_GEMM_BN", 0);
    if (forced_bn == 16 || forced_bn == 32 || forced_bn == 64 || forced_bn == 128 || forced_bn == 256) b = forced_bn;
    const int tiles = tiles_n * (int)((m + b - 1) / b);
    const int per_sm = b == 256 ? 1 : 2;
    const int slots = num_sms(device) * per_sm;
    int s = 1;
    if (m <= 64) {
        while (s < 8 && tiles * s * 2 <= slots && stages_total >= s * 2 * 2) s *= 2;
    } else if (stages_total >= 32) {
        while (s < 8 && tiles * s * 2 <= slots && stages_total >= s * 2 * 8) s *= 2;
    }
    const int forced_s = env_int("IDOL_B200_GEMM_SPLITS", 0);
    if (forced_s == 1 || forced_s == 2 || forced_s == 4 || forced_s == 8) s = forced_s;
    if (s > stages_total) s = 1;
    *bn = b;
    *splits = s;
}

static int q8_gemm_impl(const GemmCall& c, bool* head_norm_fused) {
    const Q8Matrix& w = *c.w;
    if (c.m < 0 || c.m > 0x7fffffff) return fail(IDOL_ERR_INVALID, "q8_gemm: m out of range");
    if (c.n < 0 || c.n_offset < 0 || c.n_offset + c.n > w.n) return fail(IDOL_ERR_INVALID, "q8_gemm: column window");
    if (c.m == 0 || c.n == 0) return IDOL_OK;
    if (c.x_dtype != IDOL_BF16 && c.x_dtype != IDOL_F16)
        return fail(IDOL_ERR_UNSUPPORTED, "q8_gemm: activations must be bf16 or f16");
    if (c.y_dtype != IDOL_BF16 && c.y_dtype != IDOL_F16 && c.y_dtype != IDOL_F32)
        return fail(IDOL_ERR_UNSUPPORTED, "q8_gemm: output must be bf16, f16 or f32");
    if (c.ldx < w.k || (c.ldx * 2) % 16 != 0 || (reinterpret_cast<uintptr_t>(c.x) % 16) != 0)
        return fail(IDOL_ERR_INVALID, "q8_gemm: x must be 16-byte aligned with a row stride that is a multiple of 8");
    if (c.ldy < c.n || (c.residual && c.ldr < c.n)) return fail(IDOL_ERR_INVALID, "q8_gemm: output row stride");
    if (c.act < IDOL_ACT_NONE || c.act > IDOL_ACT_SILU) return fail(IDOL_ERR_INVALID, "q8_gemm: activation");

    Params p = {};
    p.tiles = w.tiles;
    p.bias = w.bias;
    p.residual = c.residual;
    p.y = c.y;
    p.m = (int)c.m;
    p.n = w.n;
    p.k = w.k;
    p.kb = w.k / 32;
    p.row_tiles = row_tiles(w.n);
    p.layout_stages = k_stages(w.k);
    p.row_begin = (c.n_offset / kRowsPerTile) * kRowsPerTile;
    p.n_offset = c.n_offset;
    p.n_count = c.n;
    p.ldy = c.ldy;
    p.ldr = c.ldr;
    p.act = c.act;
    p.bias_after_round = (c.flags & IDOL_EPI_BIAS_AFTER_ROUND) ? 1 : 0;
    p.stages_total = (w.k + kStageK - 1) / kStageK;

    // Decode-sized batches stream W through the register-dequant kernel (IDOL_B200_GEMV=0 forces the tcgen05 path).
    if (c.m <= 16 && env_int("IDOL_B200_GEMV", 1) != 0) {
        const int groups = (c.n_offset + c.n - p.row_begin + 31) / 32;
        int gemv_splits = q8_gemv_splits(w.device, groups, p.stages_total);
        const int forced = env_int("IDOL_B200_GEMV_SPLITS", 0);  // sweeps and tests: 1, 2, 4 or 8
        if (gemv_splits > 0 && (forced == 1 || forced == 2 || forced == 4 || forced == 8) &&
            (p.stages_total + forced - 1) / forced <= 16)
            gemv_splits = forced;
        if (gemv_splits > 0) return q8_gemv(c, p, gemv_splits);
    }

    const int tiles_n = (c.n_offset + c.n - p.row_begin + kRowsPerTile - 1) / kRowsPerTile;
    int bn = 0, splits = 1;
    choose_tiles(w.device, c.m, tiles_n, p.stages_total, &bn, &splits);
    if (c.flags & IDOL_GEMM_WHOLE_K) splits = 1;

    // The persistent CTA-pair kernel overlaps each tile's epilogue with the next tile's main loop, which pays when the
    // main loop is short: measured on B200, K <= 512 with N >= 256 and M >= 4096 (the Gaussian MLP's 128->512 and
    // 512->512 layers: 0.50 against 0.57 ms per MLP step); with longer K the single-CTA kernel is 5-15% faster.
    // IDOL_B200_GEMM_PAIR = 1 / 0 forces it on (for 128- or 256-token tiles) / off.
    const int forced_pair = env_int("IDOL_B200_GEMM_PAIR", -1);
    const bool q8 = w.format == kFmtQ8;  // the persistent kernels read Q8_0 tiles only
    // Large M: dequantise the window's row tiles into the dense layout (one launch, about 3 bytes of traffic per
    // weight) and run the dense persistent kernel on CTA pairs: its MMA thread no longer shares the SM with eight
    // dequantising warps and their per-stage barrier traffic, and a 256 x 256 tile per pair halves the token bytes
    // each CTA loads. Measured on B200 against the fused kernels (CUDA graphs, operands in HBM): 16384 x 1024 x 3072
    // 113 -> 87 us, 16384 x 1024 x 4096 147 -> 111, 16384 x 4096 x 1024 126 -> 107, 4096 x 1024 x 3072 36 -> 31; the
    // denoiser block's QKV 214 -> 162, ff1 301 -> 230, ff2 264 -> 227 (32768 tokens); the Gaussian MLP's 512 -> 512
    // layer 210 -> 181. Where the pairs' tiles do not fill the SM pairs once (4096 x 4096 x 1024: 64 tiles for 74
    // pairs) the fused kernel's split K stays faster (33 against 35 us), and a window of one 128-row tile (N = 14)
    // runs the dense kernel on one CTA (56 -> 52 us; a pair would leave half its rows empty: 72). IDOL_B200_GEMM_DENSE
    // = 0 / 2 forces it off / on for every M > 16.
    bool dense = false;
    const int dense_mode = env_int("IDOL_B200_GEMM_DENSE", 1);
    const int dense_units = (c.n_offset + c.n - p.row_begin + 2 * kRowsPerTile - 1) / (2 * kRowsPerTile);
    const bool dense_fills = (long long)dense_units * ((c.m + 255) / 256) >= num_sms(w.device) / 2;
    if (q8 && (dense_mode == 2 || (dense_mode == 1 && c.m >= kDenseMinM && dense_fills))) {
        void* scratch = dense_scratch(w.device, c.stream,
                                      (size_t)p.row_tiles * p.layout_stages * (size_t)kDenseChunkBytes);
        if (scratch) {
            const int t_first = p.row_begin / kRowsPerTile;
            const long long chunk0 = (long long)t_first * p.layout_stages;
            const unsigned grid = (unsigned)((long long)tiles_n * p.layout_stages);
            uint8_t* dense_tiles = static_cast<uint8_t*>(scratch);
            if (c.x_dtype == IDOL_BF16)
                q8_dense_tiles_kernel<true><<<grid, 128, 0, c.stream>>>(w.tiles + chunk0 * kChunkBytes,
                                                                       dense_tiles + chunk0 * kDenseChunkBytes);
            else
                q8_dense_tiles_kernel<false><<<grid, 128, 0, c.stream>>>(w.tiles + chunk0 * kChunkBytes,
                                                                        dense_tiles + chunk0 * kDenseChunkBytes);
            IDOL_CUDA(cudaGetLastError());
            p.tiles = dense_tiles;
            dense = true;
        }
    }
    const bool pair = !dense && q8 && bn >= 128 && (forced_pair == 1 ||
                                    (forced_pair != 0 && p.stages_total <= 8 && c.n >= 256 && c.m >= 4096));
    // The persistent single-CTA kernel (192-token tiles, double-buffered accumulator, a 2-byte output leaving
    // through a staging tile and TMA stores): measured on B200 it pays at K <= 1024 once the 192-token tiles number
    // 4.5 or more per SM (M = 16384, K = 1024: 864 -> 910 TFLOP/s at N = 3072, 900 -> 930 at N = 4096; 4096 x 1024 x
    // 4096, 4.75 tiles per SM: 736 -> 770; 4096 x 1024 x 3072, 3.6 per SM: 711 -> 681, so not there). An fp32
    // output (the residual-stream projections) leaves it by direct stores and pays from four tiles per SM, since its
    // epilogue's reads and writes of the fp32 stream then run under the next tile's main loop (16384 x 1024 x 1024
    // with the residual: 81.6 -> 69.8 us); 2-byte direct stores, fewer tiles or longer K (16384 x 4096 x 1024 with
    // the residual: 155 -> 158 us) keep the non-persistent kernel. IDOL_B200_GEMM_PERSIST = 1 / 0 forces it on / off.
    const bool staged = staged_output_ok(c);
    const int forced_persist = env_int("IDOL_B200_GEMM_PERSIST", -1);
    const long long tiles192 = (long long)tiles_n * ((c.m + 191) / 192);
    const bool persist1 = !dense && q8 && !pair && bn >= 256 &&
                          (forced_persist == 1 ||
                           (forced_persist != 0 && (staged || c.y_dtype == IDOL_F32) && p.stages_total <= 16 &&
                            2 * tiles192 >= (staged ? 9LL : 8LL) * num_sms(w.device)));
    if (dense || pair || persist1) {
        // The dense path runs on CTA pairs (kind 3), on one CTA (kind 2) for a window of one 128-row tile or with
        // IDOL_B200_GEMM_DENSE_PAIR = 0.
        const int kind = dense ? (tiles_n > 1 && env_int("IDOL_B200_GEMM_DENSE_PAIR", 1) != 0 ? 3 : 2)
                               : pair ? 0 : 1;
        const bool two = kind == 0 || kind == 3;  // CTA pairs
        // Two accumulators fit TMEM: beside the A slots (192 or 128 tokens), or alone (dense pair: 256).
        const int pbn = kind == 3 ? 256 : kind != 0 ? 192 : bn >= 256 ? 192 : 128;
        const int unit_rows = two ? 2 * kRowsPerTile : kRowsPerTile;
        p.stages_per_split = p.stages_total;
        const int units = (c.n_offset + c.n - p.row_begin + unit_rows - 1) / unit_rows;
        const int tiles_m = (int)((c.m + pbn - 1) / pbn);
        if ((long long)units * tiles_m > 0x7fffffffLL)
            return fail(IDOL_ERR_INVALID, "q8_gemm: m too large for one launch (split the batch)");
        CUtensorMap xmap;
        const int rc = encode_tmap_2d(&xmap, c.x_dtype == IDOL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                      c.x, (uint64_t)w.k, (uint64_t)c.m, (uint64_t)c.ldx * 2, kStageK,
                                      two ? pbn / 2 : pbn, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc != IDOL_OK) return rc;
        // The dense pair's weight tiles: the dense layout as rows of 64 values (128 bytes), one 128-row box per
        // (row tile, stage), no swizzle (the layout holds it already).
        CUtensorMap wmap = xmap;
        if (kind == 3) {
            const int wrc = encode_tmap_2d(&wmap, c.x_dtype == IDOL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                           p.tiles, (uint64_t)kStageK,
                                           (uint64_t)p.row_tiles * p.layout_stages * kRowsPerTile, kStageK * 2,
                                           kStageK, kRowsPerTile, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (wrc != IDOL_OK) return wrc;
        }
        // The output tensor map of the staged epilogue (one CTA, 2-byte output): the window [c.n features x M
        // tokens], one 128 x 192 box per tile. A TMA store needs a 16-byte aligned base and row stride, and an x
        // coordinate (tile start - n_offset) that is a non-negative multiple of 8 elements: windows that start on
        // a 128-row tile.
        CUtensorMap ymap = xmap;
        p.y_tma = 0;
        if (kind != 0 && staged) {
            if (encode_tmap_2d(&ymap, c.y_dtype == IDOL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                               c.y, (uint64_t)c.n, (uint64_t)c.m, (uint64_t)c.ldy * 2, kRowsPerTile, pbn,
                               CU_TENSOR_MAP_SWIZZLE_NONE) == IDOL_OK)
                p.y_tma = 1;
            else
                ymap = xmap;
        }
        if (head_norm_fused && p.y_tma && c.y_dtype == IDOL_BF16) {
            p.hn_gamma_a = c.head_gamma_a;
            p.hn_gamma_b = c.head_gamma_b;
            p.hn_cols = c.head_cols;
            p.hn_split = c.head_split;
            *head_norm_fused = true;
        }
        const bool bf16 = c.x_dtype == IDOL_BF16;
        const cudaStream_t st = c.stream;
        if (c.y_dtype == IDOL_F32)
            return bf16 ? dispatch_persistent<true, float>(kind, pbn, xmap, ymap, wmap, p, units, tiles_m, st)
                        : dispatch_persistent<false, float>(kind, pbn, xmap, ymap, wmap, p, units, tiles_m, st);
        if (c.y_dtype == IDOL_BF16)
            return bf16 ? dispatch_persistent<true, __nv_bfloat16>(kind, pbn, xmap, ymap, wmap, p, units, tiles_m, st)
                        : dispatch_persistent<false, __nv_bfloat16>(kind, pbn, xmap, ymap, wmap, p, units, tiles_m, st);
        return bf16 ? dispatch_persistent<true, __half>(kind, pbn, xmap, ymap, wmap, p, units, tiles_m, st)
                    : dispatch_persistent<false, __half>(kind, pbn, xmap, ymap, wmap, p, units, tiles_m, st);
    }
    p.stages_per_split = (p.stages_total + splits - 1) / splits;
    splits = (p.stages_total + p.stages_per_split - 1) / p.stages_per_split;  // every split gets >= 1 stage
    const int tiles_m = (int)((c.m + bn - 1) / bn);
    if (tiles_m > 65535) return fail(IDOL_ERR_INVALID, "q8_gemm: m too large for one launch (split the batch)");

    CUtensorMap xmap;
    const int rc = encode_tmap_2d(&xmap, c.x_dtype == IDOL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                  c.x, (uint64_t)w.k, (uint64_t)c.m, (uint64_t)c.ldx * 2, kStageK, bn,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != IDOL_OK) return rc;

    const bool bf16 = c.x_dtype == IDOL_BF16;
    if (c.y_dtype == IDOL_F32)
        return bf16 ? dispatch<true, float>(w.format, bn, xmap, p, tiles_n, tiles_m, splits, c.stream)
                    : dispatch<false, float>(w.format, bn, xmap, p, tiles_n, tiles_m, splits, c.stream);
    if (c.y_dtype == IDOL_BF16)
        return bf16 ? dispatch<true, __nv_bfloat16>(w.format, bn, xmap, p, tiles_n, tiles_m, splits, c.stream)
                    : dispatch<false, __nv_bfloat16>(w.format, bn, xmap, p, tiles_n, tiles_m, splits, c.stream);
    return bf16 ? dispatch<true, __half>(w.format, bn, xmap, p, tiles_n, tiles_m, splits, c.stream)
                : dispatch<false, __half>(w.format, bn, xmap, p, tiles_n, tiles_m, splits, c.stream);
}

int q8_gemm(const GemmCall& c) {
    if (c.head_cols <= 0) return q8_gemm_impl(c, nullptr);
    if (c.y_dtype != IDOL_BF16 || c.n_offset != 0 || c.act != IDOL_ACT_NONE || c.residual || c.head_cols % 64 ||
        c.head_split % 64 || c.head_split > c.head_cols || c.head_cols > c.n || !c.head_gamma_a ||
        (c.head_split < c.head_cols && !c.head_gamma_b))
        return fail(IDOL_ERR_INVALID, "q8_gemm: per-head norm wants a bf16 output from column 0 without activation or "
                                      "residual, whole 64-wide heads and its gammas");
    // Fused only when the normalised columns are whole 128-row tiles of the staged epilogue.
    bool fused = false;
    const int rc = q8_gemm_impl(c, c.head_cols % 128 == 0 ? &fused : nullptr);
    if (rc != IDOL_OK || fused || c.m == 0) return rc;
    // The GEMM left through direct stores: the norm runs as its own launch on the stored rows.
    if (c.head_split * 2 == c.head_cols)
        IDOL_CUDA(launch_rms_heads_qk(c.y, c.ldy, c.m, c.head_split / 64, c.head_gamma_a, c.head_gamma_b, c.stream));
    else {
        if (c.head_split > 0)
            IDOL_CUDA(launch_rms_heads(c.y, IDOL_BF16, c.ldy, c.m, c.head_split / 64, c.head_gamma_a, c.stream));
        if (c.head_cols > c.head_split)
            IDOL_CUDA(launch_rms_heads(static_cast<__nv_bfloat16*>(c.y) + c.head_split, IDOL_BF16, c.ldy, c.m,
                                       (c.head_cols - c.head_split) / 64, c.head_gamma_b, c.stream));
    }
    return IDOL_OK;
}

}  // namespace idol
