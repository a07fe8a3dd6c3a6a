// attention.cu - multi-head scaled dot-product attention on sm_100a tensor cores (head dim 64).
//
// Replaces src/kernels.cpp:629-746 attention / attention_blocked: per head, softmax(q k^T / sqrt(hd)) v over full rows,
// with q rows ldq apart and k/v rows ldkv apart (k and v may be column offsets of one packed buffer, as the decoders
// pass qkv, kv and kv + D). The reference materialises a full score row per query; this kernel streams keys in blocks
// of 128 with an online softmax, so nothing of size L x L exists anywhere.
//
// One CTA per (128 queries, head, image). Warp roles:
//   warp 0      : TMA producer - the Q tile once, then K and V tiles of 128 keys into a 3-stage ring;
//   warp 1      : TMEM owner and MMA issuer - S_j = Q K_j^T (tcgen05 SS, fp32 in TMEM, double-buffered), then
//                 O_j = P_j V_j (tcgen05 TS: P_j bf16 read from TMEM as the A operand, V_j from shared memory as an
//                 MN-major B operand) into a double-buffered partial-output region of TMEM;
//   warps 2-5   : softmax - thread r owns query row r (= TMEM lane r): reads its S row, updates the running max and
//                 sum, writes P_j (bf16) to TMEM, and folds each partial O_j into a register accumulator with the
//                 exp2(m_old - m_new) correction; at the end divides by the sum and stores bf16.
// The same 128-byte-swizzled K/V tile layout serves as the K-major B operand of Q K^T and the MN-major B operand of
// P V. Every wait is bounded (ptx.cuh); a timeout raises the sticky device error and the CTA winds down.
#include <cuda_bf16.h>

#include "internal.h"
#include "ptx.cuh"

namespace idol {

IDOL_DEVICE_ERROR_READER(take_device_error_attention)

namespace {

constexpr int kQTile = 128;    // queries per CTA (TMEM lanes)
constexpr int kKTile = 128;    // keys per block
constexpr int kHd = 64;        // head dim (128 bytes of bf16: one swizzle row)
constexpr int kStages = 3;     // K/V ring
constexpr int kThreads = 192;
constexpr int kTileBytes = kKTile * kHd * 2;  // 16 KB (Q tile has the same size)
// TMEM columns: S[0] 0-127, S[1] 128-255, P[0] 256-319, P[1] 320-383, O[0] 384-447, O[1] 448-511.
constexpr uint32_t kColS = 0, kColP = 256, kColO = 384;
constexpr int kTmemCols = 512;
constexpr int kSmemBytes = 1024 + kTileBytes * (1 + 2 * kStages) + 256;
// Pad to keep one CTA per SM: the TMEM allocation takes all 512 columns.
constexpr int kSmemLaunch = kSmemBytes < 120 * 1024 ? 120 * 1024 : kSmemBytes;

struct AttnParams {
    void* out;
    long long ldo;              // output row stride (elements)
    long long out_img_stride;   // rows of one image in the output = lq
    int lq, lk, heads;
    float scale_log2;           // log2(e) / sqrt(hd)
};

// Shared-memory descriptor for an MN-major operand stored as 128-byte-swizzled rows of 64 bf16 (the N extent), one
// row per k: 8 rows form a 1024-byte atom and atoms follow each other along k (stride byte offset 1024).
__device__ __forceinline__ uint64_t make_sdesc_sw128_mn(uint32_t start) {
    uint64_t d = 0;
    d |= (uint64_t)((start & 0x3FFFFu) >> 4);
    d |= (uint64_t)(8192 >> 4) << 16;     // leading byte offset: next 64-wide N atom (unused for N = 64)
    d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset: next 8-row group along k
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// 2^x by the hardware's approximate base-2 exponential (relative error near 2^-22, far below the bf16 rounding P gets
// next); -inf gives +0.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap, const AttnParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* qs = smem;
    uint8_t* ks = qs + kTileBytes;
    uint8_t* vs = ks + kStages * kTileBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(vs + kStages * kTileBytes);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;                 // [kStages]
    uint64_t* kv_empty = kv_full + kStages;       // [kStages]
    uint64_t* s_full = kv_empty + kStages;        // [2]
    uint64_t* p_full = s_full + 2;                // [2]
    uint64_t* o_full = p_full + 2;                // [2]
    uint64_t* o_free = o_full + 2;                // [2]
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(o_free + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int q0 = blockIdx.x * kQTile;
    const int h = blockIdx.y;
    const int img = blockIdx.z;
    const int nb = (p.lk + kKTile - 1) / kKTile;

    if (tid == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 4);  // one elected arrival per softmax warp
            mbar_init(&o_full[b], 1);
            mbar_init(&o_free[b], 4);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&qmap);
            prefetch_tmap(&kmap);
            prefetch_tmap(&vmap);
            mbar_arrive_expect_tx(q_full, kTileBytes);
            tma_load_3d(qs, &qmap, h * kHd, q0, img, q_full);
            int issued = 0;
            for (int j = 0; j < nb; ++j) {
                const int s = j % kStages, u = j / kStages;
                if (j >= kStages && !mbar_wait(&kv_empty[s], (u - 1) & 1, abort_flag)) break;
                mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
                tma_load_3d(ks + s * kTileBytes, &kmap, h * kHd, j * kKTile, img, &kv_full[s]);
                tma_load_3d(vs + s * kTileBytes, &vmap, h * kHd, j * kKTile, img, &kv_full[s]);
                ++issued;
            }
            // Every copy this CTA issued has landed before it can leave (see mbar_drain).
            mbar_drain(q_full, 0);
            for (int j = issued - kStages > 0 ? issued - kStages : 0; j < issued; ++j)
                mbar_drain(&kv_full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc_qk = make_idesc_f16(kQTile, kKTile, true);
            const uint32_t idesc_pv = make_idesc_f16(kQTile, kHd, true) | (1u << 16);  // B (V) is MN-major
            bool ok = mbar_wait(q_full, 0, abort_flag);
            const uint32_t qaddr = smem_u32(qs);
            for (int j = 0; ok && j <= nb; ++j) {
                if (j < nb) {
                    const int s = j % kStages, b = j % 2;
                    // S buffer b was last read by the softmax of block j - 2, which had finished (p_full) before
                    // P V of block j - 2 was issued in the previous iteration.
                    if (!mbar_wait(&kv_full[s], (j / kStages) & 1, abort_flag)) break;
                    tc_fence_after();
                    const uint32_t kaddr = smem_u32(ks + s * kTileBytes);
#pragma unroll
                    for (int kk = 0; kk < kHd / 16; ++kk)
                        mma_ss(tmem + kColS + b * kKTile, make_sdesc_sw128(qaddr + kk * 32),
                               make_sdesc_sw128(kaddr + kk * 32), idesc_qk, kk > 0 ? 1u : 0u);
                    mma_commit(&s_full[b]);
                }
                if (j >= 1) {
                    const int jp = j - 1, bp = jp % 2, sp = jp % kStages;
                    if (!mbar_wait(&p_full[bp], (jp / 2) & 1, abort_flag)) break;
                    if (jp >= 2 && !mbar_wait(&o_free[bp], ((jp - 2) / 2) & 1, abort_flag)) break;
                    tc_fence_after();
                    const uint32_t vaddr = smem_u32(vs + sp * kTileBytes);
#pragma unroll
                    for (int kk = 0; kk < kKTile / 16; ++kk)
                        mma_ts(tmem + kColO + bp * kHd, tmem + kColP + bp * (kKTile / 2) + kk * 8,
                               make_sdesc_sw128_mn(vaddr + kk * 2048), idesc_pv, kk > 0 ? 1u : 0u);
                    mma_commit(&o_full[bp]);
                    mma_commit(&kv_empty[sp]);
                }
            }
        }
    } else {
        // Softmax warpgroup: warp w reads TMEM lanes [32 (w % 4), +32); thread = query row.
        const int q = warp % 4;
        const int r = 32 * q + lane;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        float o_acc[kHd];
#pragma unroll
        for (int c = 0; c < kHd; ++c) o_acc[c] = 0.0f;
        float m_run = -INFINITY;   // running max (log2 domain) after the latest block
        float m_acc = -INFINITY;   // the max o_acc is scaled to
        float m_prev_blk = -INFINITY;
        float l_run = 0.0f;
        bool ok = true;

        auto fold = [&](int jo) {
            // O_jo = P_jo V_jo is in TMEM buffer jo % 2, scaled to m of block jo (passed in m_prev_blk).
            const int bo = jo % 2;
            bool got = mbar_wait(&o_full[bo], (jo / 2) & 1, abort_flag);
            if (!__all_sync(0xffffffffu, got)) return false;
            tc_fence_after();
            const float f = (m_acc == -INFINITY) ? 0.0f : ex2(m_acc - m_prev_blk);
#pragma unroll
            for (int c0 = 0; c0 < kHd; c0 += 32) {  // two halves of 32 columns, one wait each
                uint32_t v[32];
                tmem_ld16(tmem + lane_base + kColO + bo * kHd + c0, *reinterpret_cast<uint32_t(*)[16]>(v));
                tmem_ld16(tmem + lane_base + kColO + bo * kHd + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
                tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < 32; ++c) o_acc[c0 + c] = fmaf(o_acc[c0 + c], f, __uint_as_float(v[c]));
            }
            m_acc = m_prev_blk;
            tc_fence_before();
            __syncwarp();  // the warp's TMEM reads are done and fenced before lane 0 reports it
            if (lane == 0) mbar_arrive(&o_free[bo]);
            return true;
        };

        for (int j = 0; j < nb && ok; ++j) {
            const int b = j % 2;
            bool got = mbar_wait(&s_full[b], (j / 2) & 1, abort_flag);
            if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
            tc_fence_after();
            const int valid = p.lk - j * kKTile;  // keys of this block that exist
            const uint32_t s_col = kColS + b * kKTile;
            // The whole score row in registers: eight asynchronous 16-column loads, one wait.
            uint32_t sv[kKTile];
#pragma unroll
            for (int c0 = 0; c0 < kKTile; c0 += 16)
                tmem_ld16(tmem + lane_base + s_col + c0, *reinterpret_cast<uint32_t(*)[16]>(sv + c0));
            tmem_ld_wait();
            // Row maximum of the raw scores (the scale is positive, so it commutes with the max), as four independent
            // chains. Keys past the end exist only in the last block.
            const bool full = valid >= kKTile;
            if (!full) {
#pragma unroll
                for (int c = 0; c < kKTile; ++c)
                    if (c >= valid) sv[c] = __float_as_uint(-INFINITY);
            }
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < kKTile; ++c) m4[c % 4] = fmaxf(m4[c % 4], __uint_as_float(sv[c]));
            const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            const float m_new = fmaxf(m_run, mx * p.scale_log2);
            const float alpha = (m_run == -INFINITY) ? 0.0f : ex2(m_run - m_new);
            const float neg_m = -m_new;
            // P_j goes to TMEM buffer b once P V of block j - 2 (which read that buffer) has completed.
            if (j >= 2) {
                got = mbar_wait(&o_full[b], ((j - 2) / 2) & 1, abort_flag);
                if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                tc_fence_after();
            }
            // p = exp2(s scale - m) on key pairs (packed FMA), summed in four independent pairs of partial sums,
            // packed to bf16 and stored 32 keys at a time (masked keys give exp2(-inf) = 0).
            const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
            const float2 nm2 = make_float2(neg_m, neg_m);
            float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};
#pragma unroll
            for (int c0 = 0; c0 < kKTile; c0 += 32) {
                uint32_t pk[16];
#pragma unroll
                for (int c = 0; c < 32; c += 2) {
                    const float2 t = __ffma2_rn(make_float2(__uint_as_float(sv[c0 + c]), __uint_as_float(sv[c0 + c + 1])),
                                                sc2, nm2);
                    const float2 e = make_float2(ex2(t.x), ex2(t.y));
                    sum2[(c / 2) % 4] = __fadd2_rn(sum2[(c / 2) % 4], e);
                    pk[c / 2] = pack_bf16x2(e.x, e.y);
                }
                tmem_st16(tmem + lane_base + kColP + b * (kKTile / 2) + c0 / 2, pk);
            }
            const float2 s01 = __fadd2_rn(sum2[0], sum2[1]), s23 = __fadd2_rn(sum2[2], sum2[3]);
            const float2 s4 = __fadd2_rn(s01, s23);
            const float sum = s4.x + s4.y;
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();  // the warp's P stores (and S reads) are complete and fenced before lane 0 reports it
            if (lane == 0) mbar_arrive(&p_full[b]);
            l_run = l_run * alpha + sum;
            m_run = m_new;
            // Fold the partial output of the previous block (its max is m_prev_blk).
            if (j >= 1 && !fold(j - 1)) { ok = false; break; }
            m_prev_blk = m_new;
        }
        if (ok && nb >= 1) ok = fold(nb - 1);

        // Store: row r of this tile, head h, 64 bf16 = 128 contiguous bytes.
        const int qrow = q0 + r;
        if (ok && qrow < p.lq) {
            const float inv = 1.0f / l_run;
            __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) +
                               ((long long)img * p.out_img_stride + qrow) * p.ldo + (long long)h * kHd;
#pragma unroll
            for (int c0 = 0; c0 < kHd; c0 += 8) {
                uint4 pkt;
                pkt.x = pack_bf16x2(o_acc[c0 + 0] * inv, o_acc[c0 + 1] * inv);
                pkt.y = pack_bf16x2(o_acc[c0 + 2] * inv, o_acc[c0 + 3] * inv);
                pkt.z = pack_bf16x2(o_acc[c0 + 4] * inv, o_acc[c0 + 5] * inv);
                pkt.w = pack_bf16x2(o_acc[c0 + 6] * inv, o_acc[c0 + 7] * inv);
                *reinterpret_cast<uint4*>(o + c0) = pkt;
            }
        }
        tc_fence_before();
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// 3-D map over [images][rows][cols] bf16: rows `row_stride` elements apart, images `img_rows` rows apart; boxes of
// 64 columns x 128 rows x 1 image with the 128-byte swizzle. Rows past `rows` inside an image read as zeros.
int encode_tmap_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t images,
                   uint64_t row_stride, uint64_t img_rows) {
    static_assert(kQTile == kKTile, "one box shape for Q, K and V");
    const cuuint64_t dims[3] = {cols, rows, images};
    const cuuint64_t strides[2] = {row_stride * 2, img_rows * row_stride * 2};
    const cuuint32_t box[3] = {kHd, kKTile, 1};
    return encode_tmap_nd(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

int attention(const AttentionCall& c) {
    if (c.head_dim != kHd) return fail(IDOL_ERR_UNSUPPORTED, "attention: only head_dim 64 is implemented");
    if (c.lq < 0 || c.lk < 1 || c.heads < 1 || c.batch < 1) return fail(IDOL_ERR_INVALID, "attention: sizes");
    if (c.lq == 0) return IDOL_OK;
    const long long dim = (long long)c.heads * kHd;
    if (c.ldq < dim || c.ldkv < dim || c.ldo < dim || c.ldq % 8 || c.ldkv % 8 || c.ldo % 8)
        return fail(IDOL_ERR_INVALID, "attention: row strides must cover heads * 64 and be multiples of 8");
    for (const void* ptr : {c.q, c.k, c.v, static_cast<const void*>(c.out)})
        if (!ptr || reinterpret_cast<uintptr_t>(ptr) % 16)
            return fail(IDOL_ERR_INVALID, "attention: q, k, v and out must be 16-byte aligned device pointers");
    if ((c.lq + kQTile - 1) / kQTile > 0x7fffffff || c.heads > 65535 || c.batch > 65535)
        return fail(IDOL_ERR_INVALID, "attention: grid too large");

    CUtensorMap qm, km, vm;
    int rc = encode_tmap_3d(&qm, c.q, (uint64_t)dim, (uint64_t)c.lq, (uint64_t)c.batch, (uint64_t)c.ldq,
                            (uint64_t)c.lq);
    if (rc == IDOL_OK)
        rc = encode_tmap_3d(&km, c.k, (uint64_t)dim, (uint64_t)c.lk, (uint64_t)c.batch, (uint64_t)c.ldkv,
                            (uint64_t)c.lk);
    if (rc == IDOL_OK)
        rc = encode_tmap_3d(&vm, c.v, (uint64_t)dim, (uint64_t)c.lk, (uint64_t)c.batch, (uint64_t)c.ldkv,
                            (uint64_t)c.lk);
    if (rc != IDOL_OK) return rc;

    AttnParams p;
    p.out = c.out;
    p.ldo = c.ldo;
    p.out_img_stride = c.lq;
    p.lq = (int)c.lq;
    p.lk = (int)c.lk;
    p.heads = c.heads;
    p.scale_log2 = 1.4426950408889634f / sqrtf((float)kHd);

    static unsigned long long configured = 0;
    int dev = 0;
    IDOL_CUDA(cudaGetDevice(&dev));
    if (!(configured >> (dev & 63) & 1ull)) {
        IDOL_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLaunch));
        configured |= 1ull << (dev & 63);
    }
    const dim3 grid((unsigned)((c.lq + kQTile - 1) / kQTile), (unsigned)c.heads, (unsigned)c.batch);
    attention_kernel<<<grid, kThreads, kSmemLaunch, c.stream>>>(qm, km, vm, p);
    IDOL_CUDA(cudaGetLastError());
    return IDOL_OK;
}

}  // namespace idol
