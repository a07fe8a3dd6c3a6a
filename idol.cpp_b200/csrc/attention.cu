// attention.cu - multi-head scaled dot-product attention on sm_100a tensor cores (head dim 64).
//
// Replaces src/kernels.cpp:629-746 attention / attention_blocked: per head, softmax(q k^T / sqrt(hd)) v over full rows,
// with q rows ldq apart and k/v rows ldkv apart (k and v may be column offsets of one packed buffer, as the decoders
// pass qkv, kv and kv + D). The reference materialises a full score row per query; this kernel streams keys in blocks
// of 128 with an online softmax, so nothing of size L x L exists anywhere.
//
// One CTA per (256 queries = two query tiles t of 128, head, image). Warp roles:
//   warp 0      : TMA producer - both Q tiles once, then K and V tiles of 128 keys into a 3-stage ring (each K/V
//                 tile serves both query tiles);
//   warp 1      : TMEM owner and MMA issuer - S_t,j = Q_t K_j^T (tcgen05 SS, fp32 in TMEM), then
//                 O_t += P_t,j V_j (tcgen05 TS: P_t,j bf16 read from TMEM as the A operand, V_j from shared memory as
//                 an MN-major B operand, fp32 O_t accumulated in TMEM); it interleaves the two tiles so that one
//                 tile's softmax runs while the tensor pipe works for the other;
//   warps 2-5 / 6-9 : the softmax warpgroups of tiles 0 / 1 - thread r owns query row r of its tile (= TMEM lane r):
//                 loads its S row (then frees the S buffer), updates the running max and sum, writes P (bf16) to TMEM;
//                 O and the sum are rescaled only when the row maximum grows by more than 2^8 over the one in use
//                 (P stays <= 256, exact in bf16 range, and the final O / sum cancels the stale maximum), so O stays
//                 in TMEM with no per-block fold; at the end the row is divided by its sum and stored as bf16 (or fp32).
// The same 128-byte-swizzled K/V tile layout serves as the K-major B operand of Q K^T and the MN-major B operand of
// P V. Every wait is bounded (ptx.cuh); a timeout raises the sticky device error and the CTA winds down. The waits
// use the plain try_wait, without a suspend-time hint: the kernel's pace is set by the hand-offs between the MMA
// thread and the softmax warps, and the hinted form's later wake-up measured 4% slower (3% from the MMA thread alone).
#include <cuda_bf16.h>

#include "internal.h"
#include "ptx.cuh"

namespace idol {

IDOL_DEVICE_ERROR_READER(take_device_error_attention)

namespace {

constexpr int kQTile = 128;    // queries per query tile (TMEM lanes)
constexpr int kQTiles = 2;     // query tiles per CTA, one softmax warpgroup each
constexpr int kKTile = 128;    // keys per block
constexpr int kHd = 64;        // head dim (128 bytes of bf16: one swizzle row)
constexpr int kStages = 3;     // K/V ring
constexpr int kThreads = 64 + 128 * kQTiles;  // producer warp, MMA warp, four softmax warps per query tile
constexpr int kTileBytes = kKTile * kHd * 2;  // 16 KB (a Q tile has the same size)
// TMEM columns of query tile t: S at 256 t + 0..127, P (bf16 pairs) at 256 t + 128..191, O at 256 t + 192..255.
constexpr uint32_t kColS = 0, kColP = 128, kColO = 192, kColTile = 256;
constexpr int kTmemCols = 512;
constexpr int kSmemBytes = 1024 + kTileBytes * (kQTiles + 2 * kStages) + 256;
// Pad to keep one CTA per SM: the TMEM allocation takes all 512 columns.
constexpr int kSmemLaunch = kSmemBytes < 120 * 1024 ? 120 * 1024 : kSmemBytes;
constexpr float kRescaleLog2 = 8.0f;  // rescale O and the sum once the row max exceeds the one in use by 2^8

struct AttnParams {
    void* out;
    long long ldo;              // output row stride (elements)
    int out_f32;                // 1: fp32 output rows, 0: bf16
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

// 32 lanes x 32 bits, 128 consecutive columns in one load (one instruction for a whole score row).
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&r)[128]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
                 : "r"(taddr));
}

// 32 lanes x 32 bits, 64 consecutive columns written in one store.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&r)[64]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
                 : "memory");
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100): halves the row-maximum pass.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Ten warps leave three on two of the four schedulers, whose register files hold 16K registers each: at most 168 per
// thread (ptxas holds the score row in 156, with no spill, since the row is read by one 128-column load).
__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap, const AttnParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* qs = smem;                                   // [kQTiles] Q tiles
    uint8_t* ks = qs + kQTiles * kTileBytes;
    uint8_t* vs = ks + kStages * kTileBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(vs + kStages * kTileBytes);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;                 // [kStages]
    uint64_t* kv_empty = kv_full + kStages;       // [kStages]
    uint64_t* s_full = kv_empty + kStages;        // [kQTiles] S_t,j is in TMEM
    uint64_t* s_free = s_full + kQTiles;          // [kQTiles] the softmax of tile t has read S_t,j
    uint64_t* p_full = s_free + kQTiles;          // [kQTiles] P_t,j is in TMEM (O_t rescaled if it had to be)
    uint64_t* o_full = p_full + kQTiles;          // [kQTiles] O_t += P_t,j V_j has completed
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(o_full + kQTiles);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int q0 = blockIdx.x * (kQTile * kQTiles);
    const int h = blockIdx.y;
    const int img = blockIdx.z;
    const int nb = (p.lk + kKTile - 1) / kKTile;

    if (tid == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int t = 0; t < kQTiles; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&s_free[t], 4);  // one elected arrival per softmax warp of the tile
            mbar_init(&p_full[t], 4);
            mbar_init(&o_full[t], 1);
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
            mbar_arrive_expect_tx(q_full, kQTiles * kTileBytes);
            for (int t = 0; t < kQTiles; ++t)
                tma_load_3d(qs + t * kTileBytes, &qmap, h * kHd, q0 + t * kQTile, img, q_full);
            int issued = 0;
            for (int j = 0; j < nb; ++j) {
                const int s = j % kStages, u = j / kStages;
                if (j >= kStages && !mbar_wait<false>(&kv_empty[s], (u - 1) & 1, abort_flag)) break;
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
            // S_t,j = Q_t K_j^T into tile t's S columns.
            auto issue_s = [&](int t, int j) {
                const uint32_t qaddr = smem_u32(qs + t * kTileBytes);
                const uint32_t kaddr = smem_u32(ks + (j % kStages) * kTileBytes);
#pragma unroll
                for (int kk = 0; kk < kHd / 16; ++kk)
                    mma_ss(tmem + t * kColTile + kColS, make_sdesc_sw128(qaddr + kk * 32),
                           make_sdesc_sw128(kaddr + kk * 32), idesc_qk, kk > 0 ? 1u : 0u);
                mma_commit(&s_full[t]);
            };
            // O_t (+)= P_t,j V_j (the first block overwrites O_t).
            auto issue_pv = [&](int t, int j) {
                const uint32_t vaddr = smem_u32(vs + (j % kStages) * kTileBytes);
#pragma unroll
                for (int kk = 0; kk < kKTile / 16; ++kk)
                    mma_ts(tmem + t * kColTile + kColO, tmem + t * kColTile + kColP + kk * 8,
                           make_sdesc_sw128_mn(vaddr + kk * 2048), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&o_full[t]);
            };
            bool ok = mbar_wait<false>(q_full, 0, abort_flag) && mbar_wait<false>(&kv_full[0], 0, abort_flag);
            if (ok) {
                tc_fence_after();
                for (int t = 0; t < kQTiles; ++t) issue_s(t, 0);
            }
            // Block j: per tile, S of block j + 1 (once the softmax has read S of block j) then P V of block j (once P
            // is written); the K/V stage of block j is released after both tiles' P V.
            for (int j = 0; ok && j < nb; ++j) {
                for (int t = 0; t < kQTiles && ok; ++t) {
                    if (j + 1 < nb) {
                        if (t == 0 && !mbar_wait<false>(&kv_full[(j + 1) % kStages], ((j + 1) / kStages) & 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        if (!mbar_wait<false>(&s_free[t], j & 1, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        issue_s(t, j + 1);
                    }
                    if (!mbar_wait<false>(&p_full[t], j & 1, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    issue_pv(t, j);
                }
                if (ok) mma_commit(&kv_empty[j % kStages]);
            }
        }
    } else {
        // Softmax warpgroup t: warp w reads TMEM lanes [32 (w % 4), +32) of tile t; thread = query row.
        const int t = (warp - 2) / 4;
        const int q = warp % 4;
        const int r = 32 * q + lane;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const uint32_t tt = tmem + lane_base + (uint32_t)(t * kColTile);
        float m_used = -INFINITY;  // the maximum (log2 domain) P and O are scaled to
        float l_run = 0.0f;
        bool ok = true;
        for (int j = 0; j < nb && ok; ++j) {
            bool got = mbar_wait<false>(&s_full[t], j & 1, abort_flag);
            if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
            tc_fence_after();
            // The whole score row in registers (one 128-column load and its wait), then the S buffer is
            // free for the next block's Q K^T while this block's exponentials are computed.
            uint32_t sv[kKTile];
            tmem_ld128(tt + kColS, sv);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[t]);
            // Keys past the end exist only in the last block.
            const int valid = p.lk - j * kKTile;
            if (valid < kKTile) {
#pragma unroll
                for (int c = 0; c < kKTile; ++c)
                    if (c >= valid) sv[c] = __float_as_uint(-INFINITY);
            }
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c = 0; c < kKTile; c += 2)
                m4[(c / 2) % 4] = fmax3(m4[(c / 2) % 4], __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]));
            const float m_blk = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2;
            // Lazy rescaling: keep the maximum in use unless this block's exceeds it by more than 2^8.
            float alpha = 1.0f;
            bool rescale = false;
            if (m_used == -INFINITY) {
                m_used = m_blk;  // first block: O is written, not accumulated
            } else if (m_blk > m_used + kRescaleLog2) {
                alpha = ex2(m_used - m_blk);
                m_used = m_blk;
                rescale = true;
            }
            // p = exp2(s scale - m) on key pairs (packed FMA), summed in four independent pairs of partial sums and
            // packed to bf16 in registers (masked keys give exp2(-inf) = 0). This needs nothing from the tensor pipe,
            // so it runs while P V of block j - 1 may still be reading the P buffer.
            const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
            const float2 nm2 = make_float2(-m_used, -m_used);
            float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};
            uint32_t pk[kKTile / 2];
#pragma unroll
            for (int c = 0; c < kKTile; c += 2) {
                const float2 x2 = __ffma2_rn(make_float2(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])), sc2, nm2);
                const float2 e = make_float2(ex2(x2.x), ex2(x2.y));
                sum2[(c / 2) % 4] = __fadd2_rn(sum2[(c / 2) % 4], e);
                pk[c / 2] = pack_bf16x2(e.x, e.y);
            }
            // P_t,j and a rescaled O_t go to TMEM only after P V of block j - 1 has completed.
            if (j >= 1) {
                got = mbar_wait<false>(&o_full[t], (j - 1) & 1, abort_flag);
                if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, rescale)) {  // tcgen05.ld/st are warp-collective: alpha = 1 elsewhere
#pragma unroll
                    for (int c0 = 0; c0 < kHd; c0 += 32) {
                        uint32_t o[32];
                        tmem_ld16(tt + kColO + c0, *reinterpret_cast<uint32_t(*)[16]>(o));
                        tmem_ld16(tt + kColO + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(o + 16));
                        tmem_ld_wait();
#pragma unroll
                        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                        tmem_st16(tt + kColO + c0, *reinterpret_cast<uint32_t(*)[16]>(o));
                        tmem_st16(tt + kColO + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(o + 16));
                    }
                }
            }
            tmem_st64(tt + kColP, pk);
            const float2 s01 = __fadd2_rn(sum2[0], sum2[1]), s23 = __fadd2_rn(sum2[2], sum2[3]);
            const float2 s4 = __fadd2_rn(s01, s23);
            l_run = l_run * alpha + (s4.x + s4.y);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();  // the warp's P (and O) stores are complete and fenced before lane 0 reports it
            if (lane == 0) mbar_arrive(&p_full[t]);
        }
        // O_t after the last block, divided by the row sum; row r of tile t, head h: 128 contiguous bytes.
        if (ok && nb >= 1) {
            ok = __all_sync(0xffffffffu, mbar_wait<false>(&o_full[t], (nb - 1) & 1, abort_flag));
            if (ok) {
                tc_fence_after();
                uint32_t o[kHd];
#pragma unroll
                for (int c0 = 0; c0 < kHd; c0 += 16)
                    tmem_ld16(tt + kColO + c0, *reinterpret_cast<uint32_t(*)[16]>(o + c0));
                tmem_ld_wait();
                const int qrow = q0 + t * kQTile + r;
                if (qrow < p.lq && p.out_f32) {
                    const float inv = 1.0f / l_run;
                    float* out = static_cast<float*>(p.out) +
                                 ((long long)img * p.out_img_stride + qrow) * p.ldo + (long long)h * kHd;
#pragma unroll
                    for (int c0 = 0; c0 < kHd; c0 += 4) {
                        float4 pkt;
                        pkt.x = __uint_as_float(o[c0 + 0]) * inv;
                        pkt.y = __uint_as_float(o[c0 + 1]) * inv;
                        pkt.z = __uint_as_float(o[c0 + 2]) * inv;
                        pkt.w = __uint_as_float(o[c0 + 3]) * inv;
                        *reinterpret_cast<float4*>(out + c0) = pkt;
                    }
                } else if (qrow < p.lq) {
                    const float inv = 1.0f / l_run;
                    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) +
                                         ((long long)img * p.out_img_stride + qrow) * p.ldo + (long long)h * kHd;
#pragma unroll
                    for (int c0 = 0; c0 < kHd; c0 += 8) {
                        uint4 pkt;
                        pkt.x = pack_bf16x2(__uint_as_float(o[c0 + 0]) * inv, __uint_as_float(o[c0 + 1]) * inv);
                        pkt.y = pack_bf16x2(__uint_as_float(o[c0 + 2]) * inv, __uint_as_float(o[c0 + 3]) * inv);
                        pkt.z = pack_bf16x2(__uint_as_float(o[c0 + 4]) * inv, __uint_as_float(o[c0 + 5]) * inv);
                        pkt.w = pack_bf16x2(__uint_as_float(o[c0 + 6]) * inv, __uint_as_float(o[c0 + 7]) * inv);
                        *reinterpret_cast<uint4*>(out + c0) = pkt;
                    }
                }
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
    if ((c.lq + kQTile * kQTiles - 1) / (kQTile * kQTiles) > 0x7fffffff || c.heads > 65535 || c.batch > 65535)
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
    p.out_f32 = c.out_f32 ? 1 : 0;
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
    const dim3 grid((unsigned)((c.lq + kQTile * kQTiles - 1) / (kQTile * kQTiles)), (unsigned)c.heads,
                    (unsigned)c.batch);
    attention_kernel<<<grid, kThreads, kSmemLaunch, c.stream>>>(qm, km, vm, p);
    IDOL_CUDA(cudaGetLastError());
    return IDOL_OK;
}

}  // namespace idol
