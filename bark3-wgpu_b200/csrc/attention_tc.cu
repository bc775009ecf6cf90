// attention_tc.cu — K2: fused relative-position multi-head self-attention on
// 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// For one utterance of T frames, head h (dh = 128), query i and key j:
//   s[i, j] = (qu_i . k_j + qv_i . r_(i-j)) / sqrt(128),   p = softmax_j(s),
//   o_i = sum_j p[i, j] v_j
// where qu = q + bias_u, qv = q + bias_v and r_d is the relative-position key
// for offset d = i - j (the reference's rel_shift: BD[q, T-1-q+k], with row
// T-1-j of its position table holding position j; src/cpu/layer.rs:234-294,
// src/cpu/ops.rs:133-189, src/encoder.rs:2161-2412).  Q / K / V / R are f16
// (the reference also rounds K, V and R to f16, src/cpu/ops.rs:258-259,
// src/cpu/layer.rs:234-247); scores, softmax and O accumulate in f32.
//
// One CTA per (utterance, 128-query block, head); key blocks of 64.
//   warp 0      TMA: Qu and Qv (staging) once; per key block K, V and the
//               new rows of the R band into a 2-stage ring;
//   warp 1      TMEM owner; one thread issues the MMAs:
//                 S  = Qu K^T      M128 N64  K128  (A: Qu in shared memory)
//                 G  = Qv R_band^T M128 N192 K128  (three N64 pieces, A: Qv in TMEM)
//                 O += P V         M128 N128 K64   (A: P in TMEM, B: V MN-major)
//   warps 2..9  softmax, two warps per TMEM lane quarter: one query row per
//               lane, each warp of a pair owns 32 of the block's 64 keys (and
//               64 of O's 128 columns).  A thread reads its S columns and the
//               band columns its warp spans, adds the row's diagonal of the
//               band, and the pair exchanges row maxima through shared memory;
//               online softmax in f32 with a lazily moved reference max (O and
//               l are rescaled only when the block max exceeds it by 2^8);
//               P (f16) is written over the block's S columns.
// The band of a 128 x 64 score tile covers offsets q0-k0-63 .. q0-k0+127 (191
// R rows, loaded as 192).  Consecutive key blocks share all but 64 of them,
// so R rows live in a 256-row ring and each key block loads one 64-row chunk.
// S is double-buffered in TMEM, so the S and G MMAs of the next key block run
// while the softmax of this one is still working.
//
// The diagonal read: row i of the tile needs band column 127 - i + j for key
// j, a window whose start moves by one column per row.  TMEM loads address
// the same columns for all lanes of a warp, so each softmax thread parks its
// lane's loaded band columns in a private shared-memory row and reads the 32
// it needs back at its own offset.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b3_internal.h"
#include "b3_kernels.h"
#include "b3_ptx.cuh"

namespace b3 {

namespace {

constexpr int kBQ = 128;          // queries per CTA
constexpr int kBK = 64;           // keys per block
constexpr int kThreads = 320;     // warp 0 TMA, warp 1 MMA, warps 2..9 softmax
constexpr int kSoftThreads = 256;
constexpr int kRing = 256;        // R ring rows
constexpr int kShStride = 65;     // floats per softmax thread's diagonal row (odd: conflict-free)

// shared memory (offsets from a 1024-aligned base)
constexpr uint32_t kQuOff = 0;                   // Qu: 2 dim-halves x (128 rows x 128 B)
constexpr uint32_t kKOff = 32768;                // K: 2 stages x 2 halves x (64 rows x 128 B)
constexpr uint32_t kVOff = kKOff + 32768;        // V: same
constexpr uint32_t kROff = kVOff + 32768;        // R ring: 2 halves x (256 rows x 128 B)
constexpr uint32_t kShOff = kROff + 65536;       // diagonal rows 256 x 65 f32 (Qv staging first)
constexpr uint32_t kBarOff = kShOff + kSoftThreads * kShStride * 4;
constexpr uint32_t kSmem = kBarOff + 256 + 1024;
static_assert(kSoftThreads * kShStride * 4 >= 32768, "Qv staging fits the diagonal rows");
static_assert(kSmem <= 232448, "shared memory budget");

// TMEM columns
constexpr uint32_t kTS = 0;       // S / P, 2 buffers x 64
constexpr uint32_t kTG = 128;     // band, 192
constexpr uint32_t kTO = 320;     // O, 128
constexpr uint32_t kTQ = 448;     // Qv (A operand of the band GEMM), 64

constexpr uint32_t kIdescS = idesc_f16_f32_b<128, 64, 0>();
constexpr uint32_t kIdescG192 = idesc_f16_f32_b<128, 192, 0>();
constexpr uint32_t kIdescG128 = idesc_f16_f32_b<128, 128, 0>();
constexpr uint32_t kIdescPV = idesc_f16_f32_b<128, 128, 1>();

__device__ __forceinline__ uint32_t h2u(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void named_sync_softmax() {
    asm volatile("bar.sync 1, 256;" ::: "memory");
}

// The two softmax warps of a lane quarter meet on their mbarrier (one arrival
// per warp; a bounded wait, so a warp that left early ends its partner's wait
// with an error instead of a hang).
__device__ __forceinline__ bool pair_exchange(uint64_t* bar, int lane, uint32_t parity, unsigned int site) {
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(bar));
    return mbar_wait(smem_u32(bar), parity, site);
}

__global__ void __launch_bounds__(kThreads, 1)
    k2_relpos_attention_tc(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv,
                           const __grid_constant__ CUtensorMap tm_r, const AttnParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sQu = smem + kQuOff;
    uint8_t* sK = smem + kKOff;
    uint8_t* sV = smem + kVOff;
    uint8_t* sR = smem + kROff;
    float* sSh = reinterpret_cast<float*>(smem + kShOff);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
    // K + R chunk and V have separate 2-stage rings: a K / R stage is free
    // again once the S and band MMAs that read it are done, long before the
    // P.V that frees its V stage, so the next loads start a softmax earlier
    uint64_t* kr_full = bars;        // [2]
    uint64_t* kr_empty = bars + 2;   // [2]
    uint64_t* v_full = bars + 4;     // [2]
    uint64_t* v_empty = bars + 6;    // [2]
    uint64_t* qld = bars + 8;
    uint64_t* q_tmem = bars + 9;
    uint64_t* sg_full = bars + 10;
    uint64_t* g_free = bars + 11;
    uint64_t* p_ready = bars + 12;
    uint64_t* o_ready = bars + 13;   // every P.V (waited only when O is rescaled)
    uint64_t* o_final = bars + 14;   // the last P.V
    uint64_t* xchg = bars + 15;      // [4] softmax warp pairs
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int head = blockIdx.y;
    const int2 wk = p.work[blockIdx.x];
    const int seg0 = p.cu[wk.x];
    const int T = p.cu[wk.x + 1] - seg0;
    const int q0 = wk.y;
    const int nkb = (T + kBK - 1) / kBK;
    // band of key block kb: R rows [r_lo0 + 64 kb, r_lo0 + 64 kb + 191]; ring
    // slot of R row r is (r - r_lo0) mod 256, so every 64-row chunk is contiguous
    const int r_lo0 = p.r_center - q0 - (kBQ - 1);

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_kv);
        tma_prefetch_desc(&tm_r);
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&kr_full[s]), 1);
            mbar_init(smem_u32(&kr_empty[s]), 1);
            mbar_init(smem_u32(&v_full[s]), 1);
            mbar_init(smem_u32(&v_empty[s]), 1);
        }
        mbar_init(smem_u32(qld), 1);
        mbar_init(smem_u32(q_tmem), 8);
        mbar_init(smem_u32(sg_full), 1);
        mbar_init(smem_u32(g_free), 8);
        mbar_init(smem_u32(p_ready), 8);
        mbar_init(smem_u32(o_ready), 1);
        mbar_init(smem_u32(o_final), 1);
        for (int c = 0; c < 4; ++c) mbar_init(smem_u32(&xchg[c]), 2);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc<512>(smem_u32(tmem_slot));
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ── TMA producer ──
        if (lane == 0) {
            const uint32_t qb = smem_u32(qld);
            mbar_arrive_expect_tx(qb, 4 * 16384);
            for (int h = 0; h < 2; ++h) {
                tma_load_2d(smem_u32(sQu + h * 16384), &tm_q, qb, head * 128 + h * 64, seg0 + q0);
                tma_load_2d(smem_u32(reinterpret_cast<uint8_t*>(sSh) + h * 16384), &tm_q, qb,
                            1024 + head * 128 + h * 64, seg0 + q0);
            }
            // in the order the MMAs need them: K / R of block kb, then V of kb - 1
            for (int kb = 0; kb <= nkb; ++kb) {
                if (kb < nkb) {
                    const int st = kb & 1;
                    if (kb >= 2 && !mbar_wait(smem_u32(&kr_empty[st]), ((kb >> 1) - 1) & 1, 0x21)) break;
                    const int nchunks = kb == 0 ? 3 : 1;
                    const uint32_t fb = smem_u32(&kr_full[st]);
                    mbar_arrive_expect_tx(fb, 16384 + nchunks * 16384);
                    for (int h = 0; h < 2; ++h)
                        tma_load_2d(smem_u32(sK + st * 16384 + h * 8192), &tm_kv, fb, 2048 + head * 128 + h * 64,
                                    seg0 + kb * kBK);
                    for (int c = (kb == 0 ? 0 : 2); c < 3; ++c) {
                        const int rel = kb * kBK + c * 64;            // band row - r_lo0
                        const uint32_t slot = static_cast<uint32_t>(rel) & (kRing - 1);
                        for (int h = 0; h < 2; ++h)
                            tma_load_2d(smem_u32(sR + h * 32768 + slot * 128), &tm_r, fb, head * 128 + h * 64,
                                        r_lo0 + rel);
                    }
                }
                if (kb >= 1) {
                    const int j = kb - 1, st = j & 1;
                    if (j >= 2 && !mbar_wait(smem_u32(&v_empty[st]), ((j >> 1) - 1) & 1, 0x2D)) break;
                    const uint32_t fb = smem_u32(&v_full[st]);
                    mbar_arrive_expect_tx(fb, 16384);
                    for (int h = 0; h < 2; ++h)
                        tma_load_2d(smem_u32(sV + st * 16384 + h * 8192), &tm_kv, fb, 3072 + head * 128 + h * 64,
                                    seg0 + j * kBK);
                }
            }
        }
    } else if (warp == 1) {
        // ── MMA issuer ──
        if (lane == 0) {
            bool ok = mbar_wait(smem_u32(qld), 0, 0x22) && mbar_wait(smem_u32(q_tmem), 0, 0x23);
            for (int kb = 0; kb <= nkb && ok; ++kb) {
                if (kb < nkb) {
                    const int st = kb & 1;
                    if (!(ok = mbar_wait(smem_u32(&kr_full[st]), (kb >> 1) & 1, 0x24))) break;
                    if (kb >= 1 && !(ok = mbar_wait(smem_u32(g_free), (kb - 1) & 1, 0x25))) break;
                    tc_fence_after();
                    const uint32_t dS = tmem + kTS + 64 * st;
                    // descriptors advance by 32 bytes (2 in the start-address field) per k-step
                    const uint64_t aq0 = smem_desc_sw128(smem_u32(sQu));
                    const uint64_t aq1 = smem_desc_sw128(smem_u32(sQu + 16384));
                    const uint64_t bk0 = smem_desc_sw128(smem_u32(sK + st * 16384));
                    const uint64_t bk1 = smem_desc_sw128(smem_u32(sK + st * 16384 + 8192));
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_f16_ss(dS, (kk < 4 ? aq0 : aq1) + 2 * (kk & 3), (kk < 4 ? bk0 : bk1) + 2 * (kk & 3), kIdescS,
                                   kk > 0);
                    // band rows [64 kb, 64 kb + 192) of the ring: one N192 piece when contiguous,
                    // else N128 + N64 or N64 + N128 around the wrap
                    const uint32_t s0 = static_cast<uint32_t>(kb * kBK) & (kRing - 1);
                    const int n1 = s0 <= kRing - 192 ? 192 : static_cast<int>(kRing - s0);
                    const uint64_t br0 = smem_desc_sw128(smem_u32(sR + s0 * 128));
                    const uint64_t br1 = smem_desc_sw128(smem_u32(sR + 32768 + s0 * 128));
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_f16_ts(tmem + kTG, tmem + kTQ + 8 * kk, (kk < 4 ? br0 : br1) + 2 * (kk & 3),
                                   n1 == 192 ? kIdescG192 : (n1 == 128 ? kIdescG128 : kIdescS), kk > 0);
                    if (n1 < 192) {
                        const uint64_t bw0 = smem_desc_sw128(smem_u32(sR));
                        const uint64_t bw1 = smem_desc_sw128(smem_u32(sR + 32768));
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk)
                            mma_f16_ts(tmem + kTG + n1, tmem + kTQ + 8 * kk, (kk < 4 ? bw0 : bw1) + 2 * (kk & 3),
                                       n1 == 128 ? kIdescS : kIdescG128, kk > 0);
                    }
                    mma_commit(smem_u32(sg_full));
                    mma_commit(smem_u32(&kr_empty[st]));
                }
                if (kb >= 1) {
                    const int j = kb - 1, st = j & 1;
                    if (!(ok = mbar_wait(smem_u32(p_ready), j & 1, 0x26))) break;
                    if (!(ok = mbar_wait(smem_u32(&v_full[st]), (j >> 1) & 1, 0x2E))) break;
                    tc_fence_after();
                    // V [64 keys][128 dims] as the MN-major B operand: 64-dim halves 8 KB
                    // apart, 8-key atoms 1 KB apart, 16 keys (2 KB) per MMA
                    const uint64_t bv = smem_desc_sw128_mn(smem_u32(sV + st * 16384), 8192, 1024);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16_ts(tmem + kTO, tmem + kTS + 64 * st + 8 * kk, bv + 128 * kk, kIdescPV, (j > 0 || kk > 0));
                    mma_commit(smem_u32(o_ready));
                    mma_commit(smem_u32(&v_empty[st]));
                    if (j == nkb - 1) mma_commit(smem_u32(o_final));
                }
            }
        }
    } else {
        // ── softmax: warps 2..9, pair (q, hf): lane quarter q, key half hf ──
        const int q = warp & 3;
        const int hf = (warp - 2) >> 2;
        const int i = q * 32 + lane;                   // query row / TMEM lane
        const int t = (warp - 2) * 32 + lane;          // diagonal row
        const int tp = t ^ 128;                        // the pair partner's diagonal row
        const uint32_t lrow = static_cast<uint32_t>(q * 32) << 16;
        // Qv row i, dim half hf: staging -> TMEM columns kTQ + 32 hf
        bool ok = mbar_wait(smem_u32(qld), 0, 0x27);
        if (ok) {
            uint32_t r[32];
            const uint8_t* row = reinterpret_cast<const uint8_t*>(sSh) + hf * 16384 + i * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 v = *reinterpret_cast<const uint4*>(row + ((c ^ (i & 7)) << 4));
                r[4 * c] = v.x;
                r[4 * c + 1] = v.y;
                r[4 * c + 2] = v.z;
                r[4 * c + 3] = v.w;
            }
            tmem_st_32x32b_x32(tmem + lrow + kTQ + 32 * hf, r);
            tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(q_tmem));
        named_sync_softmax();   // the staging area becomes the diagonal rows
        float* sh = sSh + t * kShStride;
        const float* shp = sSh + tp * kShStride;
        // m_use: the max the row's exponentials are taken against.  It moves
        // (and O, l are rescaled) only when a block's max exceeds it by more
        // than kRescale (log2 units), for the pair of warps as a whole; in
        // between, probabilities up to 2^kRescale are exact in f32 l and in
        // the f16 P operand.
        constexpr float kRescale = 8.0f;
        float m_use = -INFINITY, l_half = 0.f;
        for (int kb = 0; kb < nkb && ok; ++kb) {
            const int st = kb & 1;
            if (!(ok = mbar_wait(smem_u32(sg_full), kb & 1, 0x28))) break;
            tc_fence_after();
            float s[32];
            {
                // S columns [32 hf, 32 hf + 32) and band columns [96 - 32q + 32hf, +64): one wait
                uint32_t r0[32], g0[32], g1[32];
                tmem_ld_32x32b_x32(tmem + lrow + kTS + 64 * st + 32 * hf, r0);
                tmem_ld_32x32b_x32(tmem + lrow + kTG + 96 - 32 * q + 32 * hf, g0);
                tmem_ld_32x32b_x32(tmem + lrow + kTG + 128 - 32 * q + 32 * hf, g1);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(g_free));
#pragma unroll
                for (int e = 0; e < 32; ++e) s[e] = __uint_as_float(r0[e]);
                // window column c (0..62 are used) goes to position (c + lane) mod 64:
                // the columns a row needs, 31 - lane + j, then sit at 31 + j for every
                // lane (conflict-free reads at the odd row stride); position
                // (63 + lane) mod 64 and position 64 stay free for the pair exchange
#pragma unroll
                for (int e = 0; e < 32; ++e) sh[(e + lane) & 63] = __uint_as_float(g0[e]);
#pragma unroll
                for (int e = 0; e < 31; ++e) sh[(32 + e + lane) & 63] = __uint_as_float(g1[e]);
            }
            // row i, key 32 hf + j: band column 127 - i + 32 hf + j = window column 31 - lane + j
            const float* dg = sh + 31;
            const int kvalid = T - kb * kBK - 32 * hf;
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                float v = (s[j] + dg[j]) * p.scale_log2;
                if (j >= kvalid) v = -INFINITY;
                s[j] = v;
                mx[j & 3] = fmaxf(mx[j & 3], v);
            }
            const float mloc = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
            const int xs = st ? 64 : ((63 + lane) & 63);   // exchange slot, by block parity
            sh[xs] = mloc;
            if (!(ok = pair_exchange(&xchg[q], lane, kb & 1, 0x2B))) break;
            const float m_blk = fmaxf(mloc, shp[xs]);
            const bool grow = m_blk > m_use + kRescale;
            float corr = 1.f;
            if (__any_sync(0xffffffffu, grow)) {
                const float m_new = grow ? m_blk : m_use;
                corr = exp2f(m_use - m_new);   // 0 for the first block
                m_use = m_new;
                if (kb >= 1) {
                    // O columns [64 hf, 64 hf + 64) (after P_{kb-1} V) *= corr.
                    // Passing sg_full(kb) implies P_{kb-2} V is done and P_kb V is not
                    // issued yet, so o_ready is at phase kb-1 or kb: the parity is exact.
                    if (!(ok = mbar_wait(smem_u32(o_ready), (kb - 1) & 1, 0x29))) break;
                    tc_fence_after();
                    uint32_t o0[32], o1[32];
                    tmem_ld_32x32b_x32(tmem + lrow + kTO + 64 * hf, o0);
                    tmem_ld_32x32b_x32(tmem + lrow + kTO + 64 * hf + 32, o1);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        o0[e] = __float_as_uint(__uint_as_float(o0[e]) * corr);
                        o1[e] = __float_as_uint(__uint_as_float(o1[e]) * corr);
                    }
                    tmem_st_32x32b_x32(tmem + lrow + kTO + 64 * hf, o0);
                    tmem_st_32x32b_x32(tmem + lrow + kTO + 64 * hf + 32, o1);
                }
            }
            float ls[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const float a = exp2f(s[j] - m_use), b = exp2f(s[j + 1] - m_use);
                ls[(j >> 1) & 3] += a + b;
                pk[j >> 1] = h2u(a, b);
            }
            l_half = l_half * corr + ((ls[0] + ls[1]) + (ls[2] + ls[3]));
            tmem_st_32x32b_x16(tmem + lrow + kTS + 64 * st + 16 * hf, pk);   // P over this block's S columns
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(p_ready));
        }
        // ── O / l -> f16 row, columns [64 hf, 64 hf + 64) ──
        if (ok && nkb > 0 && mbar_wait(smem_u32(o_final), 0, 0x2A)) {
            tc_fence_after();
            const int xs = (nkb & 1) ? 64 : ((63 + lane) & 63);   // the slot the last block did not use
            sh[xs] = l_half;
            const bool xok = pair_exchange(&xchg[q], lane, nkb & 1, 0x2C);
            const float inv = 1.0f / (l_half + shp[xs]);
            const bool store = xok && q0 + i < T;
            __half* dst = p.out + static_cast<size_t>(seg0 + q0 + i) * 1024 + head * 128 + 64 * hf;
            uint32_t o0[32], o1[32];
            tmem_ld_32x32b_x32(tmem + lrow + kTO + 64 * hf, o0);
            tmem_ld_32x32b_x32(tmem + lrow + kTO + 64 * hf + 32, o1);
            tmem_wait_ld();
            if (store) {
#pragma unroll
                for (int e = 0; e < 32; e += 8) {
                    *reinterpret_cast<uint4*>(dst + e) =
                        make_uint4(h2u(__uint_as_float(o0[e]) * inv, __uint_as_float(o0[e + 1]) * inv),
                                   h2u(__uint_as_float(o0[e + 2]) * inv, __uint_as_float(o0[e + 3]) * inv),
                                   h2u(__uint_as_float(o0[e + 4]) * inv, __uint_as_float(o0[e + 5]) * inv),
                                   h2u(__uint_as_float(o0[e + 6]) * inv, __uint_as_float(o0[e + 7]) * inv));
                    *reinterpret_cast<uint4*>(dst + 32 + e) =
                        make_uint4(h2u(__uint_as_float(o1[e]) * inv, __uint_as_float(o1[e + 1]) * inv),
                                   h2u(__uint_as_float(o1[e + 2]) * inv, __uint_as_float(o1[e + 3]) * inv),
                                   h2u(__uint_as_float(o1[e + 4]) * inv, __uint_as_float(o1[e + 5]) * inv),
                                   h2u(__uint_as_float(o1[e + 6]) * inv, __uint_as_float(o1[e + 7]) * inv));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<512>(tmem);
    }
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error(what, e);
}

}  // namespace

int launch_attention_tc(const AttnParams& p, int M, int n_work, cudaStream_t st) {
    if (n_work <= 0) return 0;
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(k2_relpos_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kSmem));
        if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(k2 tc)", e);
        attr_done = true;
    }
    CUtensorMap tq, tkv, tr;
    int rc = make_map_2d(&tq, p.qkv, kMapF16, 4096, static_cast<uint64_t>(M), 8192, 64, kBQ, true);
    if (!rc) rc = make_map_2d(&tkv, p.qkv, kMapF16, 4096, static_cast<uint64_t>(M), 8192, 64, kBK, true);
    if (!rc) rc = make_map_2d(&tr, p.R, kMapF16, 1024, static_cast<uint64_t>(p.r_rows), 2048, 64, 64, true);
    if (rc) return rc;
    k2_relpos_attention_tc<<<dim3(n_work, 8), kThreads, kSmem, st>>>(tq, tkv, tr, p);
    return check_launch("k2_relpos_attention_tc");
}

int attention_tc_block_rows() { return kBQ; }

// Reads and clears this translation unit's device error word (stream-ordered).
int attention_take_dev_error(cudaStream_t st, unsigned int* out) {
    static const unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_b3_dev_error, sizeof(unsigned int), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbolAsync(g_b3_dev_error, &zero, sizeof(unsigned int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? 0 : set_cuda_error("reading the attention device error word", e);
}

}  // namespace b3
