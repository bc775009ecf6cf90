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
//   warp 0      TMA: Qu and Qv once per item; per key block K, the new band
//               chunk's 64 R rows and V, each in its own 2-stage ring;
//   warp 1      TMEM owner; one thread issues the MMAs:
//                 S  = Qu K^T       M128 N64  K128 (A: Qu in shared memory)
//                 Gc = Qv R_chunk^T M128 N64  K128 (A: Qv in shared memory)
//                 O += P V          M128 N128 K64  (A: P in TMEM, B: V MN-major)
//   warps 2..17 softmax, four warps per TMEM lane quarter: one query row per
//               lane, each warp of a quad owns 16 of the block's 64 keys (and
//               32 of O's 128 columns).  A thread reads its S columns and the
//               band columns its warp parks, adds the row's diagonal of the
//               band, and the quad exchanges row maxima through shared memory;
//               online softmax in f32 with a lazily moved reference max (O and
//               l are rescaled only when the block max exceeds it by 2^8);
//               P (f16) is written over the block's S columns.  Four warps
//               per quarter (not two) keep the dependent chain of each
//               thread short enough that the special-function, shared-memory
//               and tensor work of consecutive blocks overlap.
// The band of a 128 x 64 score tile covers offsets q0-k0-63 .. q0-k0+127 (191
// R rows, taken as 192 = three 64-row chunks).  Consecutive key blocks share
// two of their three chunks, so the band lives in TMEM as a ring of four
// 64-column chunk slots: block 0 of an item computes chunks 0, 1 and 2, every
// later block only the one new chunk kb + 2 (each band product once, a third
// of the band MMAs of computing all 192 columns per block).  With S double-
// buffered and the fourth slot spare, the MMAs of block kb + 1 need only the
// softmax of block kb - 1 to have read its columns, so the tensor pipe runs a
// block ahead of the softmax instead of waiting for it every block.
//
// The diagonal read: row i of the tile needs band column 127 - i + j for key
// j, a window whose start moves by one column per row.  TMEM loads address
// the same columns for all lanes of a warp, so the rows' band columns are
// parked in shared memory and each thread reads the 16 it needs back at its
// own offset.  The four warps of a lane quarter share one parked row per query
// (the 96 band columns the quad spans, 24 loaded and parked by each) and meet
// on their mbarrier between parking and reading.
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
constexpr int kThreads = 576;     // warp 0 TMA, warp 1 MMA, warps 2..17 softmax
constexpr int kShRows = 128;      // one parked row per query, shared by the quad of warps
constexpr int kShStride = 130;    // floats per row: 96 band columns + 4 x 2 exchange slots (+ pad); a stride
                                  // of 2 mod 32 words keeps 8-byte stores and lane-shifted reads conflict-free

// shared memory (offsets from a 1024-aligned base)
constexpr uint32_t kQuOff = 0;                   // Qu: 2 dim-halves x (128 rows x 128 B)
constexpr uint32_t kQvOff = 32768;               // Qv: same (A operand of the band chunks)
constexpr uint32_t kKOff = 65536;                // K: 2 stages x 2 halves x (64 rows x 128 B)
constexpr uint32_t kVOff = kKOff + 32768;        // V: same
constexpr uint32_t kROff = kVOff + 32768;        // R chunks: same (64 R rows per chunk)
constexpr uint32_t kShOff = kROff + 32768;       // parked band rows 128 x 130 f32
constexpr uint32_t kBarOff = kShOff + kShRows * kShStride * 4;
constexpr uint32_t kBarBytes = 176;                   // 21 mbarriers + the TMEM address
constexpr uint32_t kSmemMax = 232448;
constexpr uint32_t kSmem = kSmemMax;
constexpr uint32_t kAlignSlack = kSmemMax - kBarOff - kBarBytes;   // room to align the base to 1024 B
static_assert(kBarOff + kBarBytes + 1024 <= kSmemMax, "shared memory budget");

// TMEM columns
constexpr uint32_t kTS = 0;       // S / P, 2 buffers x 64
constexpr uint32_t kTG = 128;     // band ring: 4 chunks x 64 offsets (chunk c in slot c mod 4)
constexpr uint32_t kTO = 384;     // O, 128

constexpr uint32_t kIdescS = idesc_f16_f32_b<128, 64, 0>();
constexpr uint32_t kIdescPV = idesc_f16_f32_b<128, 128, 1>();

// 2^x by the special-function unit's approximation (relative error below
// 2^-22, far inside the f16 rounding the probabilities get; results below
// 2^-126 flush to zero, where a probability is negligible beside the row's
// maximum of 1 and its f16 copy is zero anyway).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t h2u(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// The four softmax warps of lane quarter q meet on named barrier q + 1 (128
// threads) and AND their flags.  Every warp of the quad takes every one of
// these barriers in the same order: a failed bounded wait only clears the
// warp's flag, and the AND makes all four leave the item loop together at
// the next meeting, so no warp is left waiting on one that has gone.
__device__ __forceinline__ bool quad_sync_and(int q, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred t, %2, 128, p;\n\t"
        "selp.u32 %0, 1, 0, t;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "r"(q + 1)
        : "memory");
    return r != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    k2_relpos_attention_tc(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv,
                           const __grid_constant__ CUtensorMap tm_r, const AttnParams p, int n_items) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    if (static_cast<uint32_t>(smem - smem_raw) > kAlignSlack) {   // never expected: the base is 1 KB aligned
        if (threadIdx.x == 0) record_error(B3_ERR_TIMEOUT | 0x2F);
        return;
    }
    uint8_t* sQu = smem + kQuOff;
    uint8_t* sQv = smem + kQvOff;
    uint8_t* sK = smem + kKOff;
    uint8_t* sV = smem + kVOff;
    uint8_t* sR = smem + kROff;
    float* sSh = reinterpret_cast<float*>(smem + kShOff);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
    // K, R chunks and V have separate 2-stage rings: a K or R stage is free
    // again once the MMA that read it is done, long before the P.V that frees
    // its V stage.  Every phase is counted over the CTA's whole run (g = key
    // block, rc = band chunk, n = item, x = quad exchange), so the rings keep
    // prefetching across items.  sg_full, g_free and p_ready come in two
    // copies (even and odd key blocks): the MMA issuer may run a block ahead
    // of the slowest softmax warp and wait for a block two behind, and with
    // one barrier per parity no barrier can complete twice before a waiter
    // looks at it, so every parity wait is unambiguous.
    uint64_t* k_full = bars;         // [2]
    uint64_t* k_empty = bars + 2;    // [2]
    uint64_t* v_full = bars + 4;     // [2]
    uint64_t* v_empty = bars + 6;    // [2]
    uint64_t* r_full = bars + 8;     // [2]
    uint64_t* r_empty = bars + 10;   // [2]
    uint64_t* qld = bars + 12;       // Qu and Qv of item n in shared memory
    uint64_t* sg_full = bars + 13;   // [2] S and the band chunks of a block are in TMEM
    uint64_t* g_free = bars + 15;    // [2] the softmax has read a block's S and band columns
    uint64_t* p_ready = bars + 17;   // [2] a block's P is in TMEM
    uint64_t* o_ready = bars + 19;   // every P.V (waited only when O is rescaled)
    uint64_t* o_final = bars + 20;   // the last P.V of an item
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);
    static_assert(21 * 8 + 4 <= kBarBytes, "barrier area");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_kv);
        tma_prefetch_desc(&tm_r);
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&k_full[s]), 1);
            mbar_init(smem_u32(&k_empty[s]), 1);
            mbar_init(smem_u32(&v_full[s]), 1);
            mbar_init(smem_u32(&v_empty[s]), 1);
            mbar_init(smem_u32(&r_full[s]), 1);
            mbar_init(smem_u32(&r_empty[s]), 1);
            mbar_init(smem_u32(&sg_full[s]), 1);
            mbar_init(smem_u32(&g_free[s]), 16);
            mbar_init(smem_u32(&p_ready[s]), 16);
        }
        mbar_init(smem_u32(qld), 1);
        mbar_init(smem_u32(o_ready), 1);
        mbar_init(smem_u32(o_final), 1);
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

    // item i: work entry i / 8 (utterance, first query), head i % 8
    struct Item {
        int seg0, T, q0, head, nkb, r_lo0;
    };
    auto item = [&](int i) {
        Item it;
        const int4 wk = __ldg(p.work + (i >> 3));   // one load: no dependent reads at an item's start
        it.head = i & 7;
        it.seg0 = wk.x;
        it.T = wk.y;
        it.q0 = wk.z;
        it.nkb = (it.T + kBK - 1) / kBK;
        // band of key block kb: R rows [r_lo0 + 64 kb, r_lo0 + 64 kb + 191], the
        // band chunks kb, kb + 1 and kb + 2 of 64 rows (chunk c = R rows
        // [r_lo0 + 64 c, r_lo0 + 64 c + 64)); block 0 computes chunks 0..2,
        // block kb >= 1 chunk kb + 2, so every band product is computed once
        it.r_lo0 = p.r_center - it.q0 - (kBQ - 1);
        return it;
    };

    if (warp == 0) {
        // ── TMA producer ──
        if (lane == 0) {
            int g0 = 0, rc = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
                const Item it = item(i);
                // Qu and Qv are read by the previous item's last S and band MMAs,
                // which complete before that block's K stage is released
                if (g0 >= 1 && !(ok = mbar_wait(smem_u32(&k_empty[(g0 - 1) & 1]), ((g0 - 1) >> 1) & 1, 0x20)))
                    break;
                const uint32_t qb = smem_u32(qld);
                mbar_arrive_expect_tx(qb, 4 * 16384);
                for (int h = 0; h < 2; ++h) {
                    tma_load_2d(smem_u32(sQu + h * 16384), &tm_q, qb, it.head * 128 + h * 64, it.seg0 + it.q0);
                    tma_load_2d(smem_u32(sQv + h * 16384), &tm_q, qb, 1024 + it.head * 128 + h * 64, it.seg0 + it.q0);
                }
                // in the order the MMAs need them: K of block kb, its band chunks, then V of kb - 1
                for (int kb = 0; kb <= it.nkb && ok; ++kb) {
                    if (kb < it.nkb) {
                        const int g = g0 + kb, st = g & 1;
                        if (g >= 2 && !(ok = mbar_wait(smem_u32(&k_empty[st]), ((g >> 1) - 1) & 1, 0x21))) break;
                        const uint32_t fb = smem_u32(&k_full[st]);
                        mbar_arrive_expect_tx(fb, 16384);
                        for (int h = 0; h < 2; ++h)
                            tma_load_2d(smem_u32(sK + st * 16384 + h * 8192), &tm_kv, fb,
                                        2048 + it.head * 128 + h * 64, it.seg0 + kb * kBK);
                        for (int c = (kb == 0 ? 0 : kb + 2); c <= kb + 2; ++c, ++rc) {
                            const int rs = rc & 1;
                            if (rc >= 2 && !(ok = mbar_wait(smem_u32(&r_empty[rs]), ((rc >> 1) - 1) & 1, 0x2E))) break;
                            const uint32_t rb = smem_u32(&r_full[rs]);
                            mbar_arrive_expect_tx(rb, 16384);
                            for (int h = 0; h < 2; ++h)
                                tma_load_2d(smem_u32(sR + rs * 16384 + h * 8192), &tm_r, rb, it.head * 128 + h * 64,
                                            it.r_lo0 + c * 64);
                        }
                    }
                    if (ok && kb >= 1) {
                        const int gv = g0 + kb - 1, st = gv & 1;
                        if (gv >= 2 && !(ok = mbar_wait(smem_u32(&v_empty[st]), ((gv >> 1) - 1) & 1, 0x2D))) break;
                        const uint32_t fb = smem_u32(&v_full[st]);
                        mbar_arrive_expect_tx(fb, 16384);
                        for (int h = 0; h < 2; ++h)
                            tma_load_2d(smem_u32(sV + st * 16384 + h * 8192), &tm_kv, fb,
                                        3072 + it.head * 128 + h * 64, it.seg0 + (kb - 1) * kBK);
                    }
                }
                g0 += it.nkb;
            }
        }
    } else if (warp == 1) {
        // ── MMA issuer ──
        if (lane == 0) {
            int g0 = 0, n = 0, rc = 0, cbase = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++n) {
                const Item it = item(i);
                if (!(ok = mbar_wait(smem_u32(qld), n & 1, 0x22))) break;
                const uint64_t aq0 = smem_desc_sw128(smem_u32(sQu));
                const uint64_t aq1 = smem_desc_sw128(smem_u32(sQu + 16384));
                const uint64_t av0 = smem_desc_sw128(smem_u32(sQv));
                const uint64_t av1 = smem_desc_sw128(smem_u32(sQv + 16384));
                for (int kb = 0; kb <= it.nkb && ok; ++kb) {
                    if (kb < it.nkb) {
                        const int g = g0 + kb, st = g & 1;
                        if (!(ok = mbar_wait(smem_u32(&k_full[st]), (g >> 1) & 1, 0x24))) break;
                        // TMEM this block writes is free: S buffer st held P of block g - 2
                        // (its P.V was issued before, MMAs run in order); the band slot of
                        // chunk c held chunk c - 4, last read by block g - 2 (block g - 1
                        // too when this is an item's first block, which writes three)
                        const int gw = kb == 0 ? g - 1 : g - 2;
                        if (gw >= 0 && !(ok = mbar_wait(smem_u32(&g_free[gw & 1]), (gw >> 1) & 1, 0x25))) break;
                        tc_fence_after();
                        const uint32_t dS = tmem + kTS + 64 * st;
                        // descriptors advance by 32 bytes (2 in the start-address field) per k-step
                        const uint64_t bk0 = smem_desc_sw128(smem_u32(sK + st * 16384));
                        const uint64_t bk1 = smem_desc_sw128(smem_u32(sK + st * 16384 + 8192));
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk)
                            mma_f16_ss(dS, (kk < 4 ? aq0 : aq1) + 2 * (kk & 3), (kk < 4 ? bk0 : bk1) + 2 * (kk & 3),
                                       kIdescS, kk > 0);
                        for (int c = (kb == 0 ? 0 : kb + 2); c <= kb + 2 && ok; ++c, ++rc) {
                            const int rs = rc & 1;
                            if (!(ok = mbar_wait(smem_u32(&r_full[rs]), (rc >> 1) & 1, 0x2F))) break;
                            tc_fence_after();
                            const uint32_t dG = tmem + kTG + 64 * ((cbase + c) & 3);
                            const uint64_t br0 = smem_desc_sw128(smem_u32(sR + rs * 16384));
                            const uint64_t br1 = smem_desc_sw128(smem_u32(sR + rs * 16384 + 8192));
#pragma unroll
                            for (int kk = 0; kk < 8; ++kk)
                                mma_f16_ss(dG, (kk < 4 ? av0 : av1) + 2 * (kk & 3), (kk < 4 ? br0 : br1) + 2 * (kk & 3),
                                           kIdescS, kk > 0);
                            mma_commit(smem_u32(&r_empty[rs]));
                        }
                        if (!ok) break;
                        mma_commit(smem_u32(&sg_full[st]));
                        mma_commit(smem_u32(&k_empty[st]));
                    }
                    if (kb >= 1) {
                        const int j = kb - 1, gj = g0 + j, st = gj & 1;
                        if (!(ok = mbar_wait(smem_u32(&p_ready[gj & 1]), (gj >> 1) & 1, 0x26))) break;
                        if (!(ok = mbar_wait(smem_u32(&v_full[st]), (gj >> 1) & 1, 0x2E))) break;
                        tc_fence_after();
                        // V [64 keys][128 dims] as the MN-major B operand: 64-dim halves 8 KB
                        // apart, 8-key atoms 1 KB apart, 16 keys (2 KB) per MMA
                        const uint64_t bv = smem_desc_sw128_mn(smem_u32(sV + st * 16384), 8192, 1024);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_f16_ts(tmem + kTO, tmem + kTS + 64 * st + 8 * kk, bv + 128 * kk, kIdescPV,
                                       (j > 0 || kk > 0));
                        mma_commit(smem_u32(o_ready));
                        mma_commit(smem_u32(&v_empty[st]));
                        if (j == it.nkb - 1) mma_commit(smem_u32(o_final));
                    }
                }
                g0 += it.nkb;
                cbase += it.nkb + 2;
            }
        }
    } else {
        // ── softmax: warps 2..17, quad (q, ks): lane quarter q, keys [16 ks, 16 ks + 16) ──
        const int q = warp & 3;
        const int ks = (warp - 2) >> 2;
        const int i = q * 32 + lane;                   // query row / TMEM lane
        const uint32_t lrow = static_cast<uint32_t>(q * 32) << 16;
        float* sh = sSh + i * kShStride;               // this query's parked row (all four warps of the quad)
        // exchange slots [4 warps][2 parities], one word further on for rows
        // 16..31 of each quarter: with the row stride of 2 mod 32 words, lane
        // l and lane l + 16 would otherwise hit the same bank
        float* xslot = sh + 96 + ((i >> 4) & 1);
        // the four warps of the quad meet: every slot of parity `par` written
        auto quad_sum = [&](int par) {
            return ((xslot[par] + xslot[2 + par]) + xslot[4 + par]) + xslot[6 + par];
        };
        auto quad_max = [&](int par) {
            return fmaxf(fmaxf(xslot[par], xslot[2 + par]), fmaxf(xslot[4 + par], xslot[6 + par]));
        };
        bool ok = true;     // uniform across the quad: set only from quad_sync_and
        bool fine = true;   // this warp's bounded waits all succeeded
        int g0 = 0, n = 0, x = 0, cbase = 0;
        for (int ii = blockIdx.x; ii < n_items && ok; ii += gridDim.x, ++n) {
            const Item it = item(ii);
            // m_use: the max the row's exponentials are taken against.  It moves
            // (and O, l are rescaled) only when a block's max exceeds it by more
            // than kRescale (log2 units), for the quad of warps as a whole; in
            // between, probabilities up to 2^kRescale are exact in f32 l and in
            // the f16 P operand.
            constexpr float kRescale = 8.0f;
            float m_use = -INFINITY, l_part = 0.f;
            for (int kb = 0; kb < it.nkb && ok; ++kb) {
                const int g = g0 + kb, st = g & 1;
                const bool got = __all_sync(0xffffffffu, mbar_wait(smem_u32(&sg_full[g & 1]), (g >> 1) & 1, 0x28));
                float s[16];
                if (got) {
                    tc_fence_after();
                    // S columns [16 ks, 16 ks + 16); the quad's band window is band
                    // columns [96 - 32q, 192 - 32q) (chunks kb .. kb + 2), of which this
                    // warp loads [24 ks, 24 ks + 24); band column w sits in ring column
                    // (64 (cbase + kb) + w) mod 256, and an 8-column load never wraps
                    uint32_t r0[16], gr[24];
                    const int w0 = 96 - 32 * q + 24 * ks;
                    auto ring = [&](int w) { return kTG + ((64 * (cbase + kb) + w) & 255); };
                    tmem_ld_32x32b_x16(tmem + lrow + kTS + 64 * st + 16 * ks, r0);
                    tmem_ld_32x32b_x8(tmem + lrow + ring(w0), *reinterpret_cast<uint32_t(*)[8]>(gr));
                    tmem_ld_32x32b_x8(tmem + lrow + ring(w0 + 8), *reinterpret_cast<uint32_t(*)[8]>(gr + 8));
                    tmem_ld_32x32b_x8(tmem + lrow + ring(w0 + 16), *reinterpret_cast<uint32_t(*)[8]>(gr + 16));
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&g_free[g & 1]));
#pragma unroll
                    for (int e = 0; e < 16; ++e) s[e] = __uint_as_float(r0[e]);
                    // window columns [24 ks, 24 ks + 24) as 8-byte stores: with the row
                    // stride of 2 mod 32 words a half-warp's stores cover all 32 banks
                    float* wp = sh + 24 * ks;
#pragma unroll
                    for (int e = 0; e < 24; e += 2) *reinterpret_cast<uint2*>(wp + e) = make_uint2(gr[e], gr[e + 1]);
                }
                // the other warps' parts of the window are parked too
                fine = fine && got;
                if (!(ok = quad_sync_and(q, fine))) break;
                ++x;
                // row i, key 16 ks + j: band column 127 - i + 16 ks + j = window column
                // 16 ks + 31 - lane + j; across a warp the word index moves by 129 per
                // lane: no conflicts
                const float* dg = sh + 16 * ks + 31 - lane;
                const int kvalid = it.T - kb * kBK - 16 * ks;
                const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                    const float2 v = __fmul2_rn(__fadd2_rn(make_float2(s[j], s[j + 1]), make_float2(dg[j], dg[j + 1])), sc2);
                    s[j] = v.x;
                    s[j + 1] = v.y;
                }
                if (kvalid < 16) {   // warp-uniform: only an utterance's last key block has keys past its end
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (j >= kvalid) s[j] = -INFINITY;
                }
                float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int j = 0; j < 16; ++j) mx[j & 3] = fmaxf(mx[j & 3], s[j]);
                const float mloc = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
                xslot[2 * ks + (x & 1)] = mloc;
                quad_sync_and(q, true);
                const float m_blk = quad_max(x & 1);
                ++x;
                const bool grow = m_blk > m_use + kRescale;
                float corr = 1.f;
                if (__any_sync(0xffffffffu, grow)) {
                    const float m_new = grow ? m_blk : m_use;
                    corr = exp2f(m_use - m_new);   // 0 for the first block
                    m_use = m_new;
                    if (kb >= 1) {
                        // O columns [32 ks, 32 ks + 32) (after P_{g-1} V) *= corr.
                        // Passing sg_full(g) implies P_{g-2} V is done and P_g V is not
                        // issued yet, so o_ready is at phase g-1 or g: the parity is exact.
                        const bool ordy = __all_sync(0xffffffffu, mbar_wait(smem_u32(o_ready), (g - 1) & 1, 0x29));
                        fine = fine && ordy;
                        if (ordy) {
                            tc_fence_after();
                            uint32_t o0[32];
                            tmem_ld_32x32b_x32(tmem + lrow + kTO + 32 * ks, o0);
                            tmem_wait_ld();
#pragma unroll
                            for (int e = 0; e < 32; ++e) o0[e] = __float_as_uint(__uint_as_float(o0[e]) * corr);
                            tmem_st_32x32b_x32(tmem + lrow + kTO + 32 * ks, o0);
                        }
                    }
                }
                float2 ls[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                uint32_t pk[8];
                const float2 mneg = make_float2(-m_use, -m_use);
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                    const float2 xv = __fadd2_rn(make_float2(s[j], s[j + 1]), mneg);
                    const float2 e = make_float2(ex2_approx(xv.x), ex2_approx(xv.y));
                    ls[(j >> 1) & 1] = __fadd2_rn(ls[(j >> 1) & 1], e);
                    pk[j >> 1] = h2u(e.x, e.y);
                }
                l_part = l_part * corr + ((ls[0].x + ls[0].y) + (ls[1].x + ls[1].y));
                tmem_st_32x32b_x8(tmem + lrow + kTS + 64 * st + 8 * ks, pk);   // P over this block's S columns
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&p_ready[g & 1]));
            }
            // ── O / l -> f16 row, columns [32 ks, 32 ks + 32) ──
            if (ok) {   // uniform: every warp of the quad takes this meeting
                const bool fin = __all_sync(0xffffffffu, mbar_wait(smem_u32(o_final), n & 1, 0x2A));
                if (fin) {
                    tc_fence_after();
                    xslot[2 * ks + (x & 1)] = l_part;
                }
                const bool xok = quad_sync_and(q, fine && fin);
                const float inv = xok ? 1.0f / quad_sum(x & 1) : 0.f;
                ++x;
                const bool store = xok && it.q0 + i < it.T;
                __half* dst = p.out + static_cast<size_t>(it.seg0 + it.q0 + i) * 1024 + it.head * 128 + 32 * ks;
                uint32_t o0[32];
                tmem_ld_32x32b_x32(tmem + lrow + kTO + 32 * ks, o0);
                tmem_wait_ld();
                if (store) {
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        *reinterpret_cast<uint4*>(dst + e) =
                            make_uint4(h2u(__uint_as_float(o0[e]) * inv, __uint_as_float(o0[e + 1]) * inv),
                                       h2u(__uint_as_float(o0[e + 2]) * inv, __uint_as_float(o0[e + 3]) * inv),
                                       h2u(__uint_as_float(o0[e + 4]) * inv, __uint_as_float(o0[e + 5]) * inv),
                                       h2u(__uint_as_float(o0[e + 6]) * inv, __uint_as_float(o0[e + 7]) * inv));
                    }
                }
                tc_fence_before();
                ok = xok;
            }
            g0 += it.nkb;
            cbase += it.nkb + 2;
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
    static PerDeviceOnce attr;
    int rc0 = set_smem_limit_once(attr, k2_relpos_attention_tc, static_cast<int>(kSmem), "cudaFuncSetAttribute(k2 tc)");
    if (rc0) return rc0;
    CUtensorMap tq, tkv, tr;
    int rc = make_map_2d(&tq, p.qkv, kMapF16, 4096, static_cast<uint64_t>(M), 8192, 64, kBQ, true);
    if (!rc) rc = make_map_2d(&tkv, p.qkv, kMapF16, 4096, static_cast<uint64_t>(M), 8192, 64, kBK, true);
    if (!rc) rc = make_map_2d(&tr, p.R, kMapF16, 1024, static_cast<uint64_t>(p.r_rows), 2048, 64, 64, true);
    if (rc) return rc;
    // persistent: one CTA per SM walks the (work entry, head) items
    const int sms = device_sms();
    const int n_items = n_work * 8;
    k2_relpos_attention_tc<<<n_items < sms ? n_items : sms, kThreads, kSmem, st>>>(tq, tkv, tr, p, n_items);
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
