// gemm_lut4.cu — K1: the encoder linear on 5th-generation tensor cores.
//
//   C[m, n] = sum_k A[m, k] * W[n, k]      (+ fused epilogue)
//
// A is f16 activations [M, K] row-major (the residual stream is f32; its
// LayerNorm / SiLU / GLU producers write the f16 copy this kernel reads).
// W is either
//   * LUT4: 4-bit codes [N, K/2] bytes (low nibble = even k, the byte order of
//     the .bark container's u32 words, bark.rs:352-358) plus a per-row
//     16-entry f16 level table [N, 16]; or
//   * F16: dense f16 [N, K] (the bf16 "Pro" checkpoint after the reference's
//     own bf16 -> f16 load-time rounding, raw.rs:68-97 / cpu/mod.rs:35-37).
// Both are the values the reference multiplies: its GPU low-bit kernel
// (encoder/gemm.rs:247-493) and CPU path (cpu/mod.rs:35, bark.rs:379-392) use
// exactly these f16 weights with f32 accumulation.
//
// Persistent, warp-specialised kernel (one CTA per SM, 448 threads).  A tile
// is SUB*128 rows x BN columns; tiles are walked m-major so the CTAs working at
// the same time share A rows in L2 while the (small) 4-bit B stays L2-resident.
//   warp 0       TMA producer: SUB A boxes (128 x 64 f16, 128-byte swizzle)
//                and the code tile (BN x 32 B) or the f16 B tile per stage,
//                into a STAGES-deep ring guarded by mbarriers;
//   warp 1       TMEM owner; one thread issues tcgen05.mma (M=128, N=BN, K=16,
//                f32 accumulators in TMEM), SUB MMAs per k-step share one B;
//   warps 2..9   LUT4 expanders: the per-row table lives in registers as
//                low/high byte planes; PRMT looks up four codes at a time and
//                the f16 rows are written straight into the 128-byte-swizzled
//                K-major B tile the MMA reads;
//   warps 10..13 epilogue: tcgen05.ld -> bias / SiLU / GLU / residual /
//                q-k-v split -> global.  TMEM holds two accumulator sets, so
//                the epilogue of one tile overlaps the mainloop of the next.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b3_internal.h"
#include "b3_ptx.cuh"

namespace b3 {

namespace {

constexpr int kBM = 128;      // rows per MMA / per A box
constexpr int kBK = 64;       // k per stage (one 128-byte swizzle row of f16)
constexpr int kBoxN = 64;     // rows per B / code TMA box
constexpr int kThreads = 448;
constexpr int kExpThreads = 256;  // warps 2..9
constexpr int kEpiWarp0 = 10;

template <int BN, int SUB, bool LUT>
struct GemmCfg {
    static constexpr uint32_t kABytes = kBM * kBK * 2;          // one A box
    static constexpr uint32_t kBBytes = BN * kBK * 2;
    static constexpr uint32_t kCBytes = LUT ? BN * kBK / 2 : 0;
    static constexpr uint32_t kStageBytes = SUB * kABytes + kBBytes + kCBytes;
    static constexpr uint32_t kOutBytes = 4 * 4096;              // one 32 x 128 B slab per epilogue warp
    static constexpr uint32_t kBarBytes = 512;
    static constexpr uint32_t kRingBudget = 232448 - kOutBytes - kBarBytes - 1024;
    static constexpr int kStages = kRingBudget / kStageBytes > 8 ? 8 : kRingBudget / kStageBytes;
    static constexpr uint32_t kAccCols = SUB * BN;               // one accumulator set
    static constexpr uint32_t kTmemCols = 2 * kAccCols <= 32 ? 32 : 2 * kAccCols;
    static constexpr uint32_t kSmemBytes = kStages * kStageBytes + kOutBytes + kBarBytes + 1024;
    static constexpr int kTPR = kExpThreads / BN;               // expander threads per B row
    static constexpr int kWPT = 8 / kTPR;                       // 16-byte chunks per thread per stage
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    static_assert(kTmemCols <= 512, "TMEM budget");
    static_assert(kStages >= 2, "pipeline depth");
};

__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }
__device__ __forceinline__ float sigmoid_f(float v) { return __fdividef(1.0f, 1.0f + __expf(-v)); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Expand 8 codes (one u32: nibble i = column k0+i) through the row's table.
// lo[q] / hi[q] hold the low / high bytes of entries 4q..4q+3.
__device__ __forceinline__ void lut_expand8(uint32_t w, const uint32_t (&lo)[4],
                                            const uint32_t (&hi)[4], uint32_t (&out)[4]) {
    // index within 8 entries for all eight nibbles at once (PRMT reads only
    // the low 16 bits of its selector, so half 1 takes the upper half shifted)
    const uint32_t s3a = w & 0x77777777u;
    const uint32_t s3[2] = {s3a, s3a >> 16};
    // byte i of m[h] = 0xFF where nibble i of half h is >= 8: the sign bit of
    // the byte holding that nibble's bit 3 (w for odd nibbles, w << 4 for even)
    const uint32_t w4 = w << 4;
    const uint32_t m[2] = {prmt(w, w4, 0x9D8Cu), prmt(w, w4, 0xBFAEu)};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const uint32_t l = bitsel(prmt(lo[0], lo[1], s3[half]), prmt(lo[2], lo[3], s3[half]), m[half]);
        const uint32_t h = bitsel(prmt(hi[0], hi[1], s3[half]), prmt(hi[2], hi[3], s3[half]), m[half]);
        out[2 * half + 0] = prmt(l, h, 0x5140u);  // f16 of columns 0,1 of this half
        out[2 * half + 1] = prmt(l, h, 0x7362u);  // columns 2,3
    }
}

__device__ __forceinline__ uint32_t f2u(float v) { return __float_as_uint(v); }

// 32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void load_acc32(uint32_t taddr, float* v) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr, r);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// One epilogue warp's output slab: 32 rows (one per lane) of up to 128 bytes.
// 128-byte rows use the TMA 128-byte swizzle (16-byte chunk j of row r sits at
// chunk j ^ (r & 7)), which also makes a warp's row writes bank-conflict free;
// 64-byte rows (the GLU output of a 64-column tile) are stored plainly.
template <bool SW>
__device__ __forceinline__ void slab_put(uint8_t* slab, int r, int j, uint4 v, int row_bytes) {
    const int off = SW ? r * 128 + ((j ^ (r & 7)) << 4) : r * row_bytes + (j << 4);
    *reinterpret_cast<uint4*>(slab + off) = v;
}

// An epilogue warp's NS output slabs (32 x 128 B each), used in turn: a slab
// is rewritten only after the bulk store that last read it has finished
// reading, so with NS = 2 the next slab fills while the previous one drains.
template <int NS>
struct Slabs {
    uint8_t* base;
    int idx;
    __device__ __forceinline__ uint8_t* acquire(int lane) {
        uint8_t* s = base + idx * 4096;
        idx = NS == 1 ? 0 : (idx + 1) % NS;
        if (lane == 0) bulk_wait_read<NS - 1>();
        __syncwarp();
        return s;
    }
};

// The slab goes out as one TMA tile store, or an f32 add-reduction into the
// destination (the residual update x += alpha * acc, done in L2).
__device__ __forceinline__ void slab_flush(const CUtensorMap* map, uint8_t* slab, int lane, int x, int y, bool reduce) {
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
        if (reduce)
            tma_reduce_add_2d(map, smem_u32(slab), x, y);
        else
            tma_store_2d(map, smem_u32(slab), x, y);
        bulk_commit();
    }
}

__device__ __forceinline__ void add_vec(float* v, const float* b, int n) {
    const float4* b4 = reinterpret_cast<const float4*>(b);
    for (int i = 0; i < n / 4; ++i) {
        const float4 t = __ldg(b4 + i);
        v[4 * i] += t.x;
        v[4 * i + 1] += t.y;
        v[4 * i + 2] += t.z;
        v[4 * i + 3] += t.w;
    }
}

// Packs 64 values (plus an optional per-column bias) to f16 into the slab
// (8 chunks of 16 bytes).
__device__ __forceinline__ void slab_put_f16x64(uint8_t* slab, int lane, const float* v, const float* bias) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
        if (bias) {
            b0 = __ldg(reinterpret_cast<const float4*>(bias + 8 * j));
            b1 = __ldg(reinterpret_cast<const float4*>(bias + 8 * j + 4));
        }
        slab_put<true>(slab, lane, j,
                       make_uint4(pack_h2(v[8 * j] + b0.x, v[8 * j + 1] + b0.y),
                                  pack_h2(v[8 * j + 2] + b0.z, v[8 * j + 3] + b0.w),
                                  pack_h2(v[8 * j + 4] + b1.x, v[8 * j + 5] + b1.y),
                                  pack_h2(v[8 * j + 6] + b1.z, v[8 * j + 7] + b1.w)),
                       128);
    }
}

// Epilogue of one 128-row subtile held in TMEM columns [tacc, tacc + BN):
// this warp's 32 rows start at output row y0.
template <int BN, int EPI, int NS>
__device__ __forceinline__ void epilogue_subtile(const GemmParams& p, const CUtensorMap* map_c, Slabs<NS>& slabs,
                                                 uint32_t tacc, int lane, int n0, int y0, bool with_bias) {
    if (EPI == EPI_F32 || EPI == EPI_RESID) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            float v[32];
            load_acc32(tacc + c * 32, v);
            if (EPI == EPI_F32 && p.bias && with_bias) add_vec(v, p.bias + n0 + c * 32, 32);
            if (EPI == EPI_RESID) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] *= p.alpha;
            }
            uint8_t* slab = slabs.acquire(lane);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                slab_put<true>(slab, lane, j, make_uint4(f2u(v[4 * j]), f2u(v[4 * j + 1]), f2u(v[4 * j + 2]), f2u(v[4 * j + 3])), 128);
            slab_flush(map_c, slab, lane, n0 + c * 32, y0, EPI == EPI_RESID);
        }
    } else if (EPI == EPI_F16 || EPI == EPI_SILU_F16 || EPI == EPI_QKV || EPI == EPI_RELU_F16) {
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
            const int n = n0 + c * 64;
            float v[64];
            load_acc32(tacc + c * 64, v);
            load_acc32(tacc + c * 64 + 32, v + 32);
            if (EPI == EPI_QKV) {
                // row layout [q + bias_u | q + bias_v | k | v], 1024 f16 each
                if (n < 1024) {
                    uint8_t* slab = slabs.acquire(lane);
                    slab_put_f16x64(slab, lane, v, p.bias_u + n);
                    slab_flush(map_c, slab, lane, n, y0, false);
                    slab = slabs.acquire(lane);
                    slab_put_f16x64(slab, lane, v, p.bias_v + n);
                    slab_flush(map_c, slab, lane, n + 1024, y0, false);
                } else {
                    uint8_t* slab = slabs.acquire(lane);
                    slab_put_f16x64(slab, lane, v, nullptr);
                    slab_flush(map_c, slab, lane, n + 1024, y0, false);
                }
            } else {
                if (p.bias) add_vec(v, p.bias + n, 64);
                if (EPI == EPI_SILU_F16) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) v[i] = silu_f(v[i]);
                }
                if (EPI == EPI_RELU_F16) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) v[i] = fmaxf(v[i], 0.f);
                }
                uint8_t* slab = slabs.acquire(lane);
                slab_put_f16x64(slab, lane, v, nullptr);
                slab_flush(map_c, slab, lane, n, y0, false);
            }
        }
    } else if (EPI == EPI_GLU_F16) {
        // W rows interleaved (value, gate) at load: accumulator column 2i is
        // GLU input a_i, column 2i+1 its gate b_i.  A BN-column tile gives BN/2
        // outputs: one slab row of BN bytes.
        constexpr bool kSw = (BN == 128);
        uint8_t* slab = slabs.acquire(lane);
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            float v[32];
            load_acc32(tacc + c * 32, v);
            if (p.bias) add_vec(v, p.bias + n0 + c * 32, 32);
            float g[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) g[i] = v[2 * i] * sigmoid_f(v[2 * i + 1]);
            slab_put<kSw>(slab, lane, 2 * c,
                          make_uint4(pack_h2(g[0], g[1]), pack_h2(g[2], g[3]), pack_h2(g[4], g[5]), pack_h2(g[6], g[7])), BN);
            slab_put<kSw>(slab, lane, 2 * c + 1,
                          make_uint4(pack_h2(g[8], g[9]), pack_h2(g[10], g[11]), pack_h2(g[12], g[13]), pack_h2(g[14], g[15])), BN);
        }
        slab_flush(map_c, slab, lane, n0 / 2, y0, false);
    }
}

template <int BN, int SUB, bool LUT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    k1_gemm(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
            const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    using Cfg = GemmCfg<BN, SUB, LUT>;
    constexpr int S = Cfg::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;                              // [S][SUB][128 x 64 f16]
    uint8_t* sB = smem + S * SUB * Cfg::kABytes;     // [S][BN x 64 f16]
    uint8_t* sC = sB + S * Cfg::kBBytes;             // [S][BN x 32 B]
    uint8_t* sOut = sC + S * Cfg::kCBytes;           // [4][32 x 128 B] epilogue slabs
    uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + Cfg::kOutBytes);
    uint64_t* full = bars;
    uint64_t* bready = bars + S;
    uint64_t* empty = bars + 2 * S;
    uint64_t* tfull = bars + 3 * S;       // [2]
    uint64_t* tempty = bars + 3 * S + 2;  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int ksplit = (EPI == EPI_F32 && p.ksplit > 1) ? p.ksplit : 1;   // split-K: f32 epilogue only
    const int num_k = p.K / kBK / ksplit;    // k-blocks per tile (per K part)
    const int n_tiles = p.N / BN;
    const int m_tiles = (p.M + SUB * kBM - 1) / (SUB * kBM);
    const int mn_tiles = n_tiles * m_tiles;
    const int num_tiles = mn_tiles * ksplit;  // tile = (K part, m tile, n tile)

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
        tma_prefetch_desc(&tm_c);
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&bready[s]), kExpThreads);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tfull[b]), 1);
            mbar_init(smem_u32(&tempty[b]), 128);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc<Cfg::kTmemCols>(smem_u32(tmem_slot));
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // everything above touches only this CTA's shared memory and TMEM
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        // ── TMA producer ──
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int t = EPI == EPI_F32 ? tile % mn_tiles : tile;
                const int m0 = (t / n_tiles) * SUB * kBM;
                const int n0 = (t % n_tiles) * BN;
                const int kb0 = EPI == EPI_F32 ? (tile / mn_tiles) * num_k : 0;
                for (int kb = kb0; kb < kb0 + num_k; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    if (it >= S && !(ok = mbar_wait(smem_u32(&empty[s]), ph ^ 1, 0x01))) break;
                    const uint32_t fb = smem_u32(&full[s]);
                    mbar_arrive_expect_tx(fb, SUB * Cfg::kABytes + (LUT ? Cfg::kCBytes : Cfg::kBBytes));
#pragma unroll
                    for (int sub = 0; sub < SUB; ++sub)
                        tma_load_2d(smem_u32(sA + (s * SUB + sub) * Cfg::kABytes), &tm_a, fb, kb * kBK,
                                    m0 + sub * kBM);
#pragma unroll
                    for (int r = 0; r < BN / kBoxN; ++r) {
                        if (LUT)
                            tma_load_2d(smem_u32(sC + s * Cfg::kCBytes + r * kBoxN * (kBK / 2)), &tm_b, fb,
                                        kb * (kBK / 2), n0 + r * kBoxN);
                        else
                            tma_load_2d(smem_u32(sB + s * Cfg::kBBytes + r * kBoxN * kBK * 2), &tm_b, fb,
                                        kb * kBK, n0 + r * kBoxN);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ── MMA issuer ──
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32<kBM, BN>();
            int it = 0, lt = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++lt) {
                const int b = lt & 1;
                const int use = lt >> 1;
                if (use > 0 && !(ok = mbar_wait(smem_u32(&tempty[b]), (use - 1) & 1, 0x06))) break;
                tc_fence_after();
                const uint32_t acc = tmem + b * Cfg::kAccCols;
                for (int kb = 0; kb < num_k; ++kb, ++it) {   // k-blocks of this tile's K part
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    ok = mbar_wait(smem_u32(&full[s]), ph, 0x02);
                    if (ok && LUT) ok = mbar_wait(smem_u32(&bready[s]), ph, 0x03);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t db = smem_desc_sw128(smem_u32(sB + s * Cfg::kBBytes));
                    const uint64_t da = smem_desc_sw128(smem_u32(sA + s * SUB * Cfg::kABytes));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
#pragma unroll
                        for (int sub = 0; sub < SUB; ++sub)
                            mma_f16_ss(acc + sub * BN, desc_advance(da, sub * Cfg::kABytes + kk * 32),
                                       desc_advance(db, kk * 32), idesc, kk != 0 || kb != 0);
                    }
                    mma_commit(smem_u32(&empty[s]));
                }
                if (ok) mma_commit(smem_u32(&tfull[b]));
            }
        }
    } else if (warp < kEpiWarp0) {
        // ── LUT expanders ──
        if (LUT) {
            constexpr int TPR = Cfg::kTPR, WPT = Cfg::kWPT;
            const int e = threadIdx.x - 64;
            const int row = e / TPR;           // B row within the tile
            const int w0 = (e % TPR) * WPT;    // first 16-byte chunk of this thread
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int n0 = ((EPI == EPI_F32 ? tile % mn_tiles : tile) % n_tiles) * BN;
                uint32_t lo[4], hi[4];
                {
                    const uint4* src = reinterpret_cast<const uint4*>(p.lut + static_cast<size_t>(n0 + row) * 16);
                    const uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
                    // entries (2i, 2i+1) in word i -> byte planes of 4 entries
                    lo[0] = prmt(u0.x, u0.y, 0x6420u);
                    hi[0] = prmt(u0.x, u0.y, 0x7531u);
                    lo[1] = prmt(u0.z, u0.w, 0x6420u);
                    hi[1] = prmt(u0.z, u0.w, 0x7531u);
                    lo[2] = prmt(u1.x, u1.y, 0x6420u);
                    hi[2] = prmt(u1.x, u1.y, 0x7531u);
                    lo[3] = prmt(u1.z, u1.w, 0x6420u);
                    hi[3] = prmt(u1.z, u1.w, 0x7531u);
                }
                bool ok = true;
                for (int kb = 0; kb < num_k; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    if (!(ok = mbar_wait(smem_u32(&full[s]), ph, 0x04))) break;
                    const uint8_t* codes = sC + s * Cfg::kCBytes + row * 32 + w0 * 4;
                    uint32_t wds[WPT];
                    if (WPT == 4) {
                        const uint4 c = *reinterpret_cast<const uint4*>(codes);
                        wds[0] = c.x; wds[1] = c.y; wds[2 % WPT] = c.z; wds[3 % WPT] = c.w;
                    } else if (WPT == 2) {
                        const uint2 c = *reinterpret_cast<const uint2*>(codes);
                        wds[0] = c.x; wds[1 % WPT] = c.y;
                    } else {
#pragma unroll
                        for (int j = 0; j < WPT; ++j) wds[j] = reinterpret_cast<const uint32_t*>(codes)[j];
                    }
                    uint8_t* brow = sB + s * Cfg::kBBytes + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
                    for (int j = 0; j < WPT; ++j) {
                        uint32_t o[4];
                        lut_expand8(wds[j], lo, hi, o);
                        *reinterpret_cast<uint4*>(brow + (((w0 + j) ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                    fence_async_shared();
                    mbar_arrive(smem_u32(&bready[s]));
                }
                if (!ok) break;
            }
        }
    } else {
        // ── epilogue (4 warps, one TMEM lane quarter each) ──
        const int q = warp & 3;
        Slabs<1> slabs{sOut + (warp - kEpiWarp0) * 4096, 0};
        int lt = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
            const int t = EPI == EPI_F32 ? tile % mn_tiles : tile;
            const int ks = EPI == EPI_F32 ? tile / mn_tiles : 0;
            // K part ks writes its own block of rows; the first part carries the bias
            const int m0 = ks * (ksplit > 1 ? gemm_split_rows(p.M) : 0) + (t / n_tiles) * SUB * kBM;
            const int n0 = (t % n_tiles) * BN;
            const int b = lt & 1;
            if (!mbar_wait(smem_u32(&tfull[b]), (lt >> 1) & 1, 0x05)) break;
            tc_fence_after();
            const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * Cfg::kAccCols;
#pragma unroll 1
            for (int sub = 0; sub < SUB; ++sub)
                epilogue_subtile<BN, EPI>(p, &tm_c, slabs, tq + sub * BN, lane, n0, m0 + sub * kBM + q * 32, ks == 0);
            tc_fence_before();
            mbar_arrive(smem_u32(&tempty[b]));
        }
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<Cfg::kTmemCols>(tmem);
    }
}

// ─────────────────────── K1 on CTA pairs (256 x 256 tiles) ───────────────────────
//
// A cluster of two CTAs computes one 256 x 256 tile with tcgen05.mma
// cta_group::2 (M = 256, N = 256, K = 16): CTA r holds A rows [128 r, 128 r +
// 128) and B rows (output columns) [128 r, 128 r + 128) of the tile, and its
// TMEM receives accumulator rows [128 r, 128 r + 128) x all 256 columns.  Per
// SM and k-block this moves 16 KB of A and 4 KB of codes (LUT4) instead of
// 32 KB + 4 KB for a 256 x 128 single-CTA tile at the same FLOPs, so the ring
// is deeper and L2 traffic per FLOP is ~1.8x lower.
//
// Roles per CTA are those of k1_gemm.  Only CTA 0's MMA thread issues MMAs;
// it waits on CTA 0's barriers, which count both CTAs' work:
//   full[s]    A (and f16 B) tiles of both CTAs: CTA 0 posts the expected
//              bytes of both, each CTA's TMA completes on CTA 0's barrier;
//   bready[s]  LUT4 B tiles expanded in both CTAs: one arrival per expander
//              warp of either CTA (16);
//   tempty[b]  accumulator set b drained by both CTAs' epilogues: one
//              arrival per epilogue warp (8).
// CTA-local barriers: empty[s] (stage s free again; the MMA commit arrives
// on it in both CTAs), cfull[s] (this CTA's codes landed) and tfull[b]
// (accumulator set b complete; the MMA commit arrives in both CTAs).
namespace pair {
constexpr int kBN = 256;                      // tile columns (both CTAs)
constexpr int kHalfN = 128;                   // B rows per CTA
constexpr uint32_t kABytes = kBM * kBK * 2;   // 16 KB
constexpr uint32_t kBBytes = kHalfN * kBK * 2;
constexpr uint32_t kCBytes = kHalfN * kBK / 2;
constexpr uint32_t kOutBytes = 4 * 2 * 4096;    // two slabs per epilogue warp
constexpr uint32_t kBarBytes = 512;
constexpr uint32_t kAccCols = kBN;            // one accumulator set: 256 f32 columns
constexpr uint32_t kTmemCols = 2 * kAccCols;  // double-buffered: all 512 columns
template <bool LUT>
struct Cfg {
    static constexpr uint32_t kStageBytes = kABytes + kBBytes + (LUT ? kCBytes : 0);
    static constexpr uint32_t kRingBudget = 232448 - kOutBytes - kBarBytes - 1024;
    static constexpr int kStages = kRingBudget / kStageBytes > 8 ? 8 : kRingBudget / kStageBytes;
    static constexpr uint32_t kSmemBytes = kStages * kStageBytes + kOutBytes + kBarBytes + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
    static_assert(kStages * 5 * 8 + 4 * 8 + 8 <= kBarBytes, "barrier space");
};
}  // namespace pair

template <bool LUT, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    k1_gemm_pair(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                 const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
    using Cfg = pair::Cfg<LUT>;
    constexpr int S = Cfg::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // identical offsets in both CTAs: the MMA addresses the peer's tiles by them
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;                              // [S][128 x 64 f16]
    uint8_t* sB = smem + S * pair::kABytes;          // [S][128 x 64 f16]
    uint8_t* sC = sB + S * pair::kBBytes;            // [S][128 x 32 B] (LUT4)
    uint8_t* sOut = sC + (LUT ? S * pair::kCBytes : 0);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + pair::kOutBytes);
    uint64_t* full = bars;
    uint64_t* bready = bars + S;
    uint64_t* empty = bars + 2 * S;
    uint64_t* cfull = bars + 3 * S;
    uint64_t* tfull = bars + 4 * S;       // [2]
    uint64_t* tempty = bars + 4 * S + 2;  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * S + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair_id = blockIdx.x >> 1;
    const int n_pairs = gridDim.x >> 1;
    const int num_k = p.K / kBK;
    const int n_tiles = p.N / pair::kBN;
    const int m_tiles = (p.M + 2 * kBM - 1) / (2 * kBM);
    const int num_tiles = n_tiles * m_tiles;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
        tma_prefetch_desc(&tm_c);
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&bready[s]), 16);
            mbar_init(smem_u32(&empty[s]), 1);
            mbar_init(smem_u32(&cfull[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tfull[b]), 1);
            mbar_init(smem_u32(&tempty[b]), 8);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair<pair::kTmemCols>(smem_u32(tmem_slot));
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();   // barriers of both CTAs initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ── TMA producer (both CTAs) ──
        if (lane == 0) {
            const uint32_t full0 = mapa_shared(smem_u32(full), 0);   // CTA 0's full[0]
            int it = 0;
            bool ok = true;
            for (int tile = pair_id; tile < num_tiles && ok; tile += n_pairs) {
                const int m0 = (tile / n_tiles) * 2 * kBM + rank * kBM;
                const int n0 = (tile % n_tiles) * pair::kBN + rank * pair::kHalfN;
                for (int kb = 0; kb < num_k; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    if (it >= S && !(ok = mbar_wait(smem_u32(&empty[s]), ph ^ 1, 0x11))) break;
                    const uint32_t fb = full0 + s * 8;
                    if (rank == 0)
                        mbar_arrive_expect_tx(smem_u32(&full[s]), 2 * (pair::kABytes + (LUT ? 0 : pair::kBBytes)));
                    tma_load_2d_pair(smem_u32(sA + s * pair::kABytes), &tm_a, fb, kb * kBK, m0);
                    if (LUT) {
                        const uint32_t cb = smem_u32(&cfull[s]);
                        mbar_arrive_expect_tx(cb, pair::kCBytes);
#pragma unroll
                        for (int r = 0; r < pair::kHalfN / kBoxN; ++r)
                            tma_load_2d(smem_u32(sC + s * pair::kCBytes + r * kBoxN * (kBK / 2)), &tm_b, cb,
                                        kb * (kBK / 2), n0 + r * kBoxN);
                    } else {
#pragma unroll
                        for (int r = 0; r < pair::kHalfN / kBoxN; ++r)
                            tma_load_2d_pair(smem_u32(sB + s * pair::kBBytes + r * kBoxN * kBK * 2), &tm_b, fb,
                                             kb * kBK, n0 + r * kBoxN);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ── MMA issuer (CTA 0 only) ──
        if (rank == 0 && lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32<2 * kBM, pair::kBN>();
            int it = 0, lt = 0;
            bool ok = true;
            for (int tile = pair_id; tile < num_tiles && ok; tile += n_pairs, ++lt) {
                const int b = lt & 1;
                const int use = lt >> 1;
                if (use > 0 && !(ok = mbar_wait_cluster(smem_u32(&tempty[b]), (use - 1) & 1, 0x16))) break;
                tc_fence_after();
                const uint32_t acc = tmem + b * pair::kAccCols;
                for (int kb = 0; kb < num_k; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    ok = mbar_wait_cluster(smem_u32(&full[s]), ph, 0x12);
                    if (ok && LUT) ok = mbar_wait(smem_u32(&bready[s]), ph, 0x13);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t da = smem_desc_sw128(smem_u32(sA + s * pair::kABytes));
                    const uint64_t db = smem_desc_sw128(smem_u32(sB + s * pair::kBBytes));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_f16_ss_pair(acc, desc_advance(da, kk * 32), desc_advance(db, kk * 32), idesc,
                                        kk != 0 || kb != 0);
                    mma_commit_pair_mc(smem_u32(&empty[s]), 0x3);
                }
                if (ok) mma_commit_pair_mc(smem_u32(&tfull[b]), 0x3);
            }
        }
    } else if (warp < kEpiWarp0) {
        // ── LUT expanders (both CTAs): this CTA's 128 B rows ──
        if (LUT) {
            constexpr int TPR = kExpThreads / pair::kHalfN, WPT = 8 / TPR;
            const int e = threadIdx.x - 64;
            const int row = e / TPR;
            const int w0 = (e % TPR) * WPT;
            const uint32_t bready0 = mapa_shared(smem_u32(bready), 0);
            int it = 0;
            for (int tile = pair_id; tile < num_tiles; tile += n_pairs) {
                const int n0 = (tile % n_tiles) * pair::kBN + rank * pair::kHalfN;
                uint32_t lo[4], hi[4];
                {
                    const uint4* src = reinterpret_cast<const uint4*>(p.lut + static_cast<size_t>(n0 + row) * 16);
                    const uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
                    lo[0] = prmt(u0.x, u0.y, 0x6420u);
                    hi[0] = prmt(u0.x, u0.y, 0x7531u);
                    lo[1] = prmt(u0.z, u0.w, 0x6420u);
                    hi[1] = prmt(u0.z, u0.w, 0x7531u);
                    lo[2] = prmt(u1.x, u1.y, 0x6420u);
                    hi[2] = prmt(u1.x, u1.y, 0x7531u);
                    lo[3] = prmt(u1.z, u1.w, 0x6420u);
                    hi[3] = prmt(u1.z, u1.w, 0x7531u);
                }
                bool ok = true;
                for (int kb = 0; kb < num_k; ++kb, ++it) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    if (!(ok = mbar_wait(smem_u32(&cfull[s]), ph, 0x14))) break;
                    const uint8_t* codes = sC + s * pair::kCBytes + row * 32 + w0 * 4;
                    const uint4 c = *reinterpret_cast<const uint4*>(codes);
                    const uint32_t wds[4] = {c.x, c.y, c.z, c.w};
                    uint8_t* brow = sB + s * pair::kBBytes + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
                    for (int j = 0; j < WPT; ++j) {
                        uint32_t o[4];
                        lut_expand8(wds[j], lo, hi, o);
                        *reinterpret_cast<uint4*>(brow + (((w0 + j) ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                    fence_async_shared();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(bready0 + s * 8);
                }
                if (!ok) break;
            }
        }
    } else {
        // ── epilogue (both CTAs): 4 warps, one TMEM lane quarter each ──
        const int q = warp & 3;
        Slabs<2> slabs{sOut + (warp - kEpiWarp0) * 8192, 0};
        const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
        int lt = 0;
        for (int tile = pair_id; tile < num_tiles; tile += n_pairs, ++lt) {
            const int m0 = (tile / n_tiles) * 2 * kBM + rank * kBM;
            const int n0 = (tile % n_tiles) * pair::kBN;
            const int b = lt & 1;
            if (!mbar_wait(smem_u32(&tfull[b]), (lt >> 1) & 1, 0x15)) break;
            tc_fence_after();
            const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * pair::kAccCols;
#pragma unroll 1
            for (int h = 0; h < 2; ++h)
                epilogue_subtile<128, EPI>(p, &tm_c, slabs, tq + h * 128, lane, n0 + h * 128, m0 + q * 32, true);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + b * 8);
        }
        if (lane == 0) bulk_wait_all();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();   // no CTA leaves while the pair MMA or a remote arrival may touch it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair<pair::kTmemCols>(tmem);
    }
}

// Output map of one epilogue warp's slab (32 rows of 128 bytes, or the GLU
// output of a 128-column half tile), shared by both kernels.
template <int EPI>
int make_out_map(CUtensorMap* tc, const GemmParams& p, int ksplit) {
    if (EPI == EPI_F32 || EPI == EPI_RESID)
        return make_map_2d(tc, p.out_f32, kMapF32, p.N,
                           ksplit > 1 ? static_cast<uint64_t>(ksplit) * gemm_split_rows(p.M) : p.M,
                           static_cast<uint64_t>(p.ldo) * 4, 32, 32, true);
    if (EPI == EPI_GLU_F16)
        return make_map_2d(tc, p.out_f16, kMapF16, p.N / 2, p.M, static_cast<uint64_t>(p.ldo) * 2, 64, 32, true);
    if (EPI == EPI_QKV)
        return make_map_2d(tc, p.out_f16, kMapF16, 4096, p.M, static_cast<uint64_t>(p.ldo) * 2, 64, 32, true);
    return make_map_2d(tc, p.out_f16, kMapF16, p.N, p.M, static_cast<uint64_t>(p.ldo) * 2, 64, 32, true);
}

template <bool LUT, int EPI>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st);

template <int BN, int SUB, bool LUT, int EPI>
int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    using Cfg = GemmCfg<BN, SUB, LUT>;
    auto kern = k1_gemm<BN, SUB, LUT, EPI>;
    static PerDeviceOnce smem_once;  // per template instance
    const int rc0 = set_smem_limit_once(smem_once, kern, static_cast<int>(Cfg::kSmemBytes), "cudaFuncSetAttribute(k1_gemm)");
    if (rc0) return rc0;
    const int g_num_sms = device_sms();
    // output map: 32-row boxes of 128-byte rows (64-byte rows for the GLU
    // output of a 64-column tile), matching the epilogue's slab layout
    CUtensorMap tc;
    const int ksplit = p.ksplit > 1 ? p.ksplit : 1;
    int rc;
    if (EPI == EPI_GLU_F16 && BN != 128)
        rc = make_map_2d(&tc, p.out_f16, kMapF16, p.N / 2, p.M, static_cast<uint64_t>(p.ldo) * 2, BN / 2, 32, false);
    else
        rc = make_out_map<EPI>(&tc, p, ksplit);
    if (rc) return rc;
    const int tiles = (p.N / BN) * ((p.M + SUB * kBM - 1) / (SUB * kBM)) * ksplit;
    const int grid = tiles < g_num_sms ? tiles : g_num_sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, p);
    if (e != cudaSuccess) return set_cuda_error("k1_gemm launch", e);
    return 0;
}

template <int BN, int SUB, bool LUT>
int launch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    switch (epi) {
        case EPI_F32: return launch_one<BN, SUB, LUT, EPI_F32>(ta, tb, p, st);
        case EPI_RESID: return launch_one<BN, SUB, LUT, EPI_RESID>(ta, tb, p, st);
        case EPI_F16: return launch_one<BN, SUB, LUT, EPI_F16>(ta, tb, p, st);
        case EPI_SILU_F16: return launch_one<BN, SUB, LUT, EPI_SILU_F16>(ta, tb, p, st);
        case EPI_GLU_F16: return launch_one<BN, SUB, LUT, EPI_GLU_F16>(ta, tb, p, st);
        case EPI_QKV: return launch_one<BN, SUB, LUT, EPI_QKV>(ta, tb, p, st);
        case EPI_RELU_F16: return launch_one<BN, SUB, LUT, EPI_RELU_F16>(ta, tb, p, st);
        default: return set_error(B3_EINVAL, "unknown GEMM epilogue %d", epi);
    }
}

template <bool LUT, int EPI>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    using Cfg = pair::Cfg<LUT>;
    auto kern = k1_gemm_pair<LUT, EPI>;
    static PerDeviceOnce smem_once;  // per template instance
    const int rc0 = set_smem_limit_once(smem_once, kern, static_cast<int>(Cfg::kSmemBytes),
                                        "cudaFuncSetAttribute(k1_gemm_pair)");
    if (rc0) return rc0;
    CUtensorMap tc;
    int rc = make_out_map<EPI>(&tc, p, 1);
    if (rc) return rc;
    const int tiles = (p.N / pair::kBN) * ((p.M + 2 * kBM - 1) / (2 * kBM));
    const int g_num_sms = device_sms();
    const int pairs = tiles < g_num_sms / 2 ? tiles : g_num_sms / 2;
    kern<<<2 * pairs, kThreads, Cfg::kSmemBytes, st>>>(ta, tb, tc, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("k1_gemm_pair launch", e);
    return 0;
}

template <bool LUT>
int launch_pair_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    switch (epi) {
        case EPI_F32: return launch_pair<LUT, EPI_F32>(ta, tb, p, st);
        case EPI_RESID: return launch_pair<LUT, EPI_RESID>(ta, tb, p, st);
        case EPI_F16: return launch_pair<LUT, EPI_F16>(ta, tb, p, st);
        case EPI_SILU_F16: return launch_pair<LUT, EPI_SILU_F16>(ta, tb, p, st);
        case EPI_GLU_F16: return launch_pair<LUT, EPI_GLU_F16>(ta, tb, p, st);
        case EPI_QKV: return launch_pair<LUT, EPI_QKV>(ta, tb, p, st);
        case EPI_RELU_F16: return launch_pair<LUT, EPI_RELU_F16>(ta, tb, p, st);
        default: return set_error(B3_EINVAL, "unknown GEMM epilogue %d", epi);
    }
}

}  // namespace

// Reads and clears this translation unit's device error word (stream-ordered).
int gemm_take_dev_error(cudaStream_t st, unsigned int* out) {
    static const unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_b3_dev_error, sizeof(unsigned int), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbolAsync(g_b3_dev_error, &zero, sizeof(unsigned int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? 0 : set_cuda_error("reading the device error word", e);
}

int gemm_validate(const GemmParams& p, bool lut) {
    if (p.M <= 0 || p.N <= 0 || p.K <= 0)
        return set_error(B3_EINVAL, "GEMM sizes must be positive (M=%d N=%d K=%d)", p.M, p.N, p.K);
    if (p.K % kBK) return set_error(B3_EINVAL, "GEMM K=%d must be a multiple of %d", p.K, kBK);
    if (p.N % 128) return set_error(B3_EINVAL, "GEMM N=%d must be a multiple of 128", p.N);
    if (lut && !p.lut) return set_error(B3_EINVAL, "LUT4 GEMM needs a level table");
    if (p.ksplit > 1 && (p.K / kBK) % p.ksplit)
        return set_error(B3_EINVAL, "GEMM split-K: %d parts do not divide %d k-blocks", p.ksplit, p.K / kBK);
    return 0;
}

void gemm_plan_split(int M, int N, int K, bool lut, int num_sms, int max_parts, int* tiles, int* ksplit) {
    // cost of one SM's share: waves x (k-blocks per part x bytes per k-block
    // + a fixed per-tile cost of about two k-blocks for the fill and the
    // epilogue); parts of fewer than 2 k-blocks are not considered
    const int nk = K / kBK;
    double best = 1e300;
    *tiles = 1;
    *ksplit = 1;
    for (int shape = 1; shape <= 2; ++shape) {
        const int bn = shape == 2 ? 128 : 64, bm = shape == 2 ? 256 : 128;
        if (N % bn) continue;
        const double kb_bytes = (bm * kBK * 2.0) + (lut ? bn * kBK / 2.0 : bn * kBK * 2.0);
        const long t = static_cast<long>(N / bn) * ((M + bm - 1) / bm);
        for (int s = 1; s <= nk; ++s) {
            if (nk % s || s > max_parts || (s > 1 && nk / s < 2)) continue;
            const long units = t * s;
            const long waves = (units + num_sms - 1) / num_sms;
            const double cost = waves * ((nk / s + 2) * kb_bytes);
            if (cost < best * 0.999) {
                best = cost;
                *tiles = shape;
                *ksplit = s;
            }
        }
    }
}

// Tile shape by problem size: large problems take 256 x 128 tiles (two MMAs
// share each expanded B tile); small ones take 128 x 64 tiles to spread over
// the SMs.
int gemm_launch(const GemmOp& op, cudaStream_t st) {
    const GemmParams& p = op.p;
    int rc = gemm_validate(p, op.lut);
    if (rc) return rc;
    // 256 x 128 tiles as soon as they fill every SM once; below that the
    // 128 x 64 tiles win by spreading the work.
    const long big_tiles = static_cast<long>(p.N / 128) * ((p.M + 255) / 256);
    const bool big = p.tiles ? p.tiles == 2 : big_tiles >= 148;
    if (p.ksplit > 1 && op.epi != EPI_F32) return set_error(B3_EINVAL, "GEMM split-K needs the f32 epilogue");
    // CTA pairs with 256 x 256 tiles once they fill every SM pair once
    const int g_num_sms = device_sms();
    const long pair_tiles = static_cast<long>(p.N / 256) * ((p.M + 255) / 256);
    const bool use_pair = p.tiles ? p.tiles == 3 : (p.N % 256 == 0 && p.ksplit <= 1 && pair_tiles >= g_num_sms / 2);
    if (use_pair) {
        if (p.N % 256) return set_error(B3_EINVAL, "GEMM pair tiles need N %% 256 == 0 (N=%d)", p.N);
        return op.lut ? launch_pair_epi<true>(op.epi, op.map_a, op.map_b, p, st)
                      : launch_pair_epi<false>(op.epi, op.map_a, op.map_b, p, st);
    }
    if (op.lut) {
        if (big) return launch_epi<128, 2, true>(op.epi, op.map_a, op.map_b, p, st);
        return launch_epi<64, 1, true>(op.epi, op.map_a, op.map_b, p, st);
    }
    if (big) return launch_epi<128, 2, false>(op.epi, op.map_a, op.map_b, p, st);
    return launch_epi<64, 1, false>(op.epi, op.map_a, op.map_b, p, st);
}

// ───────────────────────────── tensor maps ─────────────────────────────

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}
}  // namespace

int make_map_2d(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(B3_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15))
        return set_error(B3_EINVAL, "TMA base/stride must be 16-byte aligned");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = dtype == kMapF32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : dtype == kMapF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    CUresult r = fn(map, dt, 2,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(B3_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return 0;
}

int make_map_3d(CUtensorMap* map, const void* base, int dtype, const uint64_t dims[3], const uint64_t stride_bytes[2],
                const uint32_t box[3], bool swizzle128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(B3_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (stride_bytes[0] & 15) || (stride_bytes[1] & 15))
        return set_error(B3_EINVAL, "TMA base/stride must be 16-byte aligned");
    cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    cuuint64_t st[2] = {stride_bytes[0], stride_bytes[1]};
    cuuint32_t bx[3] = {box[0], box[1], box[2]};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt = dtype == kMapF32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : dtype == kMapF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    CUresult r = fn(map, dt, 3, const_cast<void*>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(B3_ECUDA, "cuTensorMapEncodeTiled (3D) failed (%d)", static_cast<int>(r));
    return 0;
}

int gemm_make_a_map(CUtensorMap* map, const __half* a, int M, int K, int lda) {
    return make_map_2d(map, a, true, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
                       static_cast<uint64_t>(lda) * 2, kBK, kBM, true);
}

// B boxes are 64 rows tall whatever the tile width; the producer issues
// BN / 64 of them per stage.
int gemm_make_b_map(CUtensorMap* map, const void* w, bool lut, int N, int K) {
    if (lut)
        return make_map_2d(map, w, false, static_cast<uint64_t>(K / 2), static_cast<uint64_t>(N),
                           static_cast<uint64_t>(K / 2), kBK / 2, kBoxN, false);
    return make_map_2d(map, w, true, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                       static_cast<uint64_t>(K) * 2, kBK, kBoxN, true);
}

}  // namespace b3
