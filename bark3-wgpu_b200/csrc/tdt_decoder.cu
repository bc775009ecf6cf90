// tdt_decoder.cu — batched greedy TDT decoding (the reference decodes one
// utterance at a time on the CPU, src/tdt.rs:416-467, or with one WGSL
// workgroup set per step, src/tdt_gpu.rs).
//
// All utterances of a batch advance in lock step: one step is
//   joint input   x_b = ReLU(enc_b[frame_b] + dec_b)
//   joint GEMM    scores = x . head^T + bias                    (tensor cores)
//   argmax/update first-max token over the vocabulary, first-max duration
//                 over the 5 duration rows; blank advances >= 1 frame, a
//                 token is recorded and advances `duration` frames
//   LSTM layer 0  gates = E0[token] + h0 . W_hh^T          (tensor cores) + cell
//   LSTM layer 1  gates = [h0 | h1] . [W_ih | W_hh]^T + b  (tensor cores) + cell
//   projector     dec = h1 . W_p^T + b                     (tensor cores)
// E0[v] = W_ih0 . emb(v) + b_ih0 + b_hh0 is computed once per vocabulary
// entry at load, so layer 0's GEMM only carries the recurrent half.  Rows
// that did not emit keep their LSTM state (their gates are computed and
// dropped), so recomputing dec for them reproduces the same value.  The whole
// decode is one cooperative launch of k_dec_persist (below).
//
// The GEMMs have M = batch rows only, so they run split-K over all SMs; every
// consumer adds the K parts in a fixed order (deterministic).
//
// Precision: each GEMM input x is split into f16 hi = f16(x) and
// lo = f16(x - hi) and the weight is repeated along K ([W | W]), so the
// tensor cores see ~22 significant bits of every activation against the
// reference's f16 weights with f32 accumulation.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "b3_internal.h"
#include "b3_kernels.h"
#include "b3_ptx.cuh"

namespace b3 {

namespace {

constexpr int kH = 640;
constexpr int kMaxParts = 8;   // split-K parts a consumer adds (the host plans at most this many)

__device__ __forceinline__ void split_store(__half* hi, __half* lo, float v) {
    const __half h = __float2half_rn(v);
    *hi = h;
    *lo = __float2half_rn(v - __half2float(h));
}

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

// Sum of the K parts of the 4 columns [j, j + 4) of row b of a split-K output
// with n columns: every part's load is issued before the first add.
__device__ __forceinline__ float4 parts_sum4(const float* base, int parts, int prow, int n, int b, int j) {
    const float* q = base + static_cast<size_t>(b) * n + j;
    const size_t stride = static_cast<size_t>(prow) * n;
    float4 v[kMaxParts];
#pragma unroll
    for (int p = 0; p < kMaxParts; ++p)
        v[p] = p < parts ? __ldcg(reinterpret_cast<const float4*>(q + p * stride)) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 r = v[0];
#pragma unroll
    for (int p = 1; p < kMaxParts; ++p) {
        if (p < parts) {
            r.x += v[p].x;
            r.y += v[p].y;
            r.z += v[p].z;
            r.w += v[p].w;
        }
    }
    return r;
}

__device__ __forceinline__ float parts_sum1(const float* base, int parts, int prow, int n, int b, int j) {
    const float* q = base + static_cast<size_t>(b) * n + j;
    const size_t stride = static_cast<size_t>(prow) * n;
    float v[kMaxParts];
#pragma unroll
    for (int p = 0; p < kMaxParts; ++p) v[p] = p < parts ? __ldcg(q + p * stride) : 0.f;
    float r = v[0];
#pragma unroll
    for (int p = 1; p < kMaxParts; ++p)
        if (p < parts) r += v[p];
    return r;
}

// 4 values as f16 hi | lo halves at hi[0..3] and lo[0..3].
__device__ __forceinline__ void split_store4(__half* hi, __half* lo, float4 v) {
    const __half2 h01 = __floats2half2_rn(v.x, v.y), h23 = __floats2half2_rn(v.z, v.w);
    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
    const __half2 l01 = __floats2half2_rn(v.x - f01.x, v.y - f01.y), l23 = __floats2half2_rn(v.z - f23.x, v.w - f23.y);
    uint2 uh, ul;
    uh.x = *reinterpret_cast<const uint32_t*>(&h01);
    uh.y = *reinterpret_cast<const uint32_t*>(&h23);
    ul.x = *reinterpret_cast<const uint32_t*>(&l01);
    ul.y = *reinterpret_cast<const uint32_t*>(&l23);
    *reinterpret_cast<uint2*>(hi) = uh;
    *reinterpret_cast<uint2*>(lo) = ul;
}

// Initial state: h = c = 0, every row runs one LSTM step on the blank
// embedding (src/tdt.rs:424-428).
__global__ void k_dec_init(DecState s) {
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.x;
    if (b >= s.B) return;
    const int T = s.len[b];
    const __half z = __float2half_rn(0.f);
    for (int j = threadIdx.x; j < kH; j += blockDim.x) {
        __half* a0 = s.a0 + static_cast<size_t>(b) * 2 * kH;
        __half* a1 = s.a1 + static_cast<size_t>(b) * 4 * kH;
        a0[j] = z;
        a0[kH + j] = z;
        a1[2 * kH + j] = z;
        a1[3 * kH + j] = z;
        s.c[(static_cast<size_t>(b) * 2 + 0) * kH + j] = 0.f;
        s.c[(static_cast<size_t>(b) * 2 + 1) * kH + j] = 0.f;
    }
    if (threadIdx.x == 0) {
        s.tok[b] = s.blank;
        s.frame[b] = 0;
        s.count[b] = 0;
        s.guard[b] = 0;
        s.emit[b] = 1;
        s.active[b] = T > 0 ? 1 : 0;
    }
}

// (value, index) pair that wins under the reference's strict `>` scan:
// larger value, or the lower index on a tie.
__device__ __forceinline__ bool wins(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (wins(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

// Embedding rows as f16 hi | lo (load time).
__global__ void k_split_rows(const float* __restrict__ src, __half* hi, __half* lo, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        split_store(hi + i, lo + i, src[i]);
}

// ─────────────────────── persistent decoder (one launch) ───────────────────────
//
// The lock step above as ONE cooperative launch: every CTA stays resident
// (one per SM) and the step's six dependent phases are separated by grid
// barriers instead of kernel boundaries:
//   A  joint head GEMM  +  layer-0 recurrent GEMM (h0 is not changed by the
//      argmax, so both read inputs that are ready)
//   B  argmax + state update, then the layer-0 cell for the rows that emitted
//   C  layer-1 GEMM        D  layer-1 cell
//   E  projector GEMM      F  joint input x = ReLU(enc[frame] + dec)
// The first pass runs C..F after a layer-0 step on the blank token (A without
// the head, B without the argmax), as the reference starts (src/tdt.rs:424-428).
//
// GEMM phases are warp-specialised like K1: warp 0 issues TMA loads, warp 1
// issues tcgen05.mma (M 128, N = 128 or 256, f32 accumulators in TMEM, two
// buffers), warps 4..7 drain the accumulators to the split-K parts.  A work
// item is (GEMM, 128-row tile, BN-column tile, K part); items are dealt
// round-robin to the CTAs.  Activations are [hi | lo] f16 halves per 640-wide
// segment and the weights are stored doubled to match ([W | W]); a stage holds
// one 64-wide logical k-block: the hi and lo A boxes and ONE weight tile, and
// the MMAs of both halves read that tile, so every weight byte crosses L2 once
// per item.  The batch is small (M = rows), so these GEMMs are bound by the
// bytes each SM pulls from L2, not by the tensor cores.
// Row phases give each row to one half of a CTA (128 threads) and issue the
// loads a phase needs together, so a phase costs one or two L2 round trips.
// Activations written by the row phases are read by the next GEMM phase
// through TMA (async proxy): writers and the TMA issuer fence the proxies
// around the grid barrier.
constexpr int kPThreads = 256;
constexpr int kPStages = 3;
constexpr uint32_t kPABytes = 128 * 64 * 2;             // one A box (hi or lo)
constexpr uint32_t kPBBytes = 256 * 64 * 2;             // weight tile, up to 256 rows
constexpr uint32_t kPStageBytes = 2 * kPABytes + kPBBytes;
constexpr uint32_t kPSlabOff = kPStages * kPStageBytes;  // [4 warps][2] 32 x 32 f32 output slabs
constexpr uint32_t kPBarOff = kPSlabOff + 8 * 4096;
constexpr uint32_t kPBiasOff = kPBarOff + 256;           // [256] f32 item bias
constexpr uint32_t kPSmem = kPBiasOff + 1024 + 1024;    // + alignment slack
static_assert(kPSmem <= 232448, "shared memory budget");
constexpr uint32_t kPTmemCols = 512;                    // two 256-column accumulators
constexpr int kPSegK = 640;                             // logical K of one [hi | lo] segment

struct PItem {
    int g, m0, n0, bn, kb0, nkb, part;
};

// Item j of a phase's GEMM list (GEMMs in order, each part-major then m, n).
__device__ __forceinline__ PItem p_item(const DecPersist& p, int g0, int g1, int j) {
    for (int i = 0; i < 2; ++i) {
        const int gi = i == 0 ? g0 : g1;
        if (gi < 0) continue;
        const DecGemm& G = p.g[gi];
        const int mn = G.m_tiles * G.n_tiles;
        if (j < mn * G.ks) {
            const int part = j / mn, t = j % mn;
            return PItem{gi, (t / G.n_tiles) * 128, (t % G.n_tiles) * G.bn, G.bn, part * G.nkb, G.nkb, part};
        }
        j -= mn * G.ks;
    }
    return PItem{-1, 0, 0, 0, 0, 0, 0};
}

__device__ __forceinline__ int p_items(const DecPersist& p, int g0, int g1) {
    int n = 0;
    if (g0 >= 0) n += p.g[g0].m_tiles * p.g[g0].n_tiles * p.g[g0].ks;
    if (g1 >= 0) n += p.g[g1].m_tiles * p.g[g1].n_tiles * p.g[g1].ks;
    return n;
}

struct PRing {
    uint8_t* ring;
    uint8_t* slabs;
    float* bias;   // [256] the epilogue's current item bias
    uint64_t* full;
    uint64_t* empty;
    uint64_t* tfull;
    uint64_t* tempty;
    uint32_t tmem;
};

// One GEMM phase on this CTA.  The role counters (`pit` ring slot of the
// producer, `mit` of the MMA issuer, `acc` accumulator uses of the MMA issuer
// and of the epilogue) persist across phases.  Returns false on a timed-out
// wait.
__device__ __forceinline__ bool p_gemm_phase(const DecMaps& maps, const DecPersist& p, const PRing& r, int g0,
                                             int g1, int& pit, int& mit, int& acc) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = p_items(p, g0, g1);
    bool ok = true;
    if (warp == 0) {
        if (lane == 0) {
            fence_async_global();   // row-phase writes -> the TMA reads below
            for (int j = blockIdx.x; j < n_items && ok; j += gridDim.x) {
                const PItem it = p_item(p, g0, g1, j);
                for (int kb = 0; kb < it.nkb; ++kb, ++pit) {
                    const int s = pit % kPStages;
                    if (pit >= kPStages && !(ok = mbar_wait(smem_u32(&r.empty[s]), ((pit / kPStages) & 1) ^ 1, 0x61)))
                        break;
                    const int k = (it.kb0 + kb) * 64;                       // logical k
                    const int x = (k / kPSegK) * 2 * kPSegK + k % kPSegK;  // its hi column
                    const uint32_t fb = smem_u32(&r.full[s]);
                    uint8_t* st = r.ring + s * kPStageBytes;
                    mbar_arrive_expect_tx(fb, 2 * kPABytes + it.bn * 128);
                    tma_load_2d(smem_u32(st), &maps.a[it.g], fb, x, it.m0);
                    tma_load_2d(smem_u32(st + kPABytes), &maps.a[it.g], fb, x + kPSegK, it.m0);
                    for (int q = 0; q < it.bn / 64; ++q)
                        tma_load_2d(smem_u32(st + 2 * kPABytes + q * 8192), &maps.b[it.g], fb, x, it.n0 + 64 * q);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int j = blockIdx.x; j < n_items && ok; j += gridDim.x, ++acc) {
                const PItem it = p_item(p, g0, g1, j);
                const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(it.bn >> 3) << 17) | ((128u >> 4) << 24);
                const int b = acc & 1, use = acc >> 1;
                if (use > 0 && !(ok = mbar_wait(smem_u32(&r.tempty[b]), (use - 1) & 1, 0x62))) break;
                tc_fence_after();
                const uint32_t d = r.tmem + b * 256;
                for (int kb = 0; kb < it.nkb; ++kb, ++mit) {
                    const int s = mit % kPStages;
                    if (!(ok = mbar_wait(smem_u32(&r.full[s]), (mit / kPStages) & 1, 0x63))) break;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(r.ring + s * kPStageBytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t bd = smem_desc_sw128(a0 + 2 * kPABytes + kk * 32);
                        mma_f16_ss(d, smem_desc_sw128(a0 + kk * 32), bd, idesc, (kb | kk) != 0);
                        mma_f16_ss(d, smem_desc_sw128(a0 + kPABytes + kk * 32), bd, idesc, 1u);
                    }
                    mma_commit(smem_u32(&r.empty[s]));
                }
                if (ok) mma_commit(smem_u32(&r.tfull[b]));
            }
        }
    } else if (warp >= 4) {
        int slab = 0;
        // The four epilogue warps meet at named barrier 3 twice per item
        // whatever happens (a timed-out wait skips the work, not the
        // barriers), so the barrier count always matches.
        const int q = warp & 3;
        for (int j = blockIdx.x; j < n_items; j += gridDim.x, ++acc) {
            const PItem it = p_item(p, g0, g1, j);
            const int b = acc & 1;
            const DecGemm& G = p.g[it.g];
            const bool bias = it.part == 0 && G.bias;
            // the item's bias into shared memory while its MMAs run (one
            // load per thread instead of a dependent load per column chunk)
            if (bias) {
                const int e = threadIdx.x - 128;
                if (e < it.bn / 2)
                    reinterpret_cast<float2*>(r.bias)[e] = __ldg(reinterpret_cast<const float2*>(G.bias + it.n0) + e);
            }
            asm volatile("bar.sync 3, 128;" ::: "memory");
            bool got = ok && mbar_wait(smem_u32(&r.tfull[b]), (acc >> 1) & 1, 0x64);
            got = __all_sync(0xffffffffu, got);
            if (!got) ok = false;
            if (got) {
                tc_fence_after();
                // 32 x 32 f32 slabs (128-byte swizzle: 16-byte chunk i of row
                // r at chunk i ^ (r & 7), conflict-free) leave by TMA tile
                // stores, two slabs per warp in turn; rows past the batch are
                // written too (they stay inside the part's rows, never read)
                const int y = it.part * p.s.prow + it.m0 + q * 32;
                const uint32_t tq = r.tmem + (static_cast<uint32_t>(q * 32) << 16) + b * 256;
                const int nc = it.bn / 32;   // 4 or 8
                // one 32-column chunk in registers -> bias -> slab -> TMA store
                auto put = [&](uint32_t (&v)[32], int c) {
                    if (bias) {
                        const float4* b4 = reinterpret_cast<const float4*>(r.bias + c * 32);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 t = b4[i];
                            v[4 * i] = __float_as_uint(__uint_as_float(v[4 * i]) + t.x);
                            v[4 * i + 1] = __float_as_uint(__uint_as_float(v[4 * i + 1]) + t.y);
                            v[4 * i + 2] = __float_as_uint(__uint_as_float(v[4 * i + 2]) + t.z);
                            v[4 * i + 3] = __float_as_uint(__uint_as_float(v[4 * i + 3]) + t.w);
                        }
                    }
                    uint8_t* sl = r.slabs + ((q * 2 + (slab & 1)) << 12);
                    ++slab;
                    if (lane == 0) bulk_wait_read<1>();   // the store that last read this slab is done reading
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *reinterpret_cast<uint4*>(sl + lane * 128 + ((i ^ (lane & 7)) << 4)) =
                            make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    fence_async_shared();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&maps.c[it.g], smem_u32(sl), it.n0 + c * 32, y);
                        bulk_commit();
                    }
                };
                // two register sets: the next chunk loads from TMEM while the
                // current one is stored
                uint32_t va[32], vb[32];
                tmem_ld_32x32b_x32(tq, va);
                tmem_wait_ld();
                for (int c = 0; c < nc; c += 2) {
                    tmem_ld_32x32b_x32(tq + (c + 1) * 32, vb);
                    put(va, c);
                    tmem_wait_ld();
                    if (c + 2 < nc) tmem_ld_32x32b_x32(tq + (c + 2) * 32, va);
                    put(vb, c + 1);
                    tmem_wait_ld();
                }
                tc_fence_before();
                mbar_arrive(smem_u32(&r.tempty[b]));
            }
            asm volatile("bar.sync 3, 128;" ::: "memory");   // bias slot free for the next item
        }
        // the phase's parts are complete in global memory before the grid barrier
        if (lane == 0) {
            bulk_wait_all();
            fence_async_global();
        }
        __syncwarp();
    }
    return ok;
}

__device__ __forceinline__ void half_sync(int h) { asm volatile("bar.sync %0, 128;" ::"r"(1 + h) : "memory"); }

__device__ __forceinline__ int ldcg_i(const int* p) { return __ldcg(p); }

// The four gate pre-activations (summed over the split-K parts) of columns
// [4 j4, 4 j4 + 4) of row b.
__device__ __forceinline__ void p_gates(const DecState& s, int parts, int b, int j4, float4 (&g)[4]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) g[q] = parts_sum4(s.gates, parts, s.prow, 4 * kH, b, q * kH + 4 * j4);
}

// LSTM cell from summed gates (+ E0[tok] for layer 0) and the old cell state.
__device__ __forceinline__ void p_cell_apply(const DecState& s, int layer, int b, int j4, float4 (&g)[4],
                                             const float4* e0, float4 c4) {
    const int j = 4 * j4;
    if (e0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            g[q].x += e0[q].x;
            g[q].y += e0[q].y;
            g[q].z += e0[q].z;
            g[q].w += e0[q].w;
        }
    }
    const float gi[4] = {g[0].x, g[0].y, g[0].z, g[0].w}, gf[4] = {g[1].x, g[1].y, g[1].z, g[1].w};
    const float gg[4] = {g[2].x, g[2].y, g[2].z, g[2].w}, go[4] = {g[3].x, g[3].y, g[3].z, g[3].w};
    const float cold[4] = {c4.x, c4.y, c4.z, c4.w};
    float cn[4], h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float in = sigm(gi[e]);
        const float fg = sigm(gf[e]);
        const float cand = tanhf(gg[e]);
        cn[e] = fg * cold[e] + in * cand;
        h[e] = sigm(go[e]) * tanhf(cn[e]);
    }
    float* cp = s.c + (static_cast<size_t>(b) * 2 + layer) * kH + j;
    *reinterpret_cast<float4*>(cp) = make_float4(cn[0], cn[1], cn[2], cn[3]);
    __half* self = layer == 0 ? s.a0 + static_cast<size_t>(b) * 2 * kH : s.a1 + static_cast<size_t>(b) * 4 * kH + 2 * kH;
    __half* next = layer == 0 ? s.a1 + static_cast<size_t>(b) * 4 * kH : s.ap + static_cast<size_t>(b) * 2 * kH;
    const float4 h4 = make_float4(h[0], h[1], h[2], h[3]);
    split_store4(self + j, self + kH + j, h4);
    split_store4(next + j, next + kH + j, h4);
}

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Row b's phase B on the 128 threads of half h: argmax (first max over the
// vocabulary and over the 5 durations, blank moves >= 1 frame; the rule of
// k_dec_argmax), state update, then the layer-0 cell if the row emitted.  The
// scores, this thread's gates and the row's state are loaded together.
__device__ __forceinline__ void p_row_b(const DecPersist& p, int b, int h, int t, bool first, float* wv, int* wi,
                                        int* wdur, int* sx, unsigned int* act_cnt) {
    const DecState& s = p.s;
    const int warp = t >> 5, lane = t & 31;
    const int ld = s.ld_scores;
    // gates of column groups j4 = t and (t < 32) t + 128
    float4 g1[4], g2[4];
    p_gates(s, s.ks_g0, b, t, g1);
    const bool two = t < kH / 4 - 128;
    if (two) p_gates(s, s.ks_g0, b, t + 128, g2);
    const float4 c1 = ldcg4(s.c + static_cast<size_t>(b) * 2 * kH + 4 * t);
    float4 c2 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (two) c2 = ldcg4(s.c + static_cast<size_t>(b) * 2 * kH + 4 * (t + 128));
    int tok = s.blank, emit = 1;
    if (!first) {
        int st_act = 0, st_frame = 0, st_count = 0, st_guard = 0, st_len = 0;
        if (t == 0) {
            st_len = s.len[b];
            st_act = ldcg_i(s.active + b);
            st_frame = ldcg_i(s.frame + b);
            st_count = ldcg_i(s.count + b);
            st_guard = ldcg_i(s.guard + b);
        }
        float best = -INFINITY;
        int bidx = 0x7fffffff;
        float dv = -INFINITY;
        int di = 0x7fffffff;
        if (warp == 0 && lane < 5) {
            dv = parts_sum1(s.scores, s.ks_h, s.prow, ld, b, s.vocab + lane);
            di = lane;
        }
        // the row in chunks of 1536 columns, three 4-column loads per thread
        // in flight (one chunk covers a 1025-entry vocabulary)
        for (int base0 = 0; base0 < s.vocab; base0 += 1536) {
            float4 sc[3];
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                const int base = base0 + 4 * t + 512 * i;
                sc[i] = base < s.vocab ? parts_sum4(s.scores, s.ks_h, s.prow, ld, b, base)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                const int base = base0 + 4 * t + 512 * i;
                const float e[4] = {sc[i].x, sc[i].y, sc[i].z, sc[i].w};
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (base + q < s.vocab && e[q] > best) {   // increasing index: strict > keeps the first max
                        best = e[q];
                        bidx = base + q;
                    }
            }
        }
        warp_argmax(best, bidx);
        if (lane == 0) {
            wv[h * 4 + warp] = best;
            wi[h * 4 + warp] = bidx;
        }
        if (warp == 0) {
            warp_argmax(dv, di);
            if (lane == 0) wdur[h] = di;
        }
        half_sync(h);
        if (t == 0) {
            int e = 0, tk = 0;
            if (st_act) {
                float tv = wv[h * 4];
                tk = wi[h * 4];
                for (int w = 1; w < 4; ++w)
                    if (wins(wv[h * 4 + w], wi[h * 4 + w], tv, tk)) {
                        tv = wv[h * 4 + w];
                        tk = wi[h * 4 + w];
                    }
                int dur = wdur[h];
                if (tk == 0x7fffffff) tk = 0;
                if (dur == 0x7fffffff) dur = 0;
                const int T = st_len;
                e = tk != s.blank;
                int nf;
                if (e) {
                    if (st_count < s.max_tokens) {
                        uint32_t* tw = s.tokens + (static_cast<size_t>(b) * s.max_tokens + st_count) * 3;
                        tw[0] = static_cast<uint32_t>(tk);
                        tw[1] = static_cast<uint32_t>(st_frame);
                        tw[2] = static_cast<uint32_t>(dur);
                    }
                    s.count[b] = st_count + 1;
                    nf = st_frame + dur;
                    s.tok[b] = tk;
                } else {
                    nf = st_frame + (dur > 0 ? dur : 1);
                }
                s.frame[b] = nf;
                s.guard[b] = st_guard + 1;
                const long max_steps = static_cast<long>(T) * (10 + 4) + 64;
                const bool act = nf < T && st_guard + 1 < max_steps;
                s.active[b] = act ? 1 : 0;
                if (act) atomicAdd(act_cnt, 1u);
            }
            s.emit[b] = e;
            sx[2 * h] = e;
            sx[2 * h + 1] = tk;
        }
        half_sync(h);
        emit = sx[2 * h];
        tok = sx[2 * h + 1];
    }
    if (!emit) return;
    const float* e0 = s.e0 + static_cast<size_t>(tok) * 4 * kH;
    float4 e1[4], e2[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) e1[q] = __ldg(reinterpret_cast<const float4*>(e0 + q * kH + 4 * t));
    if (two) {
#pragma unroll
        for (int q = 0; q < 4; ++q) e2[q] = __ldg(reinterpret_cast<const float4*>(e0 + q * kH + 4 * (t + 128)));
    }
    p_cell_apply(s, 0, b, t, g1, e1, c1);
    if (two) p_cell_apply(s, 0, b, t + 128, g2, e2, c2);
}

// Phase D for row b: the layer-1 cell if the row emitted.
__device__ __forceinline__ void p_row_d(const DecState& s, int b, int t) {
    const int emit = ldcg_i(s.emit + b);
    float4 g1[4], g2[4];
    p_gates(s, s.ks_g1, b, t, g1);
    const bool two = t < kH / 4 - 128;
    if (two) p_gates(s, s.ks_g1, b, t + 128, g2);
    const float* cb = s.c + (static_cast<size_t>(b) * 2 + 1) * kH;
    const float4 c1 = ldcg4(cb + 4 * t);
    float4 c2 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (two) c2 = ldcg4(cb + 4 * (t + 128));
    if (!emit) return;
    p_cell_apply(s, 1, b, t, g1, nullptr, c1);
    if (two) p_cell_apply(s, 1, b, t + 128, g2, nullptr, c2);
}

// Phase F for row b: joint input x = ReLU(enc[frame] + dec) as hi | lo
// (zeros for finished rows).
__device__ __forceinline__ void p_row_f(const DecState& s, int b, int t) {
    const int act = ldcg_i(s.active + b);
    const int fr = ldcg_i(s.frame + b);
    const int r0 = s.row0[b];
    float4 d1 = parts_sum4(s.dec, s.ks_p, s.prow, kH, b, 4 * t), d2 = make_float4(0.f, 0.f, 0.f, 0.f);
    const bool two = t < kH / 4 - 128;
    if (two) d2 = parts_sum4(s.dec, s.ks_p, s.prow, kH, b, 4 * (t + 128));
    __half* aj = s.aj + static_cast<size_t>(b) * 2 * kH;
    for (int u = 0; u < (two ? 2 : 1); ++u) {
        const int j = 4 * (t + 128 * u);
        const float4 d = u ? d2 : d1;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (act) {
            const float4 e = __ldg(reinterpret_cast<const float4*>(s.pooler + static_cast<size_t>(r0 + fr) * kH + j));
            v = make_float4(fmaxf(e.x + d.x, 0.f), fmaxf(e.y + d.y, 0.f), fmaxf(e.z + d.z, 0.f), fmaxf(e.w + d.w, 0.f));
        }
        split_store4(aj + j, aj + kH + j, v);
    }
}

__global__ void __launch_bounds__(kPThreads, 1)
    k_dec_persist(const __grid_constant__ DecMaps maps, const DecPersist p) {
    extern __shared__ __align__(1024) uint8_t p_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p_smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPBarOff);
    PRing r;
    r.ring = smem;
    r.slabs = smem + kPSlabOff;
    r.bias = reinterpret_cast<float*>(smem + kPBiasOff);
    r.full = bars;
    r.empty = bars + kPStages;
    r.tfull = bars + 2 * kPStages;
    r.tempty = bars + 2 * kPStages + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kPStages + 4);
    int* ok_smem = reinterpret_cast<int*>(tmem_slot + 1);
    float* wv = reinterpret_cast<float*>(tmem_slot + 2);   // [2][4]
    int* wi = reinterpret_cast<int*>(wv + 8);              // [2][4]
    int* wdur = wi + 8;                                    // [2]
    int* sx = wdur + 2;                                    // [2][emit, token]
    int* sdone = sx + 4;

    const int warp = threadIdx.x >> 5;
    const int t = threadIdx.x & 127, h = threadIdx.x >> 7;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 4; ++i) {
            tma_prefetch_desc(&maps.a[i]);
            tma_prefetch_desc(&maps.b[i]);
        }
        for (int i = 0; i < kPStages; ++i) {
            mbar_init(smem_u32(&r.full[i]), 1);
            mbar_init(smem_u32(&r.empty[i]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&r.tfull[i]), 1);
            mbar_init(smem_u32(&r.tempty[i]), 128);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc<kPTmemCols>(smem_u32(tmem_slot));
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    r.tmem = *tmem_slot;

    const DecState& s = p.s;
    unsigned int* sync = p.sync;
    const unsigned int nb = gridDim.x;
    unsigned int target = 0;
    int pit = 0, mit = 0, acc = 0;
    const int row_stride = 2 * gridDim.x;
    for (int step = -1; step < p.max_steps; ++step) {
        const bool first = step < 0;
        // A: joint head (not on the first pass) + layer-0 recurrent GEMM
        bool fail = __syncthreads_or(!p_gemm_phase(maps, p, r, first ? -1 : kDecHead, kDecLstm0, pit, mit, acc));
        if (!grid_barrier(sync, nb, target, fail, ok_smem, 0x65, p.grid_wait_ns)) break;
        // B: argmax + update, layer-0 cell
        if (threadIdx.x == 0 && blockIdx.x == 0 && !first) sync[4 + ((step + 1) & 1)] = 0;
        for (int b = blockIdx.x * 2 + h; b < s.B; b += row_stride) {
            p_row_b(p, b, h, t, first, wv, wi, wdur, sx, sync + 4 + (step & 1));
            half_sync(h);
        }
        fence_async_global();
        if (!grid_barrier(sync, nb, target, false, ok_smem, 0x66, p.grid_wait_ns)) break;
        // C: layer-1 GEMM
        fail = __syncthreads_or(!p_gemm_phase(maps, p, r, kDecLstm1, -1, pit, mit, acc));
        if (!grid_barrier(sync, nb, target, fail, ok_smem, 0x67, p.grid_wait_ns)) break;
        // every row finished at this step's argmax (the count is final since
        // the barrier after B; read here so that phase C starts at once)
        if (!first) {
            if (threadIdx.x == 0) *sdone = ld_acquire_gpu(sync + 4 + (step & 1)) == 0;
            __syncthreads();
            if (*reinterpret_cast<volatile int*>(sdone)) break;
        }
        // D: layer-1 cell
        for (int b = blockIdx.x * 2 + h; b < s.B; b += row_stride) p_row_d(s, b, t);
        fence_async_global();
        if (!grid_barrier(sync, nb, target, false, ok_smem, 0x68, p.grid_wait_ns)) break;
        // E: projector GEMM
        fail = __syncthreads_or(!p_gemm_phase(maps, p, r, kDecProj, -1, pit, mit, acc));
        if (!grid_barrier(sync, nb, target, fail, ok_smem, 0x69, p.grid_wait_ns)) break;
        // F: joint input
        for (int b = blockIdx.x * 2 + h; b < s.B; b += row_stride) p_row_f(s, b, t);
        fence_async_global();
        if (!grid_barrier(sync, nb, target, false, ok_smem, 0x6A, p.grid_wait_ns)) break;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<kPTmemCols>(r.tmem);
    }
}

// ───────────────── weight-stationary decoder (batches up to 2 x 128 rows) ─────────────────
//
// The same lock step as k_dec_persist with the weights held still: every CTA
// owns one 128-row weight tile (DecWs) for the whole decode and keeps it in
// shared memory (160 KB: 10 k-blocks of 128 rows x 64 f16, 128-byte swizzle),
// so a step streams only activations.  The GEMMs are transposed, D = W . A^T:
// the tile's 128 weight rows are the MMA's M, the batch rows (the CTA's half)
// its N, and the f16 hi and lo halves of the activation rows are stacked as
// 2 x ntile B rows of one MMA (N = 2 ntile), the epilogue adding the two
// column halves.  An LSTM tile covers whole channels (its four gate rows), so
// its owner applies the cell in its own epilogue and no split-K parts exist.
// A step is four phases behind grid barriers (one fewer per step than the
// split-K kernel's six, and a quarter of the CTAs at up to 128 rows):
//   1  head GEMM -> per-row argmax as 64-bit atomicMax keys (first maximum
//      wins: the low word is ~index); layer-0 recurrent GEMM (kept in TMEM);
//      layer-1 recurrent GEMM -> g1p
//   2  row state update (head tile 0 of each half); layer-0 cell with E0[token]
//   3  layer-1 input GEMM + g1p + bias -> layer-1 cell
//   4  projector GEMM -> joint input ReLU(enc[frame] + dec) as hi | lo
// Rows that do not emit keep their state; finished rows keep being computed
// (their results are never read), the loop ends when no row is alive.  The
// first pass (step -1) is phases 1-4 without the head, on the blank token, as
// the reference starts (src/tdt.rs:424-428).
constexpr int kWsThreads = 256;                 // warp 0 TMA, warp 1 MMA, warps 4..7 epilogue
constexpr int kWsKB = 10;                       // 640 / 64 k-blocks
constexpr uint32_t kWsWBytes = 128u * 640 * 2;  // one weight tile
constexpr uint32_t kWsRingOff = kWsWBytes;
constexpr uint32_t kWsRingBytes = 65536;        // activation ring, reused as the epilogue's exchange area
constexpr uint32_t kWsMetaOff = kWsRingOff + kWsRingBytes;
constexpr uint32_t kWsMetaBytes = 1536;
constexpr uint32_t kWsSmem = kWsMetaOff + kWsMetaBytes + 1024;   // + alignment slack
static_assert(kWsSmem <= 232448, "shared memory budget");
constexpr int kWsMaxStages = 10;
constexpr uint32_t kWsTmemCols = 256;

enum { kWsHead = 0, kWsL0 = 1, kWsL1hh = 2, kWsL1ih = 3, kWsProj = 4 };

// Gate functions of the weight-stationary kernel's cell.  The cell runs on six
// warps and is bound by the instructions they issue, so the logistic function
// uses the exponential intrinsic and the approximate divide (relative error a
// few ulp for the gate range), and tanh follows from the identity
// tanh(x) = 2 sigma(2x) - 1 (absolute error ~1e-7).  Against the precise
// functions this takes ~0.4-1.0 us off each cell phase.
__device__ __forceinline__ float ws_sigm(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float ws_tanh(float x) { return 2.0f * ws_sigm(2.0f * x) - 1.0f; }

__device__ __forceinline__ unsigned long long ws_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);   // order-preserving map of f32 onto u32
    return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(idx));
}
__device__ __forceinline__ int ws_key_index(unsigned long long k) {
    return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k));
}

// 32 lanes x 32 columns (v[j], ix[j] of column j) -> lane l holds the winner
// of column l over the 32 lanes (31 exchanges; halves of the columns travel
// at each step).
__device__ __forceinline__ void ws_transpose_argmax(float (&v)[32], int (&ix)[32], int lane) {
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        const bool up = (lane & s) != 0;
#pragma unroll
        for (int k = 0; k < s; ++k) {
            const float sv = up ? v[k] : v[k + s];
            const int si = up ? ix[k] : ix[k + s];
            float kv = up ? v[k + s] : v[k];
            int ki = up ? ix[k + s] : ix[k];
            const float rv = __shfl_xor_sync(0xffffffffu, sv, s);
            const int ri = __shfl_xor_sync(0xffffffffu, si, s);
            if (wins(rv, ri, kv, ki)) {
                kv = rv;
                ki = ri;
            }
            v[k] = kv;
            ix[k] = ki;
        }
    }
}

// Activation layout of the weight-stationary kernel: 20 panels [k-block][hi, lo]
// of [bpad rows][64 f16], so one 3D TMA box (64 x rows x 2 kc panels) brings kc
// k-blocks with each k-block's hi rows and lo rows stacked as the MMA's B.
__device__ __forceinline__ __half* ws_panel(__half* base, int bpad, int col, int n, int h) {
    return base + (static_cast<size_t>(2 * (col >> 6) + h) * bpad + n) * 64 + (col & 63);
}

// Named barriers that leave out warps 0 and 1 (the TMA and MMA issuers,
// which return from a GEMM only once its last stage has landed): the four
// epilogue warps (id 5), and warps 2..7, which share the LSTM cell math (id 6).
__device__ __forceinline__ void ws_sync_epi() { asm volatile("bar.sync 5, 128;" ::: "memory"); }
__device__ __forceinline__ bool ws_sync_math_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 6, 192, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v))
        : "memory");
    return r != 0;
}

// Named barrier of the four epilogue warps that also ANDs a predicate over them.
__device__ __forceinline__ bool __syncthreads_and_epi(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 5, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v))
        : "memory");
    return r != 0;
}

__global__ void __launch_bounds__(kWsThreads, 1)
    k_dec_ws(const __grid_constant__ DecWsMaps maps, const DecWs p) {
    extern __shared__ __align__(1024) uint8_t ws_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sW = smem;
    uint8_t* ring = smem + kWsRingOff;
    float* xc = reinterpret_cast<float*>(ring);               // epilogue exchange (ring idle then)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWsMetaOff);
    uint64_t* empty = full + kWsMaxStages;
    uint64_t* wfull = full + 2 * kWsMaxStages;
    uint64_t* tfull = wfull + 1;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tfull + 1);
    int* ok_smem = reinterpret_cast<int*>(tslot + 1);
    int* sdone = ok_smem + 1;
    int* em = reinterpret_cast<int*>(smem + kWsMetaOff + 512);   // [128] per-column flag
    int* tk = em + 128;                                          // [128] per-column token / pooler row

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x % p.n_roles, half = blockIdx.x / p.n_roles;
    const int n0 = half * p.ntile;
    const int ht = p.head_tiles;
    int role, t;
    if (tile < ht) {
        role = kWsHead, t = tile;
    } else if (tile < ht + kWsLstmTiles) {
        role = kWsL0, t = tile - ht;
    } else if (tile < ht + 2 * kWsLstmTiles) {
        role = kWsL1hh, t = tile - ht - kWsLstmTiles;
    } else if (tile < ht + 3 * kWsLstmTiles) {
        role = kWsL1ih, t = tile - ht - 2 * kWsLstmTiles;
    } else {
        role = kWsProj, t = tile - ht - 3 * kWsLstmTiles;
    }
    const CUtensorMap* amap = role == kWsHead ? &maps.aj : (role == kWsL0 || role == kWsL1ih) ? &maps.act0 : &maps.act1;
    const int nt = p.ntile;
    const int kc = p.kc;                                   // k-blocks per TMA box / ring stage
    const int nloads = (kWsKB + kc - 1) / kc;
    const uint32_t kb_bytes = 2u * nt * 128u;              // one k-block: hi rows then lo rows
    const uint32_t stage_bytes = kc * kb_bytes;
    const int stages = min(kWsMaxStages, static_cast<int>(kWsRingBytes / stage_bytes));
    const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>((2 * nt) >> 3) << 17) | ((128u >> 4) << 24);

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&maps.w);
        tma_prefetch_desc(amap);
        for (int i = 0; i < stages; ++i) {
            mbar_init(smem_u32(&full[i]), 1);
            mbar_init(smem_u32(&empty[i]), 1);
        }
        mbar_init(smem_u32(wfull), 1);
        mbar_init(smem_u32(tfull), 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc<kWsTmemCols>(smem_u32(tslot));
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (threadIdx.x == 0) {   // the tile's weights, once
        mbar_arrive_expect_tx(smem_u32(wfull), kWsWBytes);
        for (int kb = 0; kb < kWsKB; ++kb)
            tma_load_2d(smem_u32(sW + kb * 16384), &maps.w, smem_u32(wfull), 64 * kb, 128 * tile);
    }

    int pit = 0, mit = 0, ng_mma = 0, ng_epi = 0;
    bool wready = false;
    // One GEMM of this CTA: D[128][2 nt] = W . [hi rows | lo rows]^T.  The
    // producer and the MMA issuer return after issuing; the epilogue waits
    // for the accumulator (ws_acc).
    auto gemm = [&]() -> bool {
        bool ok = true;
        if (warp == 0 && lane == 0) {
            fence_async_global();   // activations other CTAs wrote before the barrier
            // one TMA instruction per kc k-blocks (kc divides the 10): issuing
            // TMA instructions, not their bytes, is what a phase waits for at
            // small batches
            for (int i = 0; i < nloads; ++i, ++pit) {
                const int st = pit % stages;
                if (pit >= stages && !(ok = mbar_wait(smem_u32(&empty[st]), ((pit / stages) - 1) & 1, 0x70))) break;
                const uint32_t fb = smem_u32(&full[st]);
                mbar_arrive_expect_tx(fb, stage_bytes);
                tma_load_3d(smem_u32(ring + st * stage_bytes), amap, fb, 0, n0, 2 * kc * i);
            }
        } else if (warp == 1 && lane == 0) {
            if (!wready) {
                if (!(ok = mbar_wait(smem_u32(wfull), 0, 0x71))) return ok;
                wready = true;
            }
            tc_fence_after();
            for (int i = 0; i < nloads; ++i, ++mit) {
                const int st = mit % stages;
                if (!(ok = mbar_wait(smem_u32(&full[st]), (mit / stages) & 1, 0x72))) break;
                tc_fence_after();
                for (int j = 0; j < kc && i * kc + j < kWsKB; ++j) {
                    const int kb = i * kc + j;
                    const uint64_t a = smem_desc_sw128(smem_u32(sW + kb * 16384));
                    const uint64_t b = smem_desc_sw128(smem_u32(ring + st * stage_bytes + j * kb_bytes));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) mma_f16_ss(tmem, a + 2 * kk, b + 2 * kk, idesc, (kb | kk) != 0);
                }
                mma_commit(smem_u32(&empty[st]));
            }
            if (ok) {
                mma_commit(smem_u32(tfull));
                ++ng_mma;
            }
        }
        return ok;
    };
    // Epilogue warps: wait for this CTA's latest accumulator.
    auto ws_acc = [&]() -> bool {
        bool got = mbar_wait(smem_u32(tfull), ng_epi & 1, 0x73);
        ++ng_epi;
        got = __all_sync(0xffffffffu, got);
        tc_fence_after();
        return got;
    };
    // Columns [c0, c0 + 32) of the accumulator as hi + lo (lane = weight row).
    auto acc32 = [&](int q, int c0, float (&v)[32]) {
        uint32_t h[32], l[32];
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        tmem_ld_32x32b_x32(base + c0, h);
        tmem_ld_32x32b_x32(base + nt + c0, l);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(h[j]) + __uint_as_float(l[j]);
    };
    // Per column of this half: emit flag and token of step `par` (epilogue threads).
    auto load_emit = [&](int par, bool first) {
        const int u = threadIdx.x - 128;
        if (u < nt) {
            const int n = n0 + u;
            int e = 0, tkn = p.blank;
            if (n < p.B) {   // both loads issued together
                const int a = __ldcg(p.alive + par * p.B + n);
                const unsigned long long key = __ldcg(p.keys + static_cast<size_t>(par * 2) * p.B + n);
                if (first) {
                    e = a;
                } else {
                    tkn = ws_key_index(key);
                    e = a && tkn != p.blank;
                }
            }
            em[u] = e;
            tk[u] = tkn;
        }
    };
    // LSTM cell of layer `layer` for this tile's 32 channels x this half's
    // rows (ntile <= 64), run by warps 2..7 after load_emit and their named
    // barrier.  Every global load (cell states, E0 row slices, the recurrent
    // half of the layer-1 gates) is issued before the accumulator wait, so it
    // overlaps this phase's GEMM; thread (channel ch, column group cg) of the
    // six warps takes columns cg + 6 i.
    auto cell = [&](int layer) -> bool {
        const int mt = threadIdx.x - 64, ch = mt & 31, cg = mt >> 5;
        constexpr int kCols = 11;   // ceil(64 / 6)
        bool act[kCols];
        float cold[kCols], e[kCols][4];
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
            const int col = cg + 6 * i;
            act[i] = col < nt && n0 + col < p.B && em[col];
            const int n = n0 + (act[i] ? col : 0);
            cold[i] = act[i] ? __ldcg(p.c + (static_cast<size_t>(n) * 2 + layer) * 640 + 32 * t + ch) : 0.f;
#pragma unroll
            for (int g = 0; g < 4; ++g)
                e[i][g] = (layer == 0 && act[i])
                              ? __ldg(p.e0 + static_cast<size_t>(tk[col]) * 2560 + g * 640 + 32 * t + ch)
                              : 0.f;
        }
        bool got = true;
        if (warp >= 4) {
            const int q = warp & 3;
            const int gi = q * 640 + 32 * t + lane;   // gate row in the original i | f | g | o order
            float r[64];
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const int n = n0 + j;
                r[j] = (layer == 1 && j < nt && n < p.B) ? __ldcg(p.g1p + static_cast<size_t>(n) * 2560 + gi) : 0.f;
            }
            const float b1 = layer == 1 ? __ldg(p.bias + ht * 128 + gi) : 0.f;
            got = ws_acc();
            if (got) {
#pragma unroll
                for (int c0 = 0; c0 < 64; c0 += 32) {
                    if (c0 >= nt) break;
                    float v[32];
                    acc32(q, c0, v);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        xc[(q * nt + c0 + j) * 32 + lane] = layer == 1 ? (b1 + v[j]) + r[c0 + j] : v[j];
                }
            }
            tc_fence_before();
        }
        const bool all_got = ws_sync_math_and(got);
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
            if (!all_got || !act[i]) continue;
            const int col = cg + 6 * i, n = n0 + col;
            float gate[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) gate[g] = xc[(g * nt + col) * 32 + ch] + e[i][g];
            const float in = ws_sigm(gate[0]);
            const float fg = ws_sigm(gate[1]);
            const float cand = ws_tanh(gate[2]);
            const float cn = fg * cold[i] + in * cand;
            const float h = ws_sigm(gate[3]) * ws_tanh(cn);
            p.c[(static_cast<size_t>(n) * 2 + layer) * 640 + 32 * t + ch] = cn;
            __half* a = layer == 0 ? p.act0 : p.act1;
            split_store(ws_panel(a, p.bpad, 32 * t + ch, n, 0), ws_panel(a, p.bpad, 32 * t + ch, n, 1), h);
        }
        fence_async_shared();
        return all_got;
    };

    const int epi = warp >= 4;
    unsigned int* sync = p.sync;
    const unsigned int nb = gridDim.x;
    unsigned int target = 0;
    for (int s = -1; s < p.max_steps; ++s) {
        const int par = s & 1;
        const bool first = s < 0;
        bool ok = true;
        // ── phase 1: head (argmax keys), layer-0 recurrent, layer-1 recurrent ──
        if (role == kWsL0 || role == kWsL1hh || (role == kWsHead && !first)) ok = gemm();
        if (ok && epi && role == kWsHead && !first) {
            const int q = warp & 3;
            const int wr = 128 * t + 32 * q + lane;   // head row: token < vocab <= duration < vocab + 5
            const bool is_tok = wr < p.vocab, is_dur = wr >= p.vocab && wr < p.vocab + 5;
            const bool has_dur = 128 * t < p.vocab + 5 && 128 * t + 127 >= p.vocab;
            const float br = __ldg(p.bias + wr);
            float* hx = xc;                                   // [2][4][128] (value, index) per warp
            int* hi_ = reinterpret_cast<int*>(xc + 1024);
            const bool got = ws_acc();
            {
                for (int c0 = 0; got && c0 < nt; c0 += 32) {
                    float v[32], d[32];
                    int ix[32], dx[32];
                    acc32(q, c0, v);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float sc = v[j] + br;
                        v[j] = is_tok ? sc : -INFINITY;
                        ix[j] = wr;
                        d[j] = is_dur ? sc : -INFINITY;
                        dx[j] = wr - p.vocab;
                    }
                    ws_transpose_argmax(v, ix, lane);
                    hx[q * 128 + c0 + lane] = v[0];
                    hi_[q * 128 + c0 + lane] = ix[0];
                    if (has_dur) {
                        ws_transpose_argmax(d, dx, lane);
                        hx[512 + q * 128 + c0 + lane] = d[0];
                        hi_[512 + q * 128 + c0 + lane] = dx[0];
                    }
                }
                tc_fence_before();
                ok = __syncthreads_and_epi(got);   // every epilogue warp meets here
                const int col = threadIdx.x - 128;
                const int n = n0 + col;
                if (ok && col < nt && n < p.B) {
                    for (int kind = 0; kind < (has_dur ? 2 : 1); ++kind) {
                        float bv = hx[kind * 512 + col];
                        int bi = hi_[kind * 512 + col];
                        for (int w = 1; w < 4; ++w) {
                            const float wv = hx[kind * 512 + w * 128 + col];
                            const int wi = hi_[kind * 512 + w * 128 + col];
                            if (wins(wv, wi, bv, bi)) {
                                bv = wv;
                                bi = wi;
                            }
                        }
                        if (bv > -INFINITY)
                            atomicMax(p.keys + static_cast<size_t>(par * 2 + kind) * p.B + n, ws_key(bv, bi));
                    }
                }
                fence_async_shared();
            }
        }
        if (ok && epi && role == kWsL1hh) {
            const int q = warp & 3;
            const int gi = q * 640 + 32 * t + lane;
            if ((ok = ws_acc())) {
                for (int c0 = 0; c0 < nt; c0 += 32) {
                    float v[32];
                    acc32(q, c0, v);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int n = n0 + c0 + j;
                        if (n < p.B) p.g1p[static_cast<size_t>(n) * 2560 + gi] = v[j];
                    }
                }
                tc_fence_before();
            }
        }
        bool fail = __syncthreads_or(!ok);
        if (!grid_barrier(sync, nb, target, fail, ok_smem, 0x74, p.grid_wait_ns)) break;

        // ── phase 2: row state (head tile 0 of each half), layer-0 cell ──
        if (epi && role == kWsHead && t == 0 && !first) {
            const int u = threadIdx.x - 128, n = n0 + u;
            if (u < nt && n < p.B) {
                int act = 0;
                // every load of the row issued together
                const int alive = __ldcg(p.alive + par * p.B + n);
                const int tkn = ws_key_index(__ldcg(p.keys + static_cast<size_t>(par * 2) * p.B + n));
                const int dur = ws_key_index(__ldcg(p.keys + static_cast<size_t>(par * 2 + 1) * p.B + n));
                const int T = p.len[n], fr = p.frame[n], cnt = p.count[n], gd = p.guard[n];
                if (alive) {
                    int nf;
                    if (tkn != p.blank) {
                        if (cnt < p.max_tokens) {
                            uint32_t* tw = p.tokens + (static_cast<size_t>(n) * p.max_tokens + cnt) * 3;
                            tw[0] = static_cast<uint32_t>(tkn);
                            tw[1] = static_cast<uint32_t>(fr);
                            tw[2] = static_cast<uint32_t>(dur);
                        }
                        p.count[n] = cnt + 1;
                        nf = fr + dur;
                    } else {
                        nf = fr + (dur > 0 ? dur : 1);
                    }
                    p.frame[n] = nf;
                    p.guard[n] = gd + 1;
                    const long max_steps = static_cast<long>(T) * (10 + 4) + 64;
                    act = nf < T && gd + 1 < max_steps;
                    if (act) atomicAdd(sync + 4 + par, 1u);
                }
                p.alive[(par ^ 1) * p.B + n] = act;
            }
        }
        if (role == kWsL0 && warp >= 2) {
            if (epi) load_emit(par, first);
            ws_sync_math_and(true);
            ok = cell(0);
        }
        fence_async_global();
        fail = __syncthreads_or(!ok);
        if (!grid_barrier(sync, nb, target, fail, ok_smem, 0x75, p.grid_wait_ns)) break;
        if (!first) {   // every row finished at this step's argmax
            if (threadIdx.x == 0) *sdone = ld_acquire_gpu(sync + 4 + par) == 0;
            __syncthreads();
            if (*reinterpret_cast<volatile int*>(sdone)) break;
        }

        // ── phase 3: layer-1 input GEMM + cell; the next step's keys and count cleared ──
        if (blockIdx.x == 0) {
            for (int i = threadIdx.x; i < 2 * p.B; i += blockDim.x)
                p.keys[static_cast<size_t>((par ^ 1) * 2) * p.B + i] = 0ull;
            if (threadIdx.x == 0) sync[4 + (par ^ 1)] = 0u;
        }
        if (role == kWsL1ih) {
            ok = gemm();
            if (warp >= 2) {
                if (epi) load_emit(par, first);
                ws_sync_math_and(true);
                ok = cell(1);
            }
        }
        fence_async_global();
        fail = __syncthreads_or(!ok);
        if (!grid_barrier(sync, nb, target, fail, ok_smem, 0x76, p.grid_wait_ns)) break;

        // ── phase 4: projector GEMM -> joint input ──
        if (role == kWsProj) {
            ok = gemm();
            if (epi) {
                const int u = threadIdx.x - 128;
                if (u < nt) {   // pooler row of each alive column of the next step
                    const int n = n0 + u;
                    int pr = -1;
                    if (n < p.B) {
                        const int a = __ldcg(p.alive + (par ^ 1) * p.B + n), fr = __ldcg(p.frame + n), r0 = p.row0[n];
                        if (a) pr = r0 + fr;
                    }
                    tk[u] = pr;
                }
                ws_sync_epi();
            }
            if (ok && epi) {
                const int q = warp & 3;
                const int j = 128 * t + 32 * q + lane;   // joint-input column
                const float bj = __ldg(p.bias + ht * 128 + 2560 + j);
                // every encoder-frame load before the accumulator wait (they
                // overlap the GEMM) and before any store
                float e[64];
#pragma unroll
                for (int jj = 0; jj < 64; ++jj) {
                    const int pr = jj < nt ? tk[jj] : -1;
                    e[jj] = pr >= 0 ? __ldg(p.pooler + static_cast<size_t>(pr) * 640 + j) : 0.f;
                }
                if ((ok = ws_acc())) {
#pragma unroll
                    for (int c0 = 0; c0 < 64; c0 += 32) {
                        if (c0 >= nt) break;
                        float v[32];
                        acc32(q, c0, v);
#pragma unroll
                        for (int jj = 0; jj < 32; ++jj) {
                            const int n = n0 + c0 + jj;
                            if (n >= p.B) continue;
                            const float x = tk[c0 + jj] >= 0 ? fmaxf(e[c0 + jj] + (bj + v[jj]), 0.f) : 0.f;
                            split_store(ws_panel(p.aj, p.bpad, j, n, 0), ws_panel(p.aj, p.bpad, j, n, 1), x);
                        }
                    }
                    tc_fence_before();
                }
            }
        }
        fence_async_global();
        fail = __syncthreads_or(!ok);
        if (!grid_barrier(sync, nb, target, fail, ok_smem, 0x77, p.grid_wait_ns)) break;
    }
    // Leaving (normally or on an abort between phases): the weight load and
    // the last accumulator this CTA issued (a layer-0 tile's MMAs may still
    // run when a barrier after phase 1 gave up) are waited for, bounded,
    // before TMEM is freed.
    if (warp == 1 && lane == 0) {
        if (!wready) mbar_wait(smem_u32(wfull), 0, 0x78);
        if (ng_mma > 0) mbar_wait(smem_u32(tfull), (ng_mma - 1) & 1, 0x79);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<kWsTmemCols>(tmem);
    }
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error(what, e);
}

}  // namespace

// The init kernel is launched with programmatic stream serialization: its CTAs
// are scheduled while the producer of the pooler drains and wait in pdl_wait()
// for its results.
template <typename... Args>
int launch_pdl(void (*kern)(Args...), dim3 grid, dim3 block, cudaStream_t st, const char* what, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    return e == cudaSuccess ? 0 : set_cuda_error(what, e);
}

int dec_launch_init(const DecState& s, cudaStream_t st) {
    return launch_pdl(k_dec_init, dim3(s.B), dim3(128), st, "k_dec_init", s);
}

int dec_persistent_grid(int device) {
    // per device: the shared-memory attribute and the occupancy check
    static std::atomic<int> cached[64];
    static PerDeviceOnce attr;
    if (device < 0 || device >= 64) return 0;
    const int known = cached[device].load(std::memory_order_acquire);
    if (known > 0) return known;
    if (set_smem_limit_once(attr, k_dec_persist, kPSmem, "cudaFuncSetAttribute(k_dec_persist)")) return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_dec_persist, kPThreads, kPSmem) != cudaSuccess) return 0;
    const int grid = per_sm >= 1 ? device_sms() : 0;   // one CTA per SM (TMEM and the ring are sized for it)
    cached[device].store(grid, std::memory_order_release);
    return grid;
}

// Tile widths and split-K parts for the persistent decoder.  The GEMMs are
// bound by the bytes each SM pulls from L2, so the model is bytes: per item,
// its k-blocks (two 16 KB A boxes + a bn x 64 weight tile each) plus its
// partial-output write; items are dealt round-robin, and per GEMM phase the
// plan with the smallest busiest CTA wins (ties keep fewer parts).
void dec_plan_persistent(int B, int npad, int grid, int bn[4], int ks[4]) {
    const int m_tiles = (B + 127) / 128;
    const int n[4] = {npad, 2560, 2560, 640};
    const int nk[4] = {640 / 64, 640 / 64, 1280 / 64, 640 / 64};   // logical k-blocks
    for (int i = 0; i < 4; ++i) bn[i] = n[i] % 256 == 0 ? 256 : 128;
    auto cost = [&](const int* gs, const int* kss, int ng) {
        std::vector<double> load(grid, 0.0);
        long j = 0;
        for (int i = 0; i < ng; ++i) {
            const int g = gs[i];
            const long items = static_cast<long>(m_tiles) * (n[g] / bn[g]) * kss[i];
            const double c = (nk[g] / kss[i]) * (32768.0 + bn[g] * 128.0) + 128.0 * bn[g] * 4.0 + 16384.0;
            for (long u = 0; u < items; ++u, ++j) load[j % grid] += c;
        }
        double mx = 0;
        for (double v : load) mx = v > mx ? v : mx;
        return mx;
    };
    auto ok_ks = [&](int g, int k) { return k >= 1 && k <= kMaxParts && nk[g] % k == 0; };
    double best = -1;
    for (int a = 1; a <= kMaxParts; ++a) {
        if (!ok_ks(kDecHead, a)) continue;
        for (int b = 1; b <= kMaxParts; ++b) {
            if (!ok_ks(kDecLstm0, b)) continue;
            const int gs[2] = {kDecHead, kDecLstm0}, kss[2] = {a, b};
            const double c = cost(gs, kss, 2);
            if (best < 0 || c < best * 0.999) {
                best = c;
                ks[kDecHead] = a;
                ks[kDecLstm0] = b;
            }
        }
    }
    for (int g : {kDecLstm1, kDecProj}) {
        best = -1;
        for (int k = 1; k <= kMaxParts; ++k) {
            if (!ok_ks(g, k)) continue;
            const int gs[1] = {g}, kss[1] = {k};
            const double c = cost(gs, kss, 1);
            if (best < 0 || c < best * 0.999) {
                best = c;
                ks[g] = k;
            }
        }
    }
}

int dec_launch_persistent(const DecMaps& maps, const DecPersist& p, int grid, cudaStream_t st) {
    if (grid <= 0) return set_error(B3_ECUDA, "the persistent decoder does not fit on this device");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = kPSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_dec_persist, maps, p);
    return e == cudaSuccess ? 0 : set_cuda_error("k_dec_persist", e);
}

// Reads and clears this translation unit's device error word (stream-ordered):
// the decoder's bounded waits (grid barriers and its GEMM phases) write it.
int decoder_take_dev_error(cudaStream_t st, unsigned int* out) {
    static const unsigned int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_b3_dev_error, sizeof(unsigned int), 0,
                                              cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbolAsync(g_b3_dev_error, &zero, sizeof(unsigned int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? 0 : set_cuda_error("reading the decoder device error word", e);
}


int dec_ws_grid(int device, int n_roles, int nsplit) {
    static std::atomic<int> fits[64];   // 0 unknown, 1 yes, -1 no
    static PerDeviceOnce attr;
    if (device < 0 || device >= 64 || n_roles <= 0 || nsplit <= 0) return 0;
    int f = fits[device].load(std::memory_order_acquire);
    if (f == 0) {
        int per_sm = 0;
        f = -1;
        if (!set_smem_limit_once(attr, k_dec_ws, static_cast<int>(kWsSmem), "cudaFuncSetAttribute(k_dec_ws)") &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_dec_ws, kWsThreads, kWsSmem) == cudaSuccess &&
            per_sm >= 1)
            f = 1;
        fits[device].store(f, std::memory_order_release);
    }
    const int grid = n_roles * nsplit;
    return f > 0 && grid <= device_sms() ? grid : 0;
}

int dec_ws_launch(const DecWsMaps& maps, const DecWs& p, int grid, cudaStream_t st) {
    if (grid <= 0) return set_error(B3_ECUDA, "the weight-stationary decoder does not fit on this device");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kWsThreads);
    cfg.dynamicSmemBytes = kWsSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_dec_ws, maps, p);
    return e == cudaSuccess ? 0 : set_cuda_error("k_dec_ws", e);
}

int dec_launch_split(const float* src, __half* hi, __half* lo, int64_t n, cudaStream_t st) {
    int blocks = static_cast<int>((n + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    k_split_rows<<<blocks, 256, 0, st>>>(src, hi, lo, n);
    return check_launch("k_split_rows");
}

}  // namespace b3
