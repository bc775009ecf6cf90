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
// Structure (one 128 x BN output tile per CTA, 192 threads):
//   warp 0      TMA producer: A tile (128 x 64 f16, 128-byte swizzle) and the
//               code tile (BN x 32 bytes) or the f16 B tile, into a
//               STAGES-deep ring guarded by mbarriers;
//   warp 1      allocates TMEM, one thread issues tcgen05.mma (M=128, N=BN,
//               K=16, f32 accumulator in TMEM) and commits stages back;
//   warps 2..5  LUT4: expand each code tile through the per-row table, kept
//               in registers as byte planes and indexed with PRMT, into the
//               128-byte-swizzled K-major f16 B tile the MMA reads; then all
//               four run the epilogue: tcgen05.ld -> bias / SiLU / GLU /
//               residual / q-k-v split -> global.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b3_internal.h"
#include "b3_ptx.cuh"

namespace b3 {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;

template <int BN, bool LUT>
struct GemmCfg {
    static constexpr uint32_t kABytes = kBM * kBK * 2;
    static constexpr uint32_t kBBytes = BN * kBK * 2;
    static constexpr uint32_t kCBytes = LUT ? BN * kBK / 2 : 0;
    static constexpr uint32_t kStageBytes = kABytes + kBBytes + kCBytes;
    static constexpr int kStages = (BN == 128) ? (LUT ? 5 : 6) : (LUT ? 3 : 4);
    static constexpr uint32_t kTmemCols = BN;  // power of two >= 32
    static constexpr uint32_t kBarBytes = 256;
    static constexpr uint32_t kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }
__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + __expf(-v)); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Expand 8 codes (one u32: nibble i = column k0+i) through the row's table.
// lo[q] / hi[q] hold the low / high bytes of entries 4q..4q+3.
__device__ __forceinline__ void lut_expand8(uint32_t w, const uint32_t (&lo)[4],
                                            const uint32_t (&hi)[4], uint32_t (&out)[4]) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const uint32_t sel = half ? (w >> 16) : w;  // four 4-bit indices
        const uint32_t s3 = sel & 0x7777u;          // index within 8 entries
        // byte i = 0xFF where index i >= 8 (bit 3 of nibble i, sign-replicated)
        const uint32_t m = prmt(sel, sel << 4, 0x9D8Cu);
        const uint32_t l = bitsel(prmt(lo[0], lo[1], s3), prmt(lo[2], lo[3], s3), m);
        const uint32_t h = bitsel(prmt(hi[0], hi[1], s3), prmt(hi[2], hi[3], s3), m);
        out[2 * half + 0] = prmt(l, h, 0x5140u);  // f16 of columns 0,1 of this half
        out[2 * half + 1] = prmt(l, h, 0x7362u);  // columns 2,3
    }
}

template <int BN, bool LUT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    k1_gemm(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
            const GemmParams p) {
    using Cfg = GemmCfg<BN, LUT>;
    constexpr int S = Cfg::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + S * Cfg::kABytes;
    uint8_t* sC = sB + S * Cfg::kBBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sC + S * Cfg::kCBytes);
    uint64_t* full = bars;
    uint64_t* bready = bars + S;
    uint64_t* empty = bars + 2 * S;
    uint64_t* accf = bars + 3 * S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * kBM;
    const int num_k = p.K / kBK;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&bready[s]), 128);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        mbar_init(smem_u32(accf), 1);
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

    if (warp == 0) {
        if (lane == 0) {
            for (int it = 0; it < num_k; ++it) {
                const int s = it % S;
                const uint32_t ph = (it / S) & 1;
                if (it >= S && !mbar_wait(smem_u32(&empty[s]), ph ^ 1, 0x01)) break;
                const uint32_t fb = smem_u32(&full[s]);
                mbar_arrive_expect_tx(fb, Cfg::kABytes + (LUT ? Cfg::kCBytes : Cfg::kBBytes));
                tma_load_2d(smem_u32(sA + s * Cfg::kABytes), &tm_a, fb, it * kBK, m0);
                if (LUT)
                    tma_load_2d(smem_u32(sC + s * Cfg::kCBytes), &tm_b, fb, it * (kBK / 2), n0);
                else
                    tma_load_2d(smem_u32(sB + s * Cfg::kBBytes), &tm_b, fb, it * kBK, n0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32<kBM, BN>();
            bool ok = true;
            for (int it = 0; it < num_k && ok; ++it) {
                const int s = it % S;
                const uint32_t ph = (it / S) & 1;
                ok = mbar_wait(smem_u32(&full[s]), ph, 0x02);
                if (ok && LUT) ok = mbar_wait(smem_u32(&bready[s]), ph, 0x03);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + s * Cfg::kABytes);
                const uint32_t b0 = smem_u32(sB + s * Cfg::kBBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    mma_f16_ss(tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                               idesc, (it | kk) != 0);
                }
                mma_commit(smem_u32(&empty[s]));
            }
            if (ok) mma_commit(smem_u32(accf));
        }
    } else {
        // warps 2..5: 128 threads
        const int e = threadIdx.x - 64;
        bool ok = true;
        if (LUT) {
            constexpr int RPT = BN / 128;  // rows of B per thread
            uint32_t lo[RPT][4], hi[RPT][4];
#pragma unroll
            for (int r = 0; r < RPT; ++r) {
                const int n = n0 + e + 128 * r;
                const uint4* src = reinterpret_cast<const uint4*>(p.lut + static_cast<size_t>(n) * 16);
                const uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
                // entries (2i, 2i+1) in word i; byte planes of 4 entries each
                lo[r][0] = prmt(u0.x, u0.y, 0x6420u);
                hi[r][0] = prmt(u0.x, u0.y, 0x7531u);
                lo[r][1] = prmt(u0.z, u0.w, 0x6420u);
                hi[r][1] = prmt(u0.z, u0.w, 0x7531u);
                lo[r][2] = prmt(u1.x, u1.y, 0x6420u);
                hi[r][2] = prmt(u1.x, u1.y, 0x7531u);
                lo[r][3] = prmt(u1.z, u1.w, 0x6420u);
                hi[r][3] = prmt(u1.z, u1.w, 0x7531u);
            }
            for (int it = 0; it < num_k; ++it) {
                const int s = it % S;
                const uint32_t ph = (it / S) & 1;
                if (!mbar_wait(smem_u32(&full[s]), ph, 0x04)) {
                    ok = false;
                    break;
                }
                const uint8_t* codes = sC + s * Cfg::kCBytes;
                uint8_t* bt = sB + s * Cfg::kBBytes;
#pragma unroll
                for (int r = 0; r < RPT; ++r) {
                    const int n = e + 128 * r;
                    const uint4 c0 = *reinterpret_cast<const uint4*>(codes + n * 32);
                    const uint4 c1 = *reinterpret_cast<const uint4*>(codes + n * 32 + 16);
                    const uint32_t wds[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                    uint8_t* row = bt + (n >> 3) * 1024 + (n & 7) * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        uint32_t o[4];
                        lut_expand8(wds[j], lo[r], hi[r], o);
                        *reinterpret_cast<uint4*>(row + ((j ^ (n & 7)) << 4)) =
                            make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
                fence_async_shared();
                mbar_arrive(smem_u32(&bready[s]));
            }
        }
        // ── epilogue ──
        if (ok) ok = mbar_wait(smem_u32(accf), 0, 0x05);
        if (ok) {
            tc_fence_after();
            const int q = warp & 3;
            const int row = q * 32 + lane;
            const int gm = m0 + row;
            const bool live = gm < p.M;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c * 32, r);
                tmem_wait_ld();
                if (!live) continue;
                const int n = n0 + c * 32;
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                if (EPI == EPI_F32 || EPI == EPI_F16 || EPI == EPI_SILU_F16) {
                    if (p.bias) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] += __ldg(p.bias + n + i);
                    }
                }
                if (EPI == EPI_F32) {
                    float4* dst = reinterpret_cast<float4*>(p.out_f32 + static_cast<size_t>(gm) * p.ldo + n);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                } else if (EPI == EPI_RESID) {
                    float4* dst = reinterpret_cast<float4*>(p.out_f32 + static_cast<size_t>(gm) * p.ldo + n);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        float4 x = dst[i];
                        x.x += p.alpha * v[4 * i];
                        x.y += p.alpha * v[4 * i + 1];
                        x.z += p.alpha * v[4 * i + 2];
                        x.w += p.alpha * v[4 * i + 3];
                        dst[i] = x;
                    }
                } else if (EPI == EPI_F16 || EPI == EPI_SILU_F16) {
                    uint4* dst = reinterpret_cast<uint4*>(p.out_f16 + static_cast<size_t>(gm) * p.ldo + n);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        float t[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            t[j] = (EPI == EPI_SILU_F16) ? silu_f(v[8 * i + j]) : v[8 * i + j];
                        dst[i] = make_uint4(pack_h2(t[0], t[1]), pack_h2(t[2], t[3]),
                                            pack_h2(t[4], t[5]), pack_h2(t[6], t[7]));
                    }
                } else if (EPI == EPI_GLU_F16) {
                    // rows of W interleaved (value, gate) at load: column 2i is
                    // GLU input a_i, column 2i+1 is its gate b_i.
                    float g[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float a = v[2 * i], b = v[2 * i + 1];
                        if (p.bias) {
                            a += __ldg(p.bias + n + 2 * i);
                            b += __ldg(p.bias + n + 2 * i + 1);
                        }
                        g[i] = a * sigmoid_f(b);
                    }
                    uint4* dst = reinterpret_cast<uint4*>(p.out_f16 + static_cast<size_t>(gm) * p.ldo + n / 2);
                    dst[0] = make_uint4(pack_h2(g[0], g[1]), pack_h2(g[2], g[3]), pack_h2(g[4], g[5]),
                                        pack_h2(g[6], g[7]));
                    dst[1] = make_uint4(pack_h2(g[8], g[9]), pack_h2(g[10], g[11]),
                                        pack_h2(g[12], g[13]), pack_h2(g[14], g[15]));
                } else if (EPI == EPI_QKV) {
                    // out row layout [qu | qv | k | v], 1024 f16 each.
                    __half* orow = p.out_f16 + static_cast<size_t>(gm) * p.ldo;
                    if (n < 1024) {
                        uint4* du = reinterpret_cast<uint4*>(orow + n);
                        uint4* dv = reinterpret_cast<uint4*>(orow + 1024 + n);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            float a[8], b[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                a[j] = v[8 * i + j] + __ldg(p.bias_u + n + 8 * i + j);
                                b[j] = v[8 * i + j] + __ldg(p.bias_v + n + 8 * i + j);
                            }
                            du[i] = make_uint4(pack_h2(a[0], a[1]), pack_h2(a[2], a[3]),
                                               pack_h2(a[4], a[5]), pack_h2(a[6], a[7]));
                            dv[i] = make_uint4(pack_h2(b[0], b[1]), pack_h2(b[2], b[3]),
                                               pack_h2(b[4], b[5]), pack_h2(b[6], b[7]));
                        }
                    } else {
                        uint4* dk = reinterpret_cast<uint4*>(orow + n + 1024);
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            dk[i] = make_uint4(pack_h2(v[8 * i], v[8 * i + 1]), pack_h2(v[8 * i + 2], v[8 * i + 3]),
                                               pack_h2(v[8 * i + 4], v[8 * i + 5]),
                                               pack_h2(v[8 * i + 6], v[8 * i + 7]));
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<Cfg::kTmemCols>(tmem);
    }
}

template <int BN, bool LUT, int EPI>
int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t st) {
    using Cfg = GemmCfg<BN, LUT>;
    auto kern = k1_gemm<BN, LUT, EPI>;
    static bool attr_done = false;  // per template instance
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(Cfg::kSmemBytes));
        if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(k1_gemm)", e);
        attr_done = true;
    }
    dim3 grid(p.N / BN, (p.M + kBM - 1) / kBM);
    kern<<<grid, kThreads, Cfg::kSmemBytes, st>>>(ta, tb, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("k1_gemm launch", e);
    return 0;
}

template <int BN, bool LUT>
int launch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
               cudaStream_t st) {
    switch (epi) {
        case EPI_F32: return launch_one<BN, LUT, EPI_F32>(ta, tb, p, st);
        case EPI_RESID: return launch_one<BN, LUT, EPI_RESID>(ta, tb, p, st);
        case EPI_F16: return launch_one<BN, LUT, EPI_F16>(ta, tb, p, st);
        case EPI_SILU_F16: return launch_one<BN, LUT, EPI_SILU_F16>(ta, tb, p, st);
        case EPI_GLU_F16: return launch_one<BN, LUT, EPI_GLU_F16>(ta, tb, p, st);
        case EPI_QKV: return launch_one<BN, LUT, EPI_QKV>(ta, tb, p, st);
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

int gemm_validate(const GemmParams& p, bool lut, int bn) {
    if (p.M <= 0 || p.N <= 0 || p.K <= 0) return set_error(B3_EINVAL, "GEMM sizes must be positive (M=%d N=%d K=%d)", p.M, p.N, p.K);
    if (p.K % kBK) return set_error(B3_EINVAL, "GEMM K=%d must be a multiple of %d", p.K, kBK);
    if (p.N % bn) return set_error(B3_EINVAL, "GEMM N=%d must be a multiple of %d", p.N, bn);
    if (lut && !p.lut) return set_error(B3_EINVAL, "LUT4 GEMM needs a level table");
    return 0;
}

int gemm_launch(const GemmOp& op, cudaStream_t st) {
    const GemmParams& p = op.p;
    const int bn = op.bn;
    int rc = gemm_validate(p, op.lut, bn);
    if (rc) return rc;
    if (op.lut) {
        if (bn == 128) return launch_epi<128, true>(op.epi, op.map_a, op.map_b, p, st);
        if (bn == 256) return launch_epi<256, true>(op.epi, op.map_a, op.map_b, p, st);
    } else {
        if (bn == 128) return launch_epi<128, false>(op.epi, op.map_a, op.map_b, p, st);
        if (bn == 256) return launch_epi<256, false>(op.epi, op.map_a, op.map_b, p, st);
    }
    return set_error(B3_EINVAL, "unsupported GEMM tile N=%d", bn);
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
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}
}  // namespace

int make_map_2d(CUtensorMap* map, const void* base, bool f16, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(B3_ECUDA, "cuTensorMapEncodeTiled is unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15))
        return set_error(B3_EINVAL, "TMA base/stride must be 16-byte aligned");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(B3_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return 0;
}

int gemm_make_a_map(CUtensorMap* map, const __half* a, int M, int K, int lda) {
    return make_map_2d(map, a, true, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
                       static_cast<uint64_t>(lda) * 2, kBK, kBM, true);
}

int gemm_make_b_map(CUtensorMap* map, const void* w, bool lut, int N, int K, int bn) {
    if (lut)
        return make_map_2d(map, w, false, static_cast<uint64_t>(K / 2), static_cast<uint64_t>(N),
                           static_cast<uint64_t>(K / 2), kBK / 2, bn, false);
    return make_map_2d(map, w, true, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                       static_cast<uint64_t>(K) * 2, kBK, bn, true);
}

}  // namespace b3
