// attention.cu — K2: fused relative-position multi-head self-attention.
//
// For one utterance of T frames, head h (dh = 128), query i and key j:
//   s[i, j] = (qu_i . k_j + qv_i . r_(i-j)) / sqrt(128),   p = softmax_j(s),
//   o_i = sum_j p[i, j] v_j
// where qu = q + bias_u, qv = q + bias_v and r_d is the relative-position key
// for offset d = i - j (the reference's rel_shift: BD[q, T-1-q+k], with row
// T-1-j of its position table holding position j; src/cpu/layer.rs:234-294,
// src/cpu/ops.rs:133-189, src/encoder.rs:2161-2412).
//
// Flash-style: one CTA per (utterance, 64-query block, head), key blocks of
// 64, online softmax in f32, no T x T score buffer.  The positional term of a
// 64x64 score tile needs the 127 offsets of its diagonal band: each warp
// multiplies its 16 queries by the 80 band rows it touches (one GEMM), parks
// that 16x80 strip in shared memory and reads it back along the diagonal.
// Q.K^T, Qv.R^T and P.V run on tensor cores (mma.sync m16n8k16, f16 in, f32
// accumulate); Q / K / V / R are f16 (the reference also rounds K, V and R to
// f16, src/cpu/ops.rs:258-259, src/cpu/layer.rs:234-247).
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b3_internal.h"
#include "b3_kernels.h"

namespace b3 {

namespace {

constexpr int kQ = 64;     // queries per CTA
constexpr int kKB = 64;    // keys per block
constexpr int kRW = 128;   // band rows per block (kQ + kKB - 1, rounded up)
constexpr int kGW = 80;    // band columns per warp (16 + 64 - 1, rounded up)
constexpr int kGS = 80;    // f32 row stride of a warp's band strip
constexpr int kThreads = 128;

// 128-wide f16 rows (256 B) with the 16-byte chunk index xor-swizzled by
// (row & 7) so ldmatrix row gathers are bank-conflict free.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return static_cast<uint32_t>(row * 256 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(kThreads, 2) k2_relpos_attention(const AttnParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    // [0, 32K): Qu|Qv staging, then the warps' band strips (4 x 16 x 80 f32)
    uint8_t* sQ = smem;
    uint8_t* sK = smem + 32768;
    uint8_t* sV = sK + 16384;
    uint8_t* sR = sV + 16384;
    float* sG = reinterpret_cast<float*>(smem);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int head = blockIdx.y;
    const int2 wk = p.work[blockIdx.x];
    const int seg0 = p.cu[wk.x];
    const int T = p.cu[wk.x + 1] - seg0;
    const int q0 = wk.y;
    const size_t ld = 4096;
    const __half* base = p.qkv + static_cast<size_t>(seg0) * ld;

    // ── Q tiles (qu at column 0, qv at 1024) ──
    for (int c = threadIdx.x; c < 2 * kQ * 16; c += kThreads) {
        const int which = c >> 10, row = (c >> 4) & 63, ch = c & 15;
        const bool ok = q0 + row < T;
        const __half* src = base + static_cast<size_t>(ok ? q0 + row : 0) * ld + which * 1024 + head * 128 + ch * 8;
        cp_async16(smem_u32(sQ) + which * 16384 + swz(row, ch), src, ok);
    }
    cp_async_wait_all();
    __syncthreads();
    uint32_t qu[8][4], qv[8][4];
    {
        const int row = warp * 16 + (lane & 15);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int ch = 2 * kk + (lane >> 4);
            ldsm_x4(smem_u32(sQ) + swz(row, ch), qu[kk][0], qu[kk][1], qu[kk][2], qu[kk][3]);
            ldsm_x4(smem_u32(sQ) + 16384 + swz(row, ch), qv[kk][0], qv[kk][1], qv[kk][2], qv[kk][3]);
        }
    }
    __syncthreads();  // sQ becomes the band-strip area

    float o[16][4];
#pragma unroll
    for (int t = 0; t < 16; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY};
    float lrow[2] = {0.f, 0.f};
    const int g = lane >> 2, tg = lane & 3;
    float* gs = sG + warp * 16 * kGS;

    for (int k0 = 0; k0 < T; k0 += kKB) {
        // ── K, V (64 rows) and the band of R (128 rows, reversed offsets) ──
        for (int c = threadIdx.x; c < kKB * 16; c += kThreads) {
            const int row = c >> 4, ch = c & 15;
            const bool ok = k0 + row < T;
            const __half* src = base + static_cast<size_t>(ok ? k0 + row : 0) * ld + head * 128 + ch * 8;
            cp_async16(smem_u32(sK) + swz(row, ch), src + 2048, ok);
            cp_async16(smem_u32(sV) + swz(row, ch), src + 3072, ok);
        }
        // band row c holds offset d = q0 - k0 - 63 + c, i.e. R row r_center - d
        const int jtop = p.r_center - (q0 - k0 - (kKB - 1));
        for (int c = threadIdx.x; c < kRW * 16; c += kThreads) {
            const int row = c >> 4, ch = c & 15;
            const int j = jtop - row;
            const bool ok = j >= 0 && j < p.r_rows;
            const __half* src = p.R + static_cast<size_t>(ok ? j : 0) * 1024 + head * 128 + ch * 8;
            cp_async16(smem_u32(sR) + swz(row, ch), src, ok);
        }
        cp_async_wait_all();
        __syncthreads();

        // ── S = Qu K^T (16 x 64 per warp) ──
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int kk = 0; kk < 8; kk += 2) {
                uint32_t b0, b1, b2, b3_;
                ldsm_x4(smem_u32(sK) + swz(8 * j + (lane & 7), 2 * kk + (lane >> 3)), b0, b1, b2, b3_);
                mma16816(s[j], qu[kk], b0, b1);
                mma16816(s[j], qu[kk + 1], b2, b3_);
            }
        }
        // ── band strip G = Qv R_band^T (16 x 80 per warp) -> shared ──
#pragma unroll
        for (int jb = 0; jb < kGW / 8; ++jb) {
            float gacc[4] = {0.f, 0.f, 0.f, 0.f};
            const int rrow = warp * 16 + 8 * jb + (lane & 7);
#pragma unroll
            for (int kk = 0; kk < 8; kk += 2) {
                uint32_t b0, b1, b2, b3_;
                ldsm_x4(smem_u32(sR) + swz(rrow, 2 * kk + (lane >> 3)), b0, b1, b2, b3_);
                mma16816(gacc, qv[kk], b0, b1);
                mma16816(gacc, qv[kk + 1], b2, b3_);
            }
            *reinterpret_cast<float2*>(gs + g * kGS + 8 * jb + 2 * tg) = make_float2(gacc[0], gacc[1]);
            *reinterpret_cast<float2*>(gs + (g + 8) * kGS + 8 * jb + 2 * tg) = make_float2(gacc[2], gacc[3]);
        }
        __syncwarp();
        // ── add the diagonal of the strip, scale, mask, online softmax ──
        float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = g + ((e >> 1) << 3);
                const int kk = 8 * j + 2 * tg + (e & 1);
                float v = (s[j][e] + gs[r * kGS + (r - kk + kKB - 1)]) * p.scale_log2;
                if (k0 + kk >= T) v = -INFINITY;
                s[j][e] = v;
                mnew[e >> 1] = fmaxf(mnew[e >> 1], v);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 1));
            mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 2));
        }
        float corr[2], lsum[2] = {0.f, 0.f};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            corr[r] = exp2f(mrow[r] - mnew[r]);
            mrow[r] = mnew[r];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float pe = exp2f(s[j][e] - mrow[e >> 1]);
                s[j][e] = pe;
                lsum[e >> 1] += pe;
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * corr[r] + lsum[r];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            o[t][0] *= corr[0];
            o[t][1] *= corr[0];
            o[t][2] *= corr[1];
            o[t][3] *= corr[1];
        }
        // ── O += P V ──
#pragma unroll
        for (int ks = 0; ks < kKB / 16; ++ks) {
            uint32_t a[4];
            a[0] = h2u(s[2 * ks][0], s[2 * ks][1]);
            a[1] = h2u(s[2 * ks][2], s[2 * ks][3]);
            a[2] = h2u(s[2 * ks + 1][0], s[2 * ks + 1][1]);
            a[3] = h2u(s[2 * ks + 1][2], s[2 * ks + 1][3]);
            const int vrow = 16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
            for (int t = 0; t < 16; t += 2) {
                uint32_t b0, b1, b2, b3_;
                ldsm_x4_t(smem_u32(sV) + swz(vrow, t + (lane >> 4)), b0, b1, b2, b3_);
                mma16816(o[t], a, b0, b1);
                mma16816(o[t + 1], a, b2, b3_);
            }
        }
        __syncthreads();  // K/V/R and the strips are rewritten next block
    }

    // ── normalise and store (rows past T are not written) ──
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        float l = lrow[r];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        lrow[r] = 1.0f / l;
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int qi = q0 + warp * 16 + g + 8 * r;
        if (qi >= T) continue;
        __half* dst = p.out + static_cast<size_t>(seg0 + qi) * 1024 + head * 128 + 2 * tg;
#pragma unroll
        for (int t = 0; t < 16; ++t)
            *reinterpret_cast<uint32_t*>(dst + 8 * t) = h2u(o[t][2 * r] * lrow[r], o[t][2 * r + 1] * lrow[r]);
    }
}

}  // namespace

constexpr int kAttnSmem = 32768 + 16384 + 16384 + 32768;

int launch_attention(const AttnParams& p, int n_work, cudaStream_t st) {
    if (n_work <= 0) return 0;
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(k2_relpos_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
        if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(k2)", e);
        attr_done = true;
    }
    k2_relpos_attention<<<dim3(n_work, 8), kThreads, kAttnSmem, st>>>(p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("k2_relpos_attention", e);
}

int attention_block_rows() { return kQ; }

}  // namespace b3
