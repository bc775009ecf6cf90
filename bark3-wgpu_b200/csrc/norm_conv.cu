// norm_conv.cu — the memory-bound encoder kernels.
//
//   K4  LayerNorm over 1024 channels, one warp per frame, 16-byte loads,
//       shuffle reductions; optionally two norms back to back (a block's
//       norm_out followed by the next block's first pre-norm) in one pass.
//   K3b depthwise conv over time (k = 9, zero padding 4, utterance edges
//       treated as padding) + folded BatchNorm + SiLU.
//   plus the f32 -> f16 conversion of encoder inputs and the sinusoidal
//   relative-position table.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b3_internal.h"
#include "b3_kernels.h"

namespace b3 {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Two-pass mean / variance over the 32 values a lane holds (1024 per warp).
__device__ __forceinline__ void ln_stats(const float (&v)[32], float& mean, float& rstd) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) s += v[i];
    mean = warp_sum(s) * (1.0f / 1024.0f);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float d = v[i] - mean;
        q += d * d;
    }
    const float var = warp_sum(q) * (1.0f / 1024.0f);
    rstd = rsqrtf(var + 1e-5f);
}

// lane holds channels c = 4*lane + 128*i + j  (i = 0..7, j = 0..3)
__global__ void __launch_bounds__(256) k4_layernorm(const float* __restrict__ x, int rows,
                                                    const float* __restrict__ w1,
                                                    const float* __restrict__ b1,
                                                    float* __restrict__ y32,
                                                    const float* __restrict__ w2,
                                                    const float* __restrict__ b2,
                                                    __half* __restrict__ y16) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * 1024);
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 t = xr[lane + 32 * i];
        v[4 * i] = t.x;
        v[4 * i + 1] = t.y;
        v[4 * i + 2] = t.z;
        v[4 * i + 3] = t.w;
    }
    float mean, rstd;
    ln_stats(v, mean, rstd);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(w1) + lane + 32 * i);
        const float4 b = __ldg(reinterpret_cast<const float4*>(b1) + lane + 32 * i);
        v[4 * i] = (v[4 * i] - mean) * rstd * w.x + b.x;
        v[4 * i + 1] = (v[4 * i + 1] - mean) * rstd * w.y + b.y;
        v[4 * i + 2] = (v[4 * i + 2] - mean) * rstd * w.z + b.z;
        v[4 * i + 3] = (v[4 * i + 3] - mean) * rstd * w.w + b.w;
    }
    if (y32) {
        float4* yr = reinterpret_cast<float4*>(y32 + static_cast<size_t>(row) * 1024);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            yr[lane + 32 * i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    if (y16) {
        if (w2) {
            ln_stats(v, mean, rstd);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 w = __ldg(reinterpret_cast<const float4*>(w2) + lane + 32 * i);
                const float4 b = __ldg(reinterpret_cast<const float4*>(b2) + lane + 32 * i);
                v[4 * i] = (v[4 * i] - mean) * rstd * w.x + b.x;
                v[4 * i + 1] = (v[4 * i + 1] - mean) * rstd * w.y + b.y;
                v[4 * i + 2] = (v[4 * i + 2] - mean) * rstd * w.z + b.z;
                v[4 * i + 3] = (v[4 * i + 3] - mean) * rstd * w.w + b.w;
            }
        }
        uint2* yr = reinterpret_cast<uint2*>(y16 + static_cast<size_t>(row) * 1024);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            __half2 a = __floats2half2_rn(v[4 * i], v[4 * i + 1]);
            __half2 b = __floats2half2_rn(v[4 * i + 2], v[4 * i + 3]);
            yr[lane + 32 * i] = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
        }
    }
}

// Depthwise conv k=9 + BN(a, b) + SiLU.  Persistent: one CTA per SM walks
// tiles of kDwRows consecutive frames x all 1024 channels.  A tile's
// (kDwRows + 8)-frame input (with the +-4 halo) is staged in shared memory by
// cp.async into one of two buffers while the CTA convolves the previous tile
// from the other, so the loads of tile i+1 overlap the arithmetic and stores
// of tile i.  512 threads: thread (c4, half) owns channels 4 c4 .. 4 c4 + 3
// of rows [half * kDwHalf, half * kDwHalf + kDwHalf) and slides a 9-frame
// register window (pairs of channels, packed f32x2 FMAs) over them.  Frame t
// reads t-4 .. t+4 inside its own utterance [seg.x, seg.y); anything outside
// is zero.  Rows whose whole window lies inside the utterance take a path
// without per-tap tests; the taps are summed in the same order either way.
// A row's utterance bounds come from a per-frame [start, end) table.
constexpr int kDwRows = 40;
constexpr int kDwHalf = kDwRows / 2;
constexpr int kDwTile = kDwRows + 8;
constexpr int kDwTileBytes = kDwTile * 1024 * 2;
constexpr int kDwSmem = 2 * kDwTileBytes;
constexpr int kDwThreads = 512;

__global__ void __launch_bounds__(kDwThreads, 1) k3_dwconv_bn_silu(const __half* __restrict__ src,
                                                                   const int2* __restrict__ seg, int rows,
                                                                   const float* __restrict__ dw_t,  // [9][1024]
                                                                   const float* __restrict__ bn_a,
                                                                   const float* __restrict__ bn_b,
                                                                   __half* __restrict__ dst) {
    extern __shared__ __align__(16) uint8_t tiles[];  // 2 x [kDwTile][1024] f16, frame t0-4+i in row i
    const int c4 = threadIdx.x & 255;
    const int c0 = c4 * 4;
    const int rbeg = (threadIdx.x >> 8) * kDwHalf;
    const int n_tiles = (rows + kDwRows - 1) / kDwRows;
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(tiles));
    // rows past the end of the input are zero-filled (cp.async with 0 source bytes)
    auto stage = [&](int tile, int buf) {
        const int t0 = tile * kDwRows;
        for (int c = threadIdx.x; c < kDwTile * 128; c += kDwThreads) {
            const int r = c >> 7, ch = c & 127;
            const int t = t0 - 4 + r;
            const bool ok = t >= 0 && t < rows;
            const __half* g = src + static_cast<size_t>(ok ? t : 0) * 1024 + ch * 8;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sbase + buf * kDwTileBytes + r * 2048 + ch * 16),
                         "l"(g), "r"(ok ? 16 : 0)
                         : "memory");
        }
    };
    float2 w[9][2];
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(dw_t + i * 1024 + c0));
        w[i][0] = make_float2(a.x, a.y);
        w[i][1] = make_float2(a.z, a.w);
    }
    float2 ba[2], bb[2];
    {
        const float4 a = __ldg(reinterpret_cast<const float4*>(bn_a + c0));
        const float4 b = __ldg(reinterpret_cast<const float4*>(bn_b + c0));
        ba[0] = make_float2(a.x, a.y);
        ba[1] = make_float2(a.z, a.w);
        bb[0] = make_float2(b.x, b.y);
        bb[1] = make_float2(b.z, b.w);
    }
    if (static_cast<int>(blockIdx.x) < n_tiles) stage(blockIdx.x, 0);
    asm volatile("cp.async.commit_group;" ::: "memory");
    int buf = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, buf ^= 1) {
        const int next = tile + gridDim.x;
        const int t0 = tile * kDwRows;
        // utterance bounds of this thread's first and last row, fetched before
        // the wait: with at most one utterance boundary inside its rows (the
        // first row's utterance ends where the last row's begins, or both rows
        // share one) every row's bounds are one of the two, and no row needs a
        // dependent load of its own
        const int ta = t0 + rbeg < rows ? t0 + rbeg : rows - 1;
        const int tz = t0 + rbeg + kDwHalf - 1 < rows ? t0 + rbeg + kDwHalf - 1 : rows - 1;
        const int2 sga = __ldg(seg + ta), sgz = __ldg(seg + tz);
        const bool two_segs = sga.y >= sgz.x;
        if (next < n_tiles) stage(next, buf ^ 1);
        asm volatile("cp.async.commit_group;" ::: "memory");   // possibly empty: keeps the group count fixed
        asm volatile("cp.async.wait_group 1;" ::: "memory");   // this tile's group has landed
        __syncthreads();
        const uint8_t* tb = tiles + buf * kDwTileBytes;
        auto load = [&](int r, float2 (&d)[2]) {
            const uint2 u = *reinterpret_cast<const uint2*>(tb + r * 2048 + c0 * 2);
            d[0] = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            d[1] = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        };
        // circular 9-frame window: tile row r lives in slot (r - rbeg) % 9; the
        // row loop is unrolled by 9 so every slot index is a compile-time constant
        float2 win[9][2];
#pragma unroll
        for (int i = 0; i < 8; ++i) load(rbeg + i, win[i]);
#pragma unroll 1
        for (int r0 = 0; r0 < kDwHalf; r0 += 9) {
#pragma unroll
            for (int u = 0; u < 9; ++u) {
                const int r = rbeg + r0 + u;
                const int t = t0 + r;
                if (r0 + u < kDwHalf && t < rows) {
                    load(r + 8, win[(u + 8) % 9]);
                    const int2 sg = two_segs ? (t < sga.y ? sga : sgz) : __ldg(seg + t);
                    const int lo = max(sg.x - (t - 4), 0);
                    const int hi = min(sg.y - (t - 4), 9);
                    float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                    if (lo == 0 && hi == 9) {
#pragma unroll
                        for (int i = 0; i < 9; ++i) {
                            acc[0] = __ffma2_rn(win[(u + i) % 9][0], w[i][0], acc[0]);
                            acc[1] = __ffma2_rn(win[(u + i) % 9][1], w[i][1], acc[1]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 9; ++i) {
                            if (i < lo || i >= hi) continue;
                            acc[0] = __ffma2_rn(win[(u + i) % 9][0], w[i][0], acc[0]);
                            acc[1] = __ffma2_rn(win[(u + i) % 9][1], w[i][1], acc[1]);
                        }
                    }
                    uint32_t o[2];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const float2 y = __ffma2_rn(acc[j], ba[j], bb[j]);
                        const float y0 = __fdividef(y.x, 1.0f + __expf(-y.x));
                        const float y1 = __fdividef(y.y, 1.0f + __expf(-y.y));
                        __half2 h = __floats2half2_rn(y0, y1);
                        o[j] = *reinterpret_cast<uint32_t*>(&h);
                    }
                    *reinterpret_cast<uint2*>(dst + static_cast<size_t>(t) * 1024 + c0) = make_uint2(o[0], o[1]);
                }
            }
        }
        __syncthreads();   // every thread is done with this buffer before it is restaged
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// f32 -> f16 (round to nearest even).  A thread converts kCvtUnroll float4s
// per pass with all their loads issued first (streaming: the f32 source is
// read once, while the f16 result should stay in L2 for the GEMM behind it).
constexpr int kCvtUnroll = 4;
__global__ void k_f32_to_f16(const float4* __restrict__ src, uint2* __restrict__ dst, int64_t n4) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i0 < n4;
         i0 += stride * kCvtUnroll) {
        float4 v[kCvtUnroll];
#pragma unroll
        for (int u = 0; u < kCvtUnroll; ++u) {
            const int64_t i = i0 + u * stride;
            v[u] = i < n4 ? __ldcs(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kCvtUnroll; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < n4) {
                __half2 a = __floats2half2_rn(v[u].x, v[u].y);
                __half2 b = __floats2half2_rn(v[u].z, v[u].w);
                dst[i] = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
            }
        }
    }
}

// Row j is relative position (tcap - 1 - j): [sin, cos] interleaved with the
// reference's f32 inverse frequencies (src/encoder.rs:228-246).
__global__ void k_pos_table(const float* __restrict__ inv_freq, int tcap, int rows,
                            __half2* __restrict__ out) {
    const int j = blockIdx.x;
    if (j >= rows) return;
    const float pos = static_cast<float>(tcap - 1 - j);
    for (int i = threadIdx.x; i < 512; i += blockDim.x) {
        const float f = pos * inv_freq[i];
        out[static_cast<size_t>(j) * 512 + i] = __floats2half2_rn(sinf(f), cosf(f));
    }
}

}  // namespace

int launch_layernorm(const float* x, int rows, const float* w1, const float* b1, float* y32,
                     const float* w2, const float* b2, __half* y16, cudaStream_t st) {
    if (rows <= 0) return 0;
    k4_layernorm<<<(rows + 7) / 8, 256, 0, st>>>(x, rows, w1, b1, y32, w2, b2, y16);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("k4_layernorm", e);
}

int launch_dwconv(const __half* src, const int2* seg, int rows, const float* dw_t, const float* bn_a,
                  const float* bn_b, __half* dst, cudaStream_t st) {
    if (rows <= 0) return 0;
    static PerDeviceOnce attr;
    const int rc0 = set_smem_limit_once(attr, k3_dwconv_bn_silu, kDwSmem, "cudaFuncSetAttribute(k3)");
    if (rc0) return rc0;
    const int n_sms = device_sms();
    const int tiles = (rows + kDwRows - 1) / kDwRows;
    k3_dwconv_bn_silu<<<tiles < n_sms ? tiles : n_sms, kDwThreads, kDwSmem, st>>>(src, seg, rows, dw_t, bn_a, bn_b, dst);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("k3_dwconv_bn_silu", e);
}

int launch_f32_to_f16(const float* src, __half* dst, int64_t n, cudaStream_t st) {
    if (n <= 0) return 0;
    if (n % 4) return set_error(B3_EINVAL, "f32->f16 length %lld not a multiple of 4", (long long)n);
    const int64_t n4 = n / 4;
    int64_t blocks = (n4 + 256 * kCvtUnroll - 1) / (256 * kCvtUnroll);
    if (blocks > 8 * device_sms()) blocks = 8 * device_sms();   // one wave of 8 CTAs per SM
    k_f32_to_f16<<<static_cast<int>(blocks), 256, 0, st>>>(reinterpret_cast<const float4*>(src), reinterpret_cast<uint2*>(dst), n4);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("k_f32_to_f16", e);
}

int launch_pos_table(const float* inv_freq, int tcap, int rows, __half* out, cudaStream_t st) {
    if (rows <= 0) return 0;
    k_pos_table<<<rows, 256, 0, st>>>(inv_freq, tcap, rows, reinterpret_cast<__half2*>(out));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("k_pos_table", e);
}

}  // namespace b3
