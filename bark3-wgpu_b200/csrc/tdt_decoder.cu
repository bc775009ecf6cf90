// tdt_decoder.cu — batched greedy TDT decoding (the reference decodes one
// utterance at a time on the CPU, src/tdt.rs:416-467, or with one WGSL
// workgroup set per step, src/tdt_gpu.rs).
//
// All utterances of a batch advance in lock step: one step is
//   joint input   x_b = ReLU(enc_b[frame_b] + dec_b)                 (this file)
//   joint GEMM    scores = x . head^T + bias          (K1, tensor cores)
//   argmax/update first-max token over the vocabulary, first-max duration
//                 over the 5 duration rows; blank advances >= 1 frame, a
//                 token is recorded and advances `duration` frames   (this file)
//   LSTM layer 0  gates = E0[token] + h0 . W_hh^T             (K1) + update
//   LSTM layer 1  gates = [h0 | h1] . [W_ih | W_hh]^T + b     (K1) + update
//   projector     dec = h1 . W_p^T + b                        (K1)
// E0[v] = W_ih0 . emb(v) + b_ih0 + b_hh0 is computed once per vocabulary
// entry at load, so layer 0's GEMM only carries the recurrent half.  Rows
// that did not emit keep their LSTM state (their gates are computed and
// dropped), so recomputing dec for them reproduces the same value.
//
// The GEMMs have M = batch rows only, so K1 runs them split-K over all SMs;
// every consumer below adds the K parts in a fixed order (deterministic).
//
// Precision: each GEMM input x is split into f16 hi = f16(x) and
// lo = f16(x - hi) and the weight is repeated along K ([W | W]), so the
// tensor cores see ~22 significant bits of every activation against the
// reference's f16 weights with f32 accumulation.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

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

// x_b = ReLU(enc[frame_b] + dec_b), split into hi | lo (zeros for finished
// rows).  One block of 160 threads per row, 4 columns per thread.
__global__ void __launch_bounds__(160) k_dec_joint_in(DecState s) {
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.x;
    if (b >= s.B) return;
    const int j = 4 * threadIdx.x;
    const bool act = s.active[b] != 0;
    __half* aj = s.aj + static_cast<size_t>(b) * 2 * kH;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (act) {
        const float4 e = __ldg(reinterpret_cast<const float4*>(s.pooler + static_cast<size_t>(s.row0[b] + s.frame[b]) * kH + j));
        const float4 d = parts_sum4(s.dec, s.ks_p, s.prow, kH, b, j);
        v = make_float4(fmaxf(e.x + d.x, 0.f), fmaxf(e.y + d.y, 0.f), fmaxf(e.z + d.z, 0.f), fmaxf(e.w + d.w, 0.f));
    }
    split_store4(aj + j, aj + kH + j, v);
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

// Argmax over one row of scores and the step's state update.  One block of
// 256 threads per utterance; each thread scans 4 consecutive vocabulary
// entries per 1024-wide chunk; ties keep the lowest index.
__global__ void __launch_bounds__(256) k_dec_argmax(DecState s) {
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.x;
    if (b >= s.B) return;
    __shared__ float wv[8];
    __shared__ int wi[8];
    __shared__ int wdur;
    if (!s.active[b]) {
        if (threadIdx.x == 0) s.emit[b] = 0;
        return;
    }
    const int ld = s.ld_scores;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    for (int base = 4 * threadIdx.x; base < s.vocab; base += 1024) {
        const float4 v = parts_sum4(s.scores, s.ks_h, s.prow, ld, b, base);
        const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (base + q < s.vocab && e[q] > best) {   // increasing index: strict > keeps the first max
                best = e[q];
                bidx = base + q;
            }
    }
    warp_argmax(best, bidx);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        wv[warp] = best;
        wi[warp] = bidx;
    }
    if (warp == 0) {
        // durations: the 5 rows after the vocabulary, first max
        float dv = -INFINITY;
        int di = 0x7fffffff;
        if (lane < 5) {
            dv = parts_sum1(s.scores, s.ks_h, s.prow, ld, b, s.vocab + lane);
            di = lane;
        }
        warp_argmax(dv, di);
        if (lane == 0) wdur = di;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    float tv = wv[0];
    int tok = wi[0];
    for (int w = 1; w < 8; ++w)
        if (wins(wv[w], wi[w], tv, tok)) {
            tv = wv[w];
            tok = wi[w];
        }
    int dur = wdur;
    if (tok == 0x7fffffff) tok = 0;   // every score NaN: mirrors the reference's initial index
    if (dur == 0x7fffffff) dur = 0;
    const int T = s.len[b];
    const bool emit = tok != s.blank;
    const int frame = s.frame[b];
    if (emit) {
        const int n = s.count[b];
        if (n < s.max_tokens) {
            uint32_t* t = s.tokens + (static_cast<size_t>(b) * s.max_tokens + n) * 3;
            t[0] = static_cast<uint32_t>(tok);
            t[1] = static_cast<uint32_t>(frame);
            t[2] = static_cast<uint32_t>(dur);
        }
        s.count[b] = n + 1;
        s.frame[b] = frame + dur;
        s.tok[b] = tok;
    } else {
        s.frame[b] = frame + (dur > 0 ? dur : 1);
    }
    const int g = s.guard[b] + 1;
    s.guard[b] = g;
    s.emit[b] = emit ? 1 : 0;
    const long max_steps = static_cast<long>(T) * (10 + 4) + 64;
    s.active[b] = (s.frame[b] < T && g < max_steps) ? 1 : 0;
}

// LSTM cell update for rows that emitted: gates [B][2560] (i, f, g, o).
// One block of 160 threads per row, 4 columns per thread.
__global__ void __launch_bounds__(160) k_dec_lstm_update(DecState s, int layer) {
    pdl_wait();
    pdl_launch_dependents();
    const int b = blockIdx.x;
    if (b >= s.B || !s.emit[b]) return;
    const int j = 4 * threadIdx.x;
    const int parts = layer == 0 ? s.ks_g0 : s.ks_g1;
    float4 g[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) g[q] = parts_sum4(s.gates, parts, s.prow, 4 * kH, b, q * kH + j);
    if (layer == 0) {
        const float* e0 = s.e0 + static_cast<size_t>(s.tok[b]) * 4 * kH + j;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 e = __ldg(reinterpret_cast<const float4*>(e0 + q * kH));
            g[q].x += e.x;
            g[q].y += e.y;
            g[q].z += e.z;
            g[q].w += e.w;
        }
    }
    float* cp = s.c + (static_cast<size_t>(b) * 2 + layer) * kH + j;
    const float4 c4 = *reinterpret_cast<const float4*>(cp);
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
    *reinterpret_cast<float4*>(cp) = make_float4(cn[0], cn[1], cn[2], cn[3]);
    // this layer's recurrent input and the next GEMM's input (hi | lo)
    __half* self = layer == 0 ? s.a0 + static_cast<size_t>(b) * 2 * kH : s.a1 + static_cast<size_t>(b) * 4 * kH + 2 * kH;
    __half* next = layer == 0 ? s.a1 + static_cast<size_t>(b) * 4 * kH : s.ap + static_cast<size_t>(b) * 2 * kH;
    const float4 h4 = make_float4(h[0], h[1], h[2], h[3]);
    split_store4(self + j, self + kH + j, h4);
    split_store4(next + j, next + kH + j, h4);
}

__global__ void k_dec_any_active(const int* active, int B, int* out) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ int any;
    if (threadIdx.x == 0) any = 0;
    __syncthreads();
    for (int b = threadIdx.x; b < B; b += blockDim.x)
        if (active[b]) any = 1;
    __syncthreads();
    if (threadIdx.x == 0) *out = any;
}

// Embedding rows as f16 hi | lo (load time).
__global__ void k_split_rows(const float* __restrict__ src, __half* hi, __half* lo, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        split_store(hi + i, lo + i, src[i]);
}

// Row b of a decoder group -> utterance out_row[b] of the batch outputs.
__global__ void __launch_bounds__(256) k_dec_gather(const uint32_t* __restrict__ tokens, const int* __restrict__ count,
                                                    const int* __restrict__ out_row, int B, int max_tokens,
                                                    uint32_t* __restrict__ out_tokens, int* __restrict__ out_count) {
    const int b = blockIdx.x;
    if (b >= B) return;
    const int u = out_row[b];
    const int n = count[b];
    if (threadIdx.x == 0) out_count[u] = n;
    const int words = 3 * (n < max_tokens ? n : max_tokens);
    const uint32_t* src = tokens + static_cast<size_t>(b) * max_tokens * 3;
    uint32_t* dst = out_tokens + static_cast<size_t>(u) * max_tokens * 3;
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error(what, e);
}

}  // namespace

int dec_max_parts() { return kMaxParts; }

// The step kernels are launched with programmatic stream serialization: each
// one's CTAs are scheduled while its predecessor drains and wait in pdl_wait()
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
int dec_launch_joint_in(const DecState& s, cudaStream_t st) {
    return launch_pdl(k_dec_joint_in, dim3(s.B), dim3(kH / 4), st, "k_dec_joint_in", s);
}
int dec_launch_argmax(const DecState& s, cudaStream_t st) {
    return launch_pdl(k_dec_argmax, dim3(s.B), dim3(256), st, "k_dec_argmax", s);
}
int dec_launch_lstm_update(const DecState& s, int layer, cudaStream_t st) {
    return launch_pdl(k_dec_lstm_update, dim3(s.B), dim3(kH / 4), st, "k_dec_lstm_update", s, layer);
}
int dec_launch_any_active(const DecState& s, int* out, cudaStream_t st) {
    return launch_pdl(k_dec_any_active, dim3(1), dim3(256), st, "k_dec_any_active", static_cast<const int*>(s.active),
                      s.B, out);
}
int dec_launch_gather(const DecState& s, const int* out_row, uint32_t* out_tokens, int* out_count, cudaStream_t st) {
    k_dec_gather<<<s.B, 256, 0, st>>>(s.tokens, s.count, out_row, s.B, s.max_tokens, out_tokens, out_count);
    return check_launch("k_dec_gather");
}

int dec_launch_split(const float* src, __half* hi, __half* lo, int64_t n, cudaStream_t st) {
    int blocks = static_cast<int>((n + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    k_split_rows<<<blocks, 256, 0, st>>>(src, hi, lo, n);
    return check_launch("k_split_rows");
}

}  // namespace b3
