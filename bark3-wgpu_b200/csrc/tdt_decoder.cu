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
//   LSTM layer 0  gates = [emb | h0] . [W_ih | W_hh]^T + b   (K1) + update
//   LSTM layer 1  gates = [h0 | h1] . [W_ih | W_hh]^T + b    (K1) + update
//   projector     dec = h1 . W_p^T + b                       (K1)
// Rows that did not emit keep their LSTM state (their gates are computed and
// dropped), so recomputing dec for them reproduces the same value.
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

namespace b3 {

namespace {

constexpr int kH = 640;

__device__ __forceinline__ void split_store(__half* hi, __half* lo, float v) {
    const __half h = __float2half_rn(v);
    *hi = h;
    *lo = __float2half_rn(v - __half2float(h));
}

__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

// Initial state: h = c = 0, every row runs one LSTM step on the blank
// embedding (src/tdt.rs:424-428).
__global__ void k_dec_init(DecState s) {
    const int b = blockIdx.x;
    if (b >= s.B) return;
    const int T = s.cu[b + 1] - s.cu[b];
    for (int j = threadIdx.x; j < kH; j += blockDim.x) {
        const __half* eh = s.emb_hi + static_cast<size_t>(s.blank) * kH;
        const __half* el = s.emb_lo + static_cast<size_t>(s.blank) * kH;
        __half* a0 = s.a0 + static_cast<size_t>(b) * 4 * kH;
        __half* a1 = s.a1 + static_cast<size_t>(b) * 4 * kH;
        a0[j] = eh[j];
        a0[kH + j] = el[j];
        a0[2 * kH + j] = __float2half_rn(0.f);
        a0[3 * kH + j] = __float2half_rn(0.f);
        a1[2 * kH + j] = __float2half_rn(0.f);
        a1[3 * kH + j] = __float2half_rn(0.f);
        s.c[(static_cast<size_t>(b) * 2 + 0) * kH + j] = 0.f;
        s.c[(static_cast<size_t>(b) * 2 + 1) * kH + j] = 0.f;
    }
    if (threadIdx.x == 0) {
        s.frame[b] = 0;
        s.count[b] = 0;
        s.guard[b] = 0;
        s.emit[b] = 1;
        s.active[b] = T > 0 ? 1 : 0;
    }
}

// x_b = ReLU(enc[frame_b] + dec_b), split into hi | lo (zeros for finished rows).
__global__ void k_dec_joint_in(DecState s) {
    const int b = blockIdx.x;
    if (b >= s.B) return;
    const bool act = s.active[b] != 0;
    const float* enc = s.pooler + static_cast<size_t>(s.cu[b] + (act ? s.frame[b] : 0)) * kH;
    const float* dec = s.dec + static_cast<size_t>(b) * kH;
    __half* aj = s.aj + static_cast<size_t>(b) * 2 * kH;
    for (int j = threadIdx.x; j < kH; j += blockDim.x) {
        float v = act ? enc[j] + dec[j] : 0.f;
        v = v > 0.f ? v : 0.f;
        split_store(aj + j, aj + kH + j, v);
    }
}

// Argmax over one row of scores and the step's state update.  One block per
// utterance; ties keep the lowest index (the reference's strict `>` scan).
__global__ void __launch_bounds__(256) k_dec_argmax(DecState s) {
    const int b = blockIdx.x;
    if (b >= s.B) return;
    __shared__ float bv_t[256], bv_d[256];
    __shared__ int bi_t[256], bi_d[256];
    if (!s.active[b]) {
        if (threadIdx.x == 0) s.emit[b] = 0;
        return;
    }
    const float* row = s.scores + static_cast<size_t>(b) * s.ld_scores;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    for (int r = threadIdx.x; r < s.vocab; r += blockDim.x) {
        const float v = row[r];
        if (v > best) {
            best = v;
            bidx = r;
        }
    }
    float dbest = -INFINITY;
    int didx = 0x7fffffff;
    if (threadIdx.x < 5) {
        dbest = row[s.vocab + threadIdx.x];
        didx = threadIdx.x;
    }
    bv_t[threadIdx.x] = best;
    bi_t[threadIdx.x] = bidx;
    bv_d[threadIdx.x] = dbest;
    bi_d[threadIdx.x] = didx;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o) {
            const int u = threadIdx.x + o;
            if (bv_t[u] > bv_t[threadIdx.x] || (bv_t[u] == bv_t[threadIdx.x] && bi_t[u] < bi_t[threadIdx.x])) {
                bv_t[threadIdx.x] = bv_t[u];
                bi_t[threadIdx.x] = bi_t[u];
            }
            if (bv_d[u] > bv_d[threadIdx.x] || (bv_d[u] == bv_d[threadIdx.x] && bi_d[u] < bi_d[threadIdx.x])) {
                bv_d[threadIdx.x] = bv_d[u];
                bi_d[threadIdx.x] = bi_d[u];
            }
        }
        __syncthreads();
    }
    int tok = bi_t[0];
    int dur = bi_d[0];
    if (tok == 0x7fffffff) tok = 0;   // every score NaN: mirrors the reference's initial index
    if (dur == 0x7fffffff) dur = 0;
    const int T = s.cu[b + 1] - s.cu[b];
    const bool emit = tok != s.blank;
    if (threadIdx.x == 0) {
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
        } else {
            s.frame[b] = frame + (dur > 0 ? dur : 1);
        }
        const int g = s.guard[b] + 1;
        s.guard[b] = g;
        s.emit[b] = emit ? 1 : 0;
        const long max_steps = static_cast<long>(T) * (10 + 4) + 64;
        s.active[b] = (s.frame[b] < T && g < max_steps) ? 1 : 0;
    }
    if (emit) {
        const __half* eh = s.emb_hi + static_cast<size_t>(tok) * kH;
        const __half* el = s.emb_lo + static_cast<size_t>(tok) * kH;
        __half* a0 = s.a0 + static_cast<size_t>(b) * 4 * kH;
        for (int j = threadIdx.x; j < kH; j += blockDim.x) {
            a0[j] = eh[j];
            a0[kH + j] = el[j];
        }
    }
}

// LSTM cell update for rows that emitted: gates [B][2560] (i, f, g, o).
__global__ void k_dec_lstm_update(DecState s, int layer) {
    const int b = blockIdx.x;
    if (b >= s.B || !s.emit[b]) return;
    const float* g = s.gates + static_cast<size_t>(b) * 4 * kH;
    float* c = s.c + (static_cast<size_t>(b) * 2 + layer) * kH;
    __half* self = (layer == 0 ? s.a0 : s.a1) + static_cast<size_t>(b) * 4 * kH;
    __half* next = layer == 0 ? s.a1 + static_cast<size_t>(b) * 4 * kH : s.ap + static_cast<size_t>(b) * 2 * kH;
    for (int j = threadIdx.x; j < kH; j += blockDim.x) {
        const float in = sigm(g[j]);
        const float fg = sigm(g[kH + j]);
        const float cand = tanhf(g[2 * kH + j]);
        const float cn = fg * c[j] + in * cand;
        c[j] = cn;
        const float out = sigm(g[3 * kH + j]);
        const float h = out * tanhf(cn);
        split_store(self + 2 * kH + j, self + 3 * kH + j, h);  // this layer's recurrent input
        split_store(next + j, next + kH + j, h);                // next layer's input
    }
}

__global__ void k_dec_any_active(const int* active, int B, int* out) {
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

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error(what, e);
}

}  // namespace

int dec_launch_init(const DecState& s, cudaStream_t st) {
    k_dec_init<<<s.B, 128, 0, st>>>(s);
    return check_launch("k_dec_init");
}
int dec_launch_joint_in(const DecState& s, cudaStream_t st) {
    k_dec_joint_in<<<s.B, 128, 0, st>>>(s);
    return check_launch("k_dec_joint_in");
}
int dec_launch_argmax(const DecState& s, cudaStream_t st) {
    k_dec_argmax<<<s.B, 256, 0, st>>>(s);
    return check_launch("k_dec_argmax");
}
int dec_launch_lstm_update(const DecState& s, int layer, cudaStream_t st) {
    k_dec_lstm_update<<<s.B, 128, 0, st>>>(s, layer);
    return check_launch("k_dec_lstm_update");
}
int dec_launch_any_active(const DecState& s, int* out, cudaStream_t st) {
    k_dec_any_active<<<1, 256, 0, st>>>(s.active, s.B, out);
    return check_launch("k_dec_any_active");
}
int dec_launch_split(const float* src, __half* hi, __half* lo, int64_t n, cudaStream_t st) {
    int blocks = static_cast<int>((n + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    k_split_rows<<<blocks, 256, 0, st>>>(src, hi, lo, n);
    return check_launch("k_split_rows");
}

}  // namespace b3
