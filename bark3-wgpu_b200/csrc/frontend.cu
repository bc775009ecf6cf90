// frontend.cu — log-mel features and conv subsampling on the GPU (the
// reference computes the mel on the CPU, src/mel.rs:41-138, and subsamples
// on the CPU or with WGSL, src/sub.rs:107-300, src/sub_gpu.rs).
//
// Mel: one CTA per frame: pre-emphasis (0.97), 512-point centred frame with
// the symmetric Hann(400) window, radix-2 complex FFT in shared memory (f32),
// power of the 257 bins, 128 slaney mel bins (sparse rows), log(x + 2^-24).
// Normalisation: one CTA per utterance, one thread per mel bin, mean and
// sample std over the valid frames (frames >= len/160 zeroed).
//
// Subsampling, channels-last in HBM ([time][freq][channel]):
//   conv0 (1 -> 256, 3x3, stride 2, pad 1) + ReLU + time mask and the first
//   depthwise 3x3 stride-2 conv + mask are one kernel: the conv0 tile a CTA
//   needs lives in shared memory only;
//   the two pointwise 256 -> 256 convs (+ bias + ReLU) run on K1;
//   the second depthwise conv + mask sits between them.
// The last pointwise conv writes [T][16 freq][256 ch] f16 rows, which is the
// encoder's input row with its columns in (freq, channel) order; the
// encoder's subsampling linear is loaded with its columns permuted to match.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b3_internal.h"
#include "b3_kernels.h"

namespace b3 {

namespace {

constexpr int kNfft = 512;
constexpr int kHop = 160;
constexpr int kMel = 128;

__device__ __forceinline__ int conv_len_d(int l) { return (l - 1) / 2 + 1; }

// One frame per CTA (256 threads).  frame -> utterance by binary search in
// the frame offsets.
__global__ void __launch_bounds__(256) k_mel_frames(MelParams p) {
    __shared__ float re[kNfft], im[kNfft], pw[257];
    const int f = blockIdx.x;
    int lo = 0, hi = p.n_utt;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (p.frame_off[mid] <= f) lo = mid; else hi = mid;
    }
    const int u = lo;
    const int t = f - p.frame_off[u];
    const float* x = p.wave + p.wave_off[u];
    const int64_t len = p.wave_off[u + 1] - p.wave_off[u];
    const int64_t start = static_cast<int64_t>(t) * kHop - kNfft / 2;
    for (int i = threadIdx.x; i < kNfft; i += blockDim.x) {
        const int64_t s = start + i;
        float v = 0.f;
        if (s >= 0 && s < len) {
            const float cur = x[s];
            v = (s == 0 ? cur : cur - 0.97f * x[s - 1]) * p.window[i];
        }
        const int r = __brev(i) >> (32 - 9);  // bit-reversed position
        re[r] = v;
        im[r] = 0.f;
    }
    __syncthreads();
    for (int half = 1; half < kNfft; half <<= 1) {
        const int b = threadIdx.x;  // 256 butterflies per stage
        const int grp = b / half, k = b % half;
        const int i0 = grp * 2 * half + k, i1 = i0 + half;
        const float2 w = p.twiddle[k * (kNfft / (2 * half))];  // exp(-2 pi i k / (2 half))
        const float vr = re[i1] * w.x - im[i1] * w.y;
        const float vi = re[i1] * w.y + im[i1] * w.x;
        const float ur = re[i0], ui = im[i0];
        re[i0] = ur + vr;
        im[i0] = ui + vi;
        re[i1] = ur - vr;
        im[i1] = ui - vi;
        __syncthreads();
    }
    for (int k = threadIdx.x; k < 257; k += blockDim.x) pw[k] = re[k] * re[k] + im[k] * im[k];
    __syncthreads();
    if (threadIdx.x < kMel) {
        const int m = threadIdx.x;
        const int k0 = p.fb_lo[m], k1 = p.fb_hi[m];
        float s = 0.f;
        for (int k = k0; k < k1; ++k) s += p.fb[m * 257 + k] * pw[k];
        p.mel[static_cast<size_t>(f) * kMel + m] = logf(s + 5.9604645e-08f);
    }
}

// Per-utterance normalisation over the valid frames (src/mel.rs:103-136).
__global__ void k_mel_norm(MelParams p) {
    const int u = blockIdx.x;
    const int m = threadIdx.x;
    if (u >= p.n_utt || m >= kMel) return;
    const int f0 = p.frame_off[u];
    const int nf = p.frame_off[u + 1] - f0;
    const int nvalid = static_cast<int>((p.wave_off[u + 1] - p.wave_off[u]) / kHop);
    const int nv = nvalid > 1 ? nvalid : 1;
    float* mel = p.mel + static_cast<size_t>(f0) * kMel + m;
    float s = 0.f;
    for (int t = 0; t < nvalid; ++t) s += mel[static_cast<size_t>(t) * kMel];
    const float mean = s / static_cast<float>(nv);
    float q = 0.f;
    for (int t = 0; t < nvalid; ++t) {
        const float d = mel[static_cast<size_t>(t) * kMel] - mean;
        q += d * d;
    }
    const float sd = sqrtf(q / static_cast<float>(nv - 1 > 1 ? nv - 1 : 1));
    const float inv = 1.0f / (sd + 1e-5f);
    for (int t = 0; t < nf; ++t) {
        float& v = mel[static_cast<size_t>(t) * kMel];
        v = t < nvalid ? (v - mean) * inv : 0.f;
    }
}

// conv0 + ReLU + mask, then depthwise conv1 + mask, for 8 output rows (t2) x
// all 32 freq columns x 16 channels.  The conv0 tile (17 rows x 64 cols x 16
// channels, f32) and the mel rows it needs (35 x 128) stay in shared memory.
constexpr int kT2 = 8;
constexpr int kC = 16;
constexpr int kT1 = 2 * kT2 + 1;   // conv0 rows needed
constexpr int kTm = 2 * kT1 + 1;   // mel rows needed

constexpr int kSubSmem = (kTm * (kMel + 2) + kT1 * 65 * kC) * 4;

__global__ void __launch_bounds__(256) k_sub_conv0_dw1(SubParams p) {
    extern __shared__ float sub_smem[];
    auto mel = reinterpret_cast<float(*)[kMel + 2]>(sub_smem);                    // [kTm][130]: cols -1 .. 128
    auto c0 = reinterpret_cast<float(*)[65][kC]>(sub_smem + kTm * (kMel + 2));   // [kT1][65][kC]: cols -1 .. 63
    const int4 wk = p.work[blockIdx.x];    // (utterance, t2_0, channel group)
    const int u = wk.x, t2_0 = wk.y, cg = wk.z * kC;
    const int F = p.mel_off[u + 1] - p.mel_off[u];
    const int F1 = conv_len_d(F), F2 = conv_len_d(F1);
    const int nvalid = p.n_valid[u];
    const int v1 = conv_len_d(nvalid > 1 ? nvalid : 1);
    const int v2 = conv_len_d(v1);
    const float* melu = p.mel + static_cast<size_t>(p.mel_off[u]) * kMel;
    const int t1_0 = 2 * t2_0 - 1;      // first conv0 row
    const int tm_0 = 2 * t1_0 - 1;      // first mel row
    for (int i = threadIdx.x; i < kTm * (kMel + 2); i += blockDim.x) {
        const int r = i / (kMel + 2), cidx = i % (kMel + 2);
        const int tm = tm_0 + r, fm = cidx - 1;
        mel[r][cidx] = (tm >= 0 && tm < F && fm >= 0 && fm < kMel) ? melu[static_cast<size_t>(tm) * kMel + fm] : 0.f;
    }
    __syncthreads();
    // conv0: out(t1, j) = relu(b + sum_{ki,kj} w * mel[2 t1 + ki - 1][2 j + kj - 1]), zero when masked or outside
    for (int i = threadIdx.x; i < kT1 * 65 * kC; i += blockDim.x) {
        const int c = i % kC, jj = (i / kC) % 65, r = i / (kC * 65);
        const int t1 = t1_0 + r, j = jj - 1;
        float s = 0.f;
        if (t1 >= 0 && t1 < F1 && t1 < v1 && j >= 0 && j < 64) {
            const float* w = p.w0 + (cg + c) * 9;
            s = p.b0[cg + c];
#pragma unroll
            for (int t = 0; t < 9; ++t) {
                const int ki = t / 3, kj = t % 3;
                s += w[t] * mel[2 * r + ki][2 * j + kj];  // mel row tm_0 + 2r + ki, col 2j + kj - 1 (+1 pad)
            }
            s = s > 0.f ? s : 0.f;
        }
        c0[r][jj][c] = s;
    }
    __syncthreads();
    // depthwise conv1 (+ mask): out(t2, j2) = b + sum w * c0(2 t2 + ki - 1, 2 j2 + kj - 1)
    for (int i = threadIdx.x; i < kT2 * 32 * kC; i += blockDim.x) {
        const int c = i % kC, j2 = (i / kC) % 32, r2 = i / (kC * 32);
        const int t2 = t2_0 + r2;
        if (t2 >= F2) continue;
        float s = 0.f;
        if (t2 < v2) {
            const float* w = p.w2 + (cg + c) * 9;
            s = p.b2[cg + c];
#pragma unroll
            for (int ki = 0; ki < 3; ++ki) {
                const int t1 = 2 * t2 + ki - 1;
                if (t1 < 0 || t1 >= F1) continue;
#pragma unroll
                for (int kj = 0; kj < 3; ++kj) {
                    const int j1 = 2 * j2 + kj - 1;
                    if (j1 < 0 || j1 >= 64) continue;
                    s += w[ki * 3 + kj] * c0[t1 - t1_0][j1 + 1][c];
                }
            }
        }
        p.x2[(static_cast<size_t>(p.x2_off[u] + t2) * 32 + j2) * 256 + cg + c] = __float2half_rn(s);
    }
}

// Second depthwise conv (+ bias, + mask): x3 [t2][32][256] -> x4 [t3][16][256].
__global__ void __launch_bounds__(256) k_sub_dw2(SubParams p) {
    const int row = blockIdx.x;  // global t3 row
    int lo = 0, hi = p.n_utt;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (p.x4_off[mid] <= row) lo = mid; else hi = mid;
    }
    const int u = lo;
    const int t3 = row - p.x4_off[u];
    const int F = p.mel_off[u + 1] - p.mel_off[u];
    const int F2 = conv_len_d(conv_len_d(F));
    const int nvalid = p.n_valid[u];
    const int v3 = conv_len_d(conv_len_d(conv_len_d(nvalid > 1 ? nvalid : 1)));
    const __half* x3 = p.x3 + static_cast<size_t>(p.x2_off[u]) * 32 * 256;
    for (int i = threadIdx.x; i < 16 * 256; i += blockDim.x) {
        const int c = i % 256, j3 = i / 256;
        float s = 0.f;
        if (t3 < v3) {
            s = p.b5[c];
#pragma unroll
            for (int ki = 0; ki < 3; ++ki) {
                const int t2 = 2 * t3 + ki - 1;
                if (t2 < 0 || t2 >= F2) continue;
#pragma unroll
                for (int kj = 0; kj < 3; ++kj) {
                    const int j2 = 2 * j3 + kj - 1;
                    if (j2 < 0 || j2 >= 32) continue;
                    s += p.w5[c * 9 + ki * 3 + kj] * __half2float(x3[(static_cast<size_t>(t2) * 32 + j2) * 256 + c]);
                }
            }
        }
        p.x4[(static_cast<size_t>(row) * 16 + j3) * 256 + c] = __float2half_rn(s);
    }
}

// [T][16][256] f16 (freq, channel) -> [T][4096] f32 in the reference's
// (channel, freq) order, for the subsampling parity entry point.
__global__ void k_sub_to_ref(const __half* src, float* dst, int rows) {
    const int t = blockIdx.x;
    if (t >= rows) return;
    for (int i = threadIdx.x; i < 4096; i += blockDim.x) {
        const int c = i / 16, m = i % 16;
        dst[static_cast<size_t>(t) * 4096 + i] = __half2float(src[(static_cast<size_t>(t) * 16 + m) * 256 + c]);
    }
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error(what, e);
}

}  // namespace

int launch_mel(const MelParams& p, int n_frames, cudaStream_t st) {
    if (n_frames <= 0) return 0;
    k_mel_frames<<<n_frames, 256, 0, st>>>(p);
    const int rc = check_launch("k_mel_frames");
    if (rc) return rc;
    k_mel_norm<<<p.n_utt, kMel, 0, st>>>(p);
    return check_launch("k_mel_norm");
}

int launch_sub_conv0_dw1(const SubParams& p, int n_work, cudaStream_t st) {
    if (n_work <= 0) return 0;
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(k_sub_conv0_dw1, cudaFuncAttributeMaxDynamicSharedMemorySize, kSubSmem);
        if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(k_sub_conv0_dw1)", e);
        attr_done = true;
    }
    k_sub_conv0_dw1<<<n_work, 256, kSubSmem, st>>>(p);
    return check_launch("k_sub_conv0_dw1");
}

int launch_sub_dw2(const SubParams& p, int rows, cudaStream_t st) {
    if (rows <= 0) return 0;
    k_sub_dw2<<<rows, 256, 0, st>>>(p);
    return check_launch("k_sub_dw2");
}

int launch_sub_to_ref(const __half* src, float* dst, int rows, cudaStream_t st) {
    if (rows <= 0) return 0;
    k_sub_to_ref<<<rows, 256, 0, st>>>(src, dst, rows);
    return check_launch("k_sub_to_ref");
}

int sub_work_rows() { return kT2; }
int sub_work_channels() { return kC; }

}  // namespace b3
