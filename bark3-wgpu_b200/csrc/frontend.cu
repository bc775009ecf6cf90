// frontend.cu — log-mel features and conv subsampling on the GPU (the
// reference computes the mel on the CPU, src/mel.rs:41-138, and subsamples
// on the CPU or with WGSL, src/sub.rs:107-300, src/sub_gpu.rs).
//
// Mel: one warp per frame: pre-emphasis (0.97), 512-point centred frame with
// the symmetric Hann(400) window, a real 512-point FFT as a 256-point complex
// FFT in shared memory (f32), power of the 257 bins, 128 slaney mel bins
// (sparse rows), log(x + 2^-24).  Normalisation: one CTA per (utterance, 32
// mel bins), mean and sample std over the valid frames (frames >= len/160
// zeroed).
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

// One frame per warp, 8 frames per CTA.  The 512 real samples x[n] are
// packed as 256 complex values z[m] = x[2m] + i x[2m+1]; a 256-point radix-2
// FFT of z in shared memory (eight stages, __syncwarp between them) gives the
// 512-point spectrum by the standard real-input split
//   X[k] = (Z[k] + conj Z[256-k]) / 2 + W512^k (Z[k] - conj Z[256-k]) / 2i.
constexpr int kMelWarps = 8;

// Shared-memory slot of FFT point i (an injective map of 0..255 into
// 0..256): with it the bit-reversed scatter, every butterfly stage pair and
// the forward half of the real-input split touch 32 distinct banks per warp
// access (the split's mirrored half 2-way), where plain indices gave up to
// 8-way conflicts (the scatter) and 4-way (the first two stage pairs).
__device__ __forceinline__ int fft_slot(int i) { return (i ^ ((i >> 2) & 31)) + (i >> 7); }

// The filters' packed nonzero spans are staged in shared memory when they
// fit (504 weights for the 128-filter slaney bank); otherwise each lane
// reads its span from the packed global copy.
constexpr int kMelFbSmem = 1024;

// Sample s of an utterance whose first `lead` samples are zeros (the leading
// silence, never stored) followed by x[0 .. len - lead): pre-emphasised and
// windowed.
__device__ __forceinline__ float mel_sample(const float* x, int64_t len, int lead, int64_t s, float w) {
    if (s < 0 || s >= len) return 0.f;
    const float cur = s >= lead ? __ldg(x + (s - lead)) : 0.f;
    const float prev = s - 1 >= lead ? __ldg(x + (s - 1 - lead)) : 0.f;
    return (s == 0 ? cur : cur - 0.97f * prev) * w;
}

__global__ void __launch_bounds__(256, 7) k_mel_frames(MelParams p, int f0, int f1) {
    __shared__ float zre[kMelWarps][257], zim[kMelWarps][257], pwr[kMelWarps][260];
    __shared__ float2 tw[256];
    __shared__ float fbs[kMelFbSmem];
    tw[threadIdx.x] = p.twiddle[threadIdx.x];
    const bool fb_smem = p.fb_total <= kMelFbSmem;
    if (fb_smem)
        for (int i = threadIdx.x; i < p.fb_total; i += blockDim.x) fbs[i] = __ldg(p.fb_pack + i);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int f = f0 + blockIdx.x * kMelWarps + warp;
    if (f >= f1) return;
    int lo = 0, hi = p.n_utt;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (p.frame_off[mid] <= f) lo = mid; else hi = mid;
    }
    const int u = lo;
    const int t = f - p.frame_off[u];
    const float* x = p.wave + p.wave_off[u];
    const int64_t len = p.wave_off[u + 1] - p.wave_off[u] + p.lead;
    const int64_t start = static_cast<int64_t>(t) * kHop - kNfft / 2;
    float* re = zre[warp];
    float* im = zim[warp];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const int m = lane + 32 * q;
        const int r = __brev(m) >> 24;  // 8-bit reversal
        re[fft_slot(r)] = mel_sample(x, len, p.lead, start + 2 * m, __ldg(p.window + 2 * m));
        im[fft_slot(r)] = mel_sample(x, len, p.lead, start + 2 * m + 1, __ldg(p.window + 2 * m + 1));
    }
    __syncwarp();
    // radix-2 stages taken two at a time: the 4 points i0 + {0, h, 2h, 3h}
    // of a group of 4h pass through stage lh (butterflies (i0, i1), (i2, i3))
    // and stage lh + 1 ((i0, i2), (i1, i3)) in registers, which halves the
    // shared-memory traffic; the arithmetic is that of the stages one by one
    auto bfly = [](float& ar, float& ai, float& br, float& bi, float2 w) {
        const float vr = br * w.x - bi * w.y;
        const float vi = br * w.y + bi * w.x;
        const float ur = ar, ui = ai;
        ar = ur + vr;
        ai = ui + vi;
        br = ur - vr;
        bi = ui - vi;
    };
#pragma unroll
    for (int lh = 0; lh < 8; lh += 2) {
        const int h = 1 << lh;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int b = lane + 32 * q;   // group-of-4 index, 0..63
            const int k = b & (h - 1);
            const int j0 = ((b - k) << 2) + k;
            const int i0 = fft_slot(j0), i1 = fft_slot(j0 + h), i2 = fft_slot(j0 + 2 * h), i3 = fft_slot(j0 + 3 * h);
            float r0 = re[i0], m0 = im[i0], r1 = re[i1], m1 = im[i1];
            float r2 = re[i2], m2 = im[i2], r3 = re[i3], m3 = im[i3];
            const float2 wa = tw[k << (8 - lh)];   // W256^(k * 128 / h) = W512^(k * 256 / h)
            bfly(r0, m0, r1, m1, wa);
            bfly(r2, m2, r3, m3, wa);
            bfly(r0, m0, r2, m2, tw[k << (7 - lh)]);
            bfly(r1, m1, r3, m3, tw[(k + h) << (7 - lh)]);
            re[i0] = r0;
            im[i0] = m0;
            re[i1] = r1;
            im[i1] = m1;
            re[i2] = r2;
            im[i2] = m2;
            re[i3] = r3;
            im[i3] = m3;
        }
        __syncwarp();
    }
    float* pw = pwr[warp];
#pragma unroll
    for (int q = 0; q < 9; ++q) {
        const int k = lane + 32 * q;
        if (k <= 256) {
            const int ka = k & 255, kb = (256 - k) & 255;
            const int sa = fft_slot(ka), sb = fft_slot(kb);
            const float ar = re[sa], ai = im[sa], br = re[sb], bi = -im[sb];
            const float er = 0.5f * (ar + br), ei = 0.5f * (ai + bi);
            const float orr = 0.5f * (ai - bi), oi = -0.5f * (ar - br);
            const float2 w = k < 256 ? tw[k] : make_float2(-1.f, 0.f);
            const float xr = er + (w.x * orr - w.y * oi);
            const float xi = ei + (w.x * oi + w.y * orr);
            pw[k] = xr * xr + xi * xi;
        }
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int m = lane + 32 * q;
        const int k0 = __ldg(p.fb_lo + m), k1 = __ldg(p.fb_hi + m);
        const int o = __ldg(p.fb_off + m);
        float s = 0.f;
        if (fb_smem) {
            const float* wv = fbs + o - k0;
            for (int k = k0; k < k1; ++k) s += wv[k] * pw[k];
        } else {
            const float* wv = p.fb_pack + o - k0;
            for (int k = k0; k < k1; ++k) s += __ldg(wv + k) * pw[k];
        }
        p.mel[static_cast<size_t>(f) * kMel + m] = logf(s + 5.9604645e-08f);
    }
}

// Per-utterance normalisation over the valid frames (src/mel.rs:103-136):
// one CTA per (utterance, 32 mel bins); kNormLanes frame lanes per bin
// (1024 threads, so a CTA keeps 32 rows of loads in flight per pass),
// reduced in shared memory; two passes (mean, then squared deviations) as
// the reference.  The frame loops are unrolled 16 deep so each thread keeps
// 16 loads in flight (a launch lasts as long as its longest utterance's CTA,
// which walks thousands of frames); each running sum still adds in frame
// order.
constexpr int kNormLanes = 32;
__global__ void __launch_bounds__(32 * kNormLanes) k_mel_norm(MelParams p, int u0) {
    __shared__ float red[kNormLanes][33];
    __shared__ float stat[32];
    const int u = u0 + blockIdx.x;
    const int b = threadIdx.x & 31, fl = threadIdx.x >> 5;
    const int m = blockIdx.y * 32 + b;
    const int f0 = p.frame_off[u];
    const int nf = p.frame_off[u + 1] - f0;
    const int nvalid = static_cast<int>((p.wave_off[u + 1] - p.wave_off[u] + p.lead) / kHop);
    const int nv = nvalid > 1 ? nvalid : 1;
    float* mel = p.mel + static_cast<size_t>(f0) * kMel + m;
    float s = 0.f;
#pragma unroll 16
    for (int t = fl; t < nvalid; t += kNormLanes) s += mel[static_cast<size_t>(t) * kMel];
    red[fl][b] = s;
    __syncthreads();
    if (fl == 0) {
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < kNormLanes; ++i) tot += red[i][b];
        stat[b] = tot / static_cast<float>(nv);
    }
    __syncthreads();
    const float mean = stat[b];
    float q = 0.f;
#pragma unroll 16
    for (int t = fl; t < nvalid; t += kNormLanes) {
        const float d = mel[static_cast<size_t>(t) * kMel] - mean;
        q += d * d;
    }
    red[fl][b] = q;
    __syncthreads();
    if (fl == 0) {
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < kNormLanes; ++i) tot += red[i][b];
        stat[b] = sqrtf(tot / static_cast<float>(nv - 1 > 1 ? nv - 1 : 1)) + 1e-5f;
    }
    __syncthreads();
    const float den = stat[b];
#pragma unroll 16
    for (int t = fl; t < nf; t += kNormLanes) {
        float& v = mel[static_cast<size_t>(t) * kMel];
        v = t < nvalid ? (v - mean) / den : 0.f;
    }
}

// conv0 + ReLU + mask, then depthwise conv1 + mask, for kT2 output rows (t2)
// x all 32 freq columns x kC channels.  Shared memory holds the mel rows the
// tile needs with even and odd columns split (conv0's stride-2 taps are then
// unit-stride across lanes) and the conv0 output tile [kT1][kC][65] (column
// -1 is the zero pad; the odd row stride keeps the channel-per-lane reads of
// the depthwise conv free of bank conflicts).  conv0: a warp owns 8 channels
// (4 pairs, one packed f32x2 FMA per pair and tap) with their 9 taps in
// registers over 32 of the 64 columns, so each mel value loaded feeds 8
// channels; conv1: a lane owns a channel, warps walk (row, 16-column run) with
// a sliding window, two output columns per packed FMA.  Every output keeps the
// scalar accumulation order (bias, then taps row by row, left to right).
constexpr int kT2 = 4;
constexpr int kC = 32;
constexpr int kT1 = 2 * kT2 + 1;   // conv0 rows needed (9)
constexpr int kTm = 2 * kT1 + 1;   // mel rows needed (19)
constexpr int kMelS = 130;         // [0, 64]: even cols 0..126 (+ zero); [65, 129]: odd cols -1..127
constexpr int kC0S = 65;           // conv0 row of one channel: cols -1..63
constexpr int kC0Row = kC * kC0S;  // one conv0 row of all kC channels
constexpr int kSubSmem = (kTm * kMelS + kT1 * kC0Row) * 4;

// Persistent: CTA b walks work items w0 + b, w0 + b + gridDim.x, ... up to
// w1.  Items are (utterance, t2 row block, channel group) with the group
// fastest and a multiple of 8 items per utterance, and the grid is a
// multiple of 8, so a CTA keeps one channel group: its conv0 and conv1 taps
// stay in registers for the whole launch, and the next item's mel rows are
// loaded into registers while the current item computes.  An item's work
// entry holds every table value it needs (no dependent reads); the entry of
// the item after next is read while the current one computes, so the next
// item's mel addresses are known without waiting.
__global__ void __launch_bounds__(256, 2) k_sub_conv0_dw1(SubParams p, int w0, int w1) {
    extern __shared__ float sub_smem[];
    float* mel = sub_smem;                 // [kTm][kMelS]
    float* c0 = sub_smem + kTm * kMelS;    // [kT1][kC][kC0S]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int e = w0 + blockIdx.x;
    if (e >= w1) return;
    const int cg = p.work[2 * e + 1].y * kC;
    // conv0 taps: warp w owns channels 8 (w & 3) .. +8 as 4 channel pairs (one
    // packed f32x2 FMA per pair and tap) over columns 32 (w >> 2) + lane
    const int cq = (warp & 3) * 8;
    const int j = (warp >> 2) * 32 + lane;
    float2 w[4][9], bias[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        bias[q] = make_float2(__ldg(p.b0 + cg + cq + 2 * q), __ldg(p.b0 + cg + cq + 2 * q + 1));
#pragma unroll
        for (int t = 0; t < 9; ++t)
            w[q][t] = make_float2(__ldg(p.w0 + (cg + cq + 2 * q) * 9 + t), __ldg(p.w0 + (cg + cq + 2 * q + 1) * 9 + t));
    }
    // conv1 taps: a lane per channel
    float wd[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) wd[t] = __ldg(p.w2 + (cg + lane) * 9 + t);
    const float bias2 = __ldg(p.b2 + cg + lane);
    // padding that no item overwrites: mel column slots 64 (even col 128,
    // never read) and 65 (col -1); conv0 column -1
    if (threadIdx.x < kTm) {
        mel[threadIdx.x * kMelS + 64] = 0.f;
        mel[threadIdx.x * kMelS + 65] = 0.f;
    }
    for (int i = threadIdx.x; i < kT1 * kC; i += blockDim.x) c0[i * kC0S] = 0.f;
    // an item's mel rows, 16-byte loads of columns 4 c .. 4 c + 3 (three per thread)
    constexpr int kLoads = (kTm * (kMel / 4) + 255) / 256;
    float4 pre[kLoads];
    // an item's entry: a = (first mel row, mel frames, valid frames, first
    // t2 row), b = (first x2 row, channel group, 0, 0)
    auto fetch = [&](const int4& a) {
        const int F = a.y;
        const int tm_0 = 2 * (2 * a.w - 1) - 1;
        const float* melu = p.mel + static_cast<size_t>(a.x) * kMel;
#pragma unroll
        for (int k = 0; k < kLoads; ++k) {
            const int i = threadIdx.x + 256 * k;
            const int r = i >> 5, c = i & 31;
            const int tm = tm_0 + r;
            pre[k] = (i < kTm * (kMel / 4) && tm >= 0 && tm < F)
                         ? __ldg(reinterpret_cast<const float4*>(melu + static_cast<size_t>(tm) * kMel) + c)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    // the even pair of a load goes to even slots 2 c, 2 c + 1, the odd pair
    // to odd slots 66 + 2 c, 67 + 2 c
    auto park = [&]() {
#pragma unroll
        for (int k = 0; k < kLoads; ++k) {
            const int i = threadIdx.x + 256 * k;
            if (i < kTm * (kMel / 4)) {
                const int r = i >> 5, c = i & 31;
                *reinterpret_cast<float2*>(mel + r * kMelS + 2 * c) = make_float2(pre[k].x, pre[k].z);
                *reinterpret_cast<float2*>(mel + r * kMelS + 66 + 2 * c) = make_float2(pre[k].y, pre[k].w);
            }
        }
    };
    const int G = static_cast<int>(gridDim.x);
    const int4 zero4 = make_int4(0, 0, 0, 0);
    int4 ca = __ldg(p.work + 2 * e);                            // this item
    int4 na = e + G < w1 ? __ldg(p.work + 2 * (e + G)) : zero4;  // the next
    fetch(ca);
    park();
    for (; e < w1; e += G) {
        const int t2_0 = ca.w;
        const int F = ca.y;
        const int F1 = conv_len_d(F), F2 = conv_len_d(F1);
        const int nvalid = ca.z;
        const int v1 = conv_len_d(nvalid > 1 ? nvalid : 1);
        const int v2 = conv_len_d(v1);
        const int t1_0 = 2 * t2_0 - 1;      // first conv0 row
        __syncthreads();                     // this item's mel rows are parked
        const int next = e + G;
        if (next < w1) fetch(na);            // lands while this item computes
        // the item after next: its entry lands meanwhile; this item's x2
        // row is needed only by the depthwise conv, after conv0
        const int4 fa = next + G < w1 ? __ldg(p.work + 2 * (next + G)) : zero4;
        const int x2row = __ldg(&p.work[2 * e + 1].x);
        for (int r = 0; r < kT1; ++r) {
            const int t1 = t1_0 + r;
            const bool live = t1 >= 0 && t1 < F1 && t1 < v1;
            const float* m0 = mel + 2 * r * kMelS;   // mel rows 2 t1 - 1 + ki
            float* out = c0 + (r * kC + cq) * kC0S + 1 + j;
            float2 acc[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[q] = bias[q];
            if (live) {
#pragma unroll
                for (int ki = 0; ki < 3; ++ki) {
                    const float* row = m0 + ki * kMelS;
                    const float a = row[65 + j], b = row[j], c = row[66 + j];  // cols 2j-1, 2j, 2j+1
                    const float2 a2 = make_float2(a, a), b2 = make_float2(b, b), c2 = make_float2(c, c);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        acc[q] = __ffma2_rn(w[q][ki * 3], a2, acc[q]);
                        acc[q] = __ffma2_rn(w[q][ki * 3 + 1], b2, acc[q]);
                        acc[q] = __ffma2_rn(w[q][ki * 3 + 2], c2, acc[q]);
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                out[(2 * q) * kC0S] = live ? fmaxf(acc[q].x, 0.f) : 0.f;
                out[(2 * q + 1) * kC0S] = live ? fmaxf(acc[q].y, 0.f) : 0.f;
            }
        }
        __syncthreads();
        {
            // depthwise conv: a lane per channel, warps walk (row, 16-column run)
            // two output columns at a time as one packed f32x2 FMA per tap
            const int r2 = warp >> 1, jb = (warp & 1) * 16;
            const int t2 = t2_0 + r2;
            if (t2 < F2) {
                const bool live = t2 < v2;
                // conv0 local rows 2 r2 + ki hold t1 = 2 t2 - 1 + ki; index 1 + col
                const float* base = c0 + (2 * r2 * kC + lane) * kC0S;
                __half* out = p.x2 + static_cast<size_t>(x2row + t2) * 32 * 256 + cg + lane;
                float prev[3];
#pragma unroll
                for (int ki = 0; ki < 3; ++ki) prev[ki] = base[ki * kC0Row + 2 * jb];   // col 2 jb - 1
#pragma unroll 2
                for (int jj = 0; jj < 16; jj += 2) {
                    const int j2 = jb + jj;   // outputs j2 (cols 2j2-1..2j2+1) and j2+1 (cols 2j2+1..2j2+3)
                    float2 s = make_float2(bias2, bias2);
#pragma unroll
                    for (int ki = 0; ki < 3; ++ki) {
                        const float* row = base + ki * kC0Row;
                        const float x0 = row[2 * j2 + 1], x1 = row[2 * j2 + 2], x2 = row[2 * j2 + 3], x3 = row[2 * j2 + 4];
                        s = __ffma2_rn(make_float2(wd[ki * 3], wd[ki * 3]), make_float2(prev[ki], x1), s);
                        s = __ffma2_rn(make_float2(wd[ki * 3 + 1], wd[ki * 3 + 1]), make_float2(x0, x2), s);
                        s = __ffma2_rn(make_float2(wd[ki * 3 + 2], wd[ki * 3 + 2]), make_float2(x1, x3), s);
                        prev[ki] = x3;
                    }
                    out[j2 * 256] = __float2half_rn(live ? s.x : 0.f);
                    out[(j2 + 1) * 256] = __float2half_rn(live ? s.y : 0.f);
                }
            }
        }
        __syncthreads();                     // every read of this item's mel rows and conv0 tile done
        if (next < w1) park();
        ca = na;
        na = fa;
    }
}

// Second depthwise conv (+ bias, + mask): x3 [t2][32][256] -> x4 [t3][16][256].
// Persistent: 64 threads per x4 row, 4 rows per CTA pass.  A thread owns 4
// channels, whose taps and bias stay in registers for the whole launch, and
// walks the row's 16 output columns left to right, loading each input column
// (3 rows x 4 channels, 8-byte loads) once and carrying the shared column to
// the next output; two channels per packed f32x2 FMA.  A row's table values
// (first x2 row of its utterance, depthwise-1 rows, valid x4 rows, row within
// the utterance) are one int4, read a pass ahead.  Every output keeps the
// scalar accumulation order (bias, then taps row by row, left to right).
constexpr int kDw2Rows = 4;
__global__ void __launch_bounds__(64 * kDw2Rows) k_sub_dw2(SubParams p, int r0, int r1) {
    const int c0 = (threadIdx.x & 63) * 4;
    float2 w[9][2], bias[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int ca = c0 + 2 * q;
        bias[q] = make_float2(__ldg(p.b5 + ca), __ldg(p.b5 + ca + 1));
#pragma unroll
        for (int t = 0; t < 9; ++t) w[t][q] = make_float2(__ldg(p.w5 + ca * 9 + t), __ldg(p.w5 + (ca + 1) * 9 + t));
    }
    const int stride = static_cast<int>(gridDim.x) * kDw2Rows;
    const int4 zero4 = make_int4(0, 0, 0, 0);
    int row = r0 + static_cast<int>(blockIdx.x) * kDw2Rows + (threadIdx.x >> 6);   // global x4 row
    int4 nm = row < r1 ? __ldg(p.rows3 + row) : zero4;
    for (; row < r1; row += stride) {
        const int4 m = nm;
        if (row + stride < r1) nm = __ldg(p.rows3 + row + stride);   // lands while this row computes
        const int F2 = m.y, t3 = m.w;
        const bool live = t3 < m.z;
        const __half* x3 = p.x3 + static_cast<size_t>(m.x) * 32 * 256;
        bool rok[3];
#pragma unroll
        for (int ki = 0; ki < 3; ++ki) {
            const int t2 = 2 * t3 + ki - 1;
            rok[ki] = t2 >= 0 && t2 < F2;
        }
        // column j2 of the 3 input rows: channels (c0, c0 + 1) and (c0 + 2, c0 + 3)
        auto col = [&](int j2, float2 (&v)[3][2]) {
#pragma unroll
            for (int ki = 0; ki < 3; ++ki) {
                uint2 raw = make_uint2(0u, 0u);
                if (rok[ki]) {
                    const int t2 = 2 * t3 + ki - 1;
                    raw = __ldg(reinterpret_cast<const uint2*>(x3 + (static_cast<size_t>(t2) * 32 + j2) * 256 + c0));
                }
                v[ki][0] = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                v[ki][1] = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
            }
        };
        float2 cl[3][2];   // column 2 j3 - 1 (the previous output's right column)
#pragma unroll
        for (int ki = 0; ki < 3; ++ki) cl[ki][0] = cl[ki][1] = make_float2(0.f, 0.f);
        __half* out = p.x4 + static_cast<size_t>(row) * 16 * 256 + c0;
#pragma unroll 2
        for (int j3 = 0; j3 < 16; ++j3) {
            float2 cm[3][2], cr[3][2];
            col(2 * j3, cm);
            col(2 * j3 + 1, cr);
            float2 s[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            if (live) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    s[q] = bias[q];
#pragma unroll
                    for (int ki = 0; ki < 3; ++ki) {
                        if (!rok[ki]) continue;
                        if (j3 > 0) s[q] = __ffma2_rn(w[ki * 3][q], cl[ki][q], s[q]);   // column 2 j3 - 1 exists
                        s[q] = __ffma2_rn(w[ki * 3 + 1][q], cm[ki][q], s[q]);
                        s[q] = __ffma2_rn(w[ki * 3 + 2][q], cr[ki][q], s[q]);
                    }
                }
            }
            __half2 h0 = __floats2half2_rn(s[0].x, s[0].y), h1 = __floats2half2_rn(s[1].x, s[1].y);
            *reinterpret_cast<uint2*>(out + j3 * 256) =
                make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
#pragma unroll
            for (int ki = 0; ki < 3; ++ki) {
                cl[ki][0] = cr[ki][0];
                cl[ki][1] = cr[ki][1];
            }
        }
    }
}

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

int launch_mel(const MelParams& p, int f0, int f1, int u0, int u1, cudaStream_t st) {
    if (f1 <= f0 || u1 <= u0) return 0;
    k_mel_frames<<<(f1 - f0 + kMelWarps - 1) / kMelWarps, 256, 0, st>>>(p, f0, f1);
    const int rc = check_launch("k_mel_frames");
    if (rc) return rc;
    k_mel_norm<<<dim3(u1 - u0, kMel / 32), 32 * kNormLanes, 0, st>>>(p, u0);
    return check_launch("k_mel_norm");
}

int launch_sub_conv0_dw1(const SubParams& p, int w0, int w1, cudaStream_t st) {
    const int n_work = w1 - w0;
    if (n_work <= 0) return 0;
    static PerDeviceOnce attr;
    const int rc = set_smem_limit_once(attr, k_sub_conv0_dw1, kSubSmem, "cudaFuncSetAttribute(k_sub_conv0_dw1)");
    if (rc) return rc;
    // persistent: two CTAs per SM, a multiple of 8 so each keeps one channel group
    const int per_sm = 2 * device_sms() / 8 * 8;
    const int grid = n_work < per_sm ? n_work : per_sm;
    k_sub_conv0_dw1<<<grid, 256, kSubSmem, st>>>(p, w0, w1);
    return check_launch("k_sub_conv0_dw1");
}

int launch_sub_dw2(const SubParams& p, int r0, int r1, cudaStream_t st) {
    if (r1 <= r0) return 0;
    // persistent: as many CTAs as are resident at once
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_sub_dw2, 64 * kDw2Rows, 0) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const int passes = (r1 - r0 + kDw2Rows - 1) / kDw2Rows;
    const int grid = passes < per_sm * device_sms() ? passes : per_sm * device_sms();
    k_sub_dw2<<<grid, 64 * kDw2Rows, 0, st>>>(p, r0, r1);
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
