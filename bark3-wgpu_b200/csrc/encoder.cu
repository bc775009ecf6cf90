// encoder.cu — context, weight store, launch sequence and the C ABI.
//
// The per-block launch sequence restates CpuLayer::forward
// (src/cpu/layer.rs:157-327) / Encoder::encode_pre (src/encoder.rs:2005-2651)
// with the element-wise passes fused into the GEMM epilogues:
//
//   LN1 -> ff1a[SiLU] -> ff1b[x += 0.5 acc]
//   LN2 -> qkv[+bias_u / +bias_v split] -> rel-pos attention -> o[x += acc]
//   LN3 -> pw1[GLU] -> dwconv+BN+SiLU -> pw2[x += acc]
//   LN4 -> ff2a[SiLU] -> ff2b[x += 0.5 acc]
//   norm_out (fused with the next block's LN1)
//
// Layout in HBM (rows = frames of all utterances, concatenated):
//   x     [M][1024] f32   residual stream (stays f32 like the reference)
//   a16   [M][1024] f16   GEMM input: LN output / attention output / conv output
//   h16   [M][4096] f16   FFN hidden after SiLU
//   qkv16 [M][4096] f16   q+bias_u | q+bias_v | k | v
//   g16   [M][1024] f16   GLU output (depthwise conv input)
//   sub16 [M][4096] f16   encoder input
//   pos16 [2*Tcap-1][1024] f16 positional table, R16 [2*Tmax-1][1024] f16
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <cmath>
#include <map>
#include <string>
#include <vector>
#include <algorithm>

#include "b3_internal.h"
#include "b3_kernels.h"

// ───────────────────────────── errors ─────────────────────────────

namespace b3 {
namespace {
thread_local char g_last_error[512] = "";
}

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int set_cuda_error(const char* what, cudaError_t e) {
    return set_error(B3_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

void clear_error() { g_last_error[0] = 0; }

int device_sms() {
    static std::atomic<int> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

}  // namespace b3

using namespace b3;

#define B3_TRY(expr)                \
    do {                            \
        int _rc = (expr);           \
        if (_rc) return _rc;        \
    } while (0)

#define B3_CUDA(expr)                                          \
    do {                                                       \
        cudaError_t _e = (expr);                               \
        if (_e != cudaSuccess) return set_cuda_error(#expr, _e); \
    } while (0)

namespace {

constexpr int kHidden = 1024;
constexpr int kFfn = 4096;
constexpr int kSubIn = 4096;
constexpr int kProj = 640;

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    int ensure(size_t need) {
        if (need <= bytes) return 0;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        cudaError_t e = cudaMalloc(&p, need);
        if (e != cudaSuccess) {
            p = nullptr;
            return set_error(B3_ENOMEM, "cudaMalloc(%zu bytes): %s", need, cudaGetErrorString(e));
        }
        bytes = need;
        return 0;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

// One linear layer's weight on the device.
struct Linear {
    bool present = false;
    bool lut = false;
    int N = 0, K = 0;
    DevBuf w;      // codes [N][K/2] or f16 [N][K]
    DevBuf lut16;  // [N][16] f16
    CUtensorMap map_b;
};

struct Layer {
    Linear qkv, relk, o, ff1a, ff1b, ff2a, ff2b, pw1, pw2;
    DevBuf params;  // f32: dw_t[9][1024] | bn_a | bn_b | ln_w[5] | ln_b[5] | bu | bv
    float* dw_t() const { return params.as<float>(); }
    float* bn_a() const { return params.as<float>() + 9 * kHidden; }
    float* bn_b() const { return params.as<float>() + 10 * kHidden; }
    float* ln_w(int i) const { return params.as<float>() + (11 + i) * kHidden; }
    float* ln_b(int i) const { return params.as<float>() + (16 + i) * kHidden; }
    float* bu() const { return params.as<float>() + 21 * kHidden; }
    float* bv() const { return params.as<float>() + 22 * kHidden; }
    static constexpr size_t kParamFloats = 23 * kHidden;
};

// A tensor as pushed through the ABI, kept on the host until b3_finalize.
struct Staged {
    bool lowbit = false;
    std::vector<int64_t> shape;
    std::vector<float> f32;        // dense values, widened exactly
    std::vector<uint16_t> f16;     // dense values rounded to f16 (RNE)
    std::vector<uint8_t> codes;    // lowbit: [rows][cols/2]
    std::vector<uint16_t> lut16;   // lowbit: [rows][16]
    int rows = 0, cols = 0;
};

struct Plan {
    std::vector<int32_t> cu;
    int M = 0, tmax = 0, n_work = 0;
};

// Frame bookkeeping of a front-end batch: frame / depthwise-1 / encoder row
// offsets per utterance and the subsampling CTA work list.
// Zero samples the audio front end puts before every utterance: the
// reference's 0.25 s of leading silence at 16 kHz (src/transcription.rs:48-52).
constexpr int kLeadSamples = 4000;

struct FeShape {
    std::vector<int32_t> foff, nvalid, x2off, x4off;
    std::vector<int32_t> woff;   // first conv work item of each utterance (n + 1)
    std::vector<int4> work;
    std::vector<int4> rows3;     // per encoder frame: (first x2 row, depthwise-1 rows, valid frames, frame)
};

// Per-kernel-class CUDA-event timing (the analogue of the reference's
// BARK3_ENC_PROFILE timestamp queries, src/encoder/prof.rs:1-121).  Launch
// counts are always kept; events are recorded only while enabled.
struct ProfRec {
    int kind;
    int ev;
    double flops, bytes;
};

struct Prof {
    bool on = false;
    std::vector<cudaEvent_t> pool;
    int next = 0;
    std::vector<ProfRec> recs;
    int64_t launches[B3_K_COUNT] = {};
    double ms[B3_K_COUNT] = {}, flops[B3_K_COUNT] = {}, bytes[B3_K_COUNT] = {};
    int64_t timed[B3_K_COUNT] = {};
};

}  // namespace

struct b3_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::map<std::string, Staged> staged;
    bool finalized = false;
    int n_layers = 0;
    Linear sub_w, proj_w;
    DevBuf sub_b, proj_b;
    std::vector<Layer> layers;
    DevBuf inv_freq;  // [512] f32
    int tcap = 0;     // positional table capacity (frames)
    DevBuf pos16;
    // activation arena
    int mcap = 0;
    DevBuf x, a16, h16, qkv16, g16, sub16, R16;
    DevBuf cu_d, work_d, seg_d;
    DevBuf io_in, io_out;   // device staging for host-pointer calls
    DevBuf scratch16;       // f16 copy of A for the single-linear entry points
    Plan plan;
    uint64_t plan_gen = 0;  // bumped whenever a plan, the arena or the weights change
    // A repeated small-batch encode (same rows, buffers and block count)
    // replays a CUDA graph of its launches: the 24 blocks are ~350 launches,
    // which at a few hundred rows cost more than the kernels.
    struct EncGraph {
        cudaGraphExec_t exec = nullptr;
        const float* sub = nullptr;
        float* out = nullptr;
        int M = 0, layers = -1;
        uint64_t gen = 0;
        bool seen = false;     // the key ran eagerly once (first-call set-up done)
        bool no_graph = false; // capture failed for this key: stay eager
        void reset() {
            if (exec) cudaGraphExecDestroy(exec);
            exec = nullptr;
            seen = no_graph = false;
        }
    } enc_graph;
    Prof prof;
    // wall-time bound of the decoder's grid-barrier waits (b3_set_wait_limit)
    uint64_t grid_wait_ns = kDefaultWaitNs;
    // decode every batch with the split-K persistent kernel (b3_set_decoder)
    bool dec_split_k_only = false;
    // greedy TDT decoder (optional: built when its tensors are loaded)
    struct Decoder {
        bool present = false;
        int vocab = 0, npad = 0;
        DevBuf e0;                             // [vocab][2560] f32: W_ih0 . emb + b_ih0 + b_hh0
        Linear lstm[2];                        // layer 0 [2560][1280] = W_hh | W_hh; layer 1 [2560][2560] = W_ih | W_ih | W_hh | W_hh
        Linear proj;                           // [640][1280]  = W_p | W_p
        Linear head;                           // [npad][1280] = W_head | W_head (zero rows past vocab+5)
        DevBuf bias;                           // f32: lstm0 [2560] (unused) | lstm1 [2560] | proj [640] | head [npad]
        // lock-step state (DecState), split-K parts, outputs, barrier words
        DevBuf a0, a1, ap, aj, gates, cstate, dec, scores, ints, tokens, rows, sync, pooler;
        // weight-stationary decoder (DecWs): 128-row weight tiles, their biases, argmax keys
        int ws_ht = 0;
        DevBuf ws_w, ws_bias, ws_keys;
        CUtensorMap ws_wmap;
    } dec;
    // mel front end + conv subsampling (optional: built when the conv
    // subsampling tensors are loaded)
    struct Frontend {
        bool present = false;
        DevBuf tables;        // window [512] | twiddle [256][2] | fb [128][257] (f32) | fb_lo [128] | fb_hi [128] (i32)
        DevBuf conv;          // w0 | b0 | w2 | b2 | w5 | b5 (f32, [256][9] + [256] each)
        Linear pw1, pw2;      // pointwise convs, f16 [256][256]
        DevBuf pw_bias;       // [2][256] f32
        Linear sub_w_perm;    // encoder subsampling linear, input columns in (freq, channel) order
        DevBuf wave, wave_off, frame_off, mel, x2, x3, x4, ints, work, rows3;
        int fb_packed = 0;    // weights in the packed filterbank spans
        std::vector<int32_t> sub_key;   // batch shape whose tables are on the device
        std::vector<int64_t> mel_key;   // padded wave offsets of the cached shape
        FeShape mel_shape;
        // host-pointer input: the waves go up in utterance chunks on their own
        // stream, each chunk's front end waiting only for its own copies
        cudaStream_t copy_st = nullptr;
        cudaEvent_t wave_free = nullptr;
        std::vector<cudaEvent_t> chunk_ev;
        std::vector<int> chunk_u;   // chunk c = utterances [chunk_u[c], chunk_u[c + 1])
        bool chunk_wait = false;    // chunk_ev holds this call's copies
    } fe;
    ~b3_ctx() {
        enc_graph.reset();
        for (Linear* l : {&fe.pw1, &fe.pw2, &fe.sub_w_perm}) {
            l->w.release();
            l->lut16.release();
        }
        if (fe.copy_st) cudaStreamSynchronize(fe.copy_st);
        for (DevBuf* b : {&fe.tables, &fe.conv, &fe.pw_bias, &fe.wave, &fe.wave_off, &fe.frame_off, &fe.mel, &fe.x2,
                          &fe.x3, &fe.x4, &fe.ints, &fe.work, &fe.rows3})
            b->release();
        for (cudaEvent_t e : fe.chunk_ev) cudaEventDestroy(e);
        if (fe.wave_free) cudaEventDestroy(fe.wave_free);
        if (fe.copy_st) cudaStreamDestroy(fe.copy_st);
        for (cudaEvent_t e : prof.pool) cudaEventDestroy(e);
        for (Linear* l : {&dec.lstm[0], &dec.lstm[1], &dec.proj, &dec.head}) {
            l->w.release();
            l->lut16.release();
        }
        for (DevBuf* b : {&dec.e0, &dec.bias, &dec.a0, &dec.a1, &dec.ap, &dec.aj, &dec.gates, &dec.cstate, &dec.dec,
                          &dec.scores, &dec.ints, &dec.tokens, &dec.rows, &dec.sync, &dec.pooler})
            b->release();
        auto rel = [](Linear& l) { l.w.release(); l.lut16.release(); };
        rel(sub_w);
        rel(proj_w);
        for (auto& L : layers) {
            rel(L.qkv); rel(L.relk); rel(L.o); rel(L.ff1a); rel(L.ff1b);
            rel(L.ff2a); rel(L.ff2b); rel(L.pw1); rel(L.pw2);
            L.params.release();
        }
        for (DevBuf* b : {&sub_b, &proj_b, &inv_freq, &pos16, &x, &a16, &h16, &qkv16, &g16, &sub16,
                          &R16, &cu_d, &work_d, &seg_d, &io_in, &io_out, &scratch16})
            b->release();
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Wraps one kernel launch: counts it and, when profiling, brackets it with
// events on the context stream.
struct ProfScope {
    b3_ctx* c;
    int kind;
    int ev = -1;
    double flops, bytes;
    ProfScope(b3_ctx* c_, int kind_, double flops_, double bytes_) : c(c_), kind(kind_), flops(flops_), bytes(bytes_) {
        c->prof.launches[kind]++;
        Prof& p = c->prof;
        if (p.on && p.next + 2 <= static_cast<int>(p.pool.size())) {
            ev = p.next;
            p.next += 2;
            cudaEventRecord(p.pool[ev], c->stream);
        }
    }
    ~ProfScope() {
        if (ev >= 0) {
            cudaEventRecord(c->prof.pool[ev + 1], c->stream);
            c->prof.recs.push_back({kind, ev, flops, bytes});
        }
    }
};

int prof_collect(b3_ctx* c) {
    Prof& p = c->prof;
    if (p.recs.empty()) return 0;
    B3_CUDA(cudaStreamSynchronize(c->stream));
    for (const ProfRec& r : p.recs) {
        float ms = 0.f;
        B3_CUDA(cudaEventElapsedTime(&ms, p.pool[r.ev], p.pool[r.ev + 1]));
        p.ms[r.kind] += ms;
        p.flops[r.kind] += r.flops;
        p.bytes[r.kind] += r.bytes;
        p.timed[r.kind]++;
    }
    p.recs.clear();
    p.next = 0;
    return 0;
}

uint16_t f32_to_f16_bits(float v) {
    __half h = __float2half_rn(v);
    return *reinterpret_cast<uint16_t*>(&h);
}

float f16_bits_to_f32(uint16_t b) {
    __half h = *reinterpret_cast<__half*>(&b);
    return __half2float(h);
}

float bf16_bits_to_f32(uint16_t b) {
    uint32_t x = (static_cast<uint32_t>(b) & 0x8000u) << 16 | ((static_cast<uint32_t>(b) & 0x7FFFu) << 16);
    float f;
    memcpy(&f, &x, 4);
    return f;
}

int upload(DevBuf& dst, const void* src, size_t bytes, cudaStream_t st) {
    B3_TRY(dst.ensure(bytes));
    B3_CUDA(cudaMemcpyAsync(dst.p, src, bytes, cudaMemcpyHostToDevice, st));
    return 0;
}

const Staged* find(b3_ctx* c, const std::string& name) {
    auto it = c->staged.find(name);
    return it == c->staged.end() ? nullptr : &it->second;
}

int64_t numel(const Staged& s) {
    int64_t n = 1;
    for (int64_t d : s.shape) n *= d;
    return n;
}

// Dense f32 values of a small tensor (LN, biases, BN statistics).
int get_vec(b3_ctx* c, const std::string& name, int64_t n, std::vector<float>& out) {
    const Staged* s = find(c, name);
    if (!s) return set_error(B3_ENOTFOUND, "tensor %s was not loaded", name.c_str());
    if (s->lowbit || numel(*s) != n)
        return set_error(B3_EINVAL, "tensor %s: expected %lld dense values", name.c_str(), (long long)n);
    out = s->f32;
    return 0;
}

// Build a device linear from one or more staged (N_i, K) matrices stacked by
// rows.  All parts must share the storage kind (the reference refuses a mixed
// fused q|k|v too, src/encoder.rs:389-392).  `interleave_halves` reorders the
// rows as (0, N/2, 1, N/2+1, ...) so a GLU pair lands in adjacent columns.
int build_linear(b3_ctx* c, Linear& L, const std::vector<std::string>& names, int n_each, int K,
                 bool interleave_halves) {
    std::vector<const Staged*> parts;
    for (auto& nm : names) {
        const Staged* s = find(c, nm);
        if (!s) return set_error(B3_ENOTFOUND, "tensor %s was not loaded", nm.c_str());
        parts.push_back(s);
    }
    const bool lut = parts[0]->lowbit;
    for (auto* s : parts)
        if (s->lowbit != lut)
            return set_error(B3_EINVAL, "%s: fused parts mix 4-bit and dense storage", names[0].c_str());
    const int N = n_each * static_cast<int>(parts.size());
    for (size_t i = 0; i < parts.size(); ++i) {
        const Staged* s = parts[i];
        const int64_t rows = lut ? s->rows : (s->shape.empty() ? 0 : s->shape[0]);
        const int64_t cols = lut ? s->cols : (rows ? numel(*s) / rows : 0);
        if (rows != n_each || cols != K)
            return set_error(B3_EINVAL, "tensor %s: shape (%lld, %lld), expected (%d, %d)", names[i].c_str(),
                             (long long)rows, (long long)cols, n_each, K);
    }
    auto src_row = [&](int r) -> std::pair<const Staged*, int> {
        int rr = r;
        if (interleave_halves) rr = (r & 1) ? N / 2 + r / 2 : r / 2;
        return {parts[rr / n_each], rr % n_each};
    };
    L.present = true;
    L.lut = lut;
    L.N = N;
    L.K = K;
    if (lut) {
        std::vector<uint8_t> codes(static_cast<size_t>(N) * K / 2);
        std::vector<uint16_t> tab(static_cast<size_t>(N) * 16);
        for (int r = 0; r < N; ++r) {
            auto [s, sr] = src_row(r);
            memcpy(&codes[static_cast<size_t>(r) * K / 2], &s->codes[static_cast<size_t>(sr) * K / 2], K / 2);
            memcpy(&tab[static_cast<size_t>(r) * 16], &s->lut16[static_cast<size_t>(sr) * 16], 32);
        }
        B3_TRY(upload(L.w, codes.data(), codes.size(), c->stream));
        B3_TRY(upload(L.lut16, tab.data(), tab.size() * 2, c->stream));
        B3_CUDA(cudaStreamSynchronize(c->stream));
    } else {
        std::vector<uint16_t> w(static_cast<size_t>(N) * K);
        for (int r = 0; r < N; ++r) {
            auto [s, sr] = src_row(r);
            memcpy(&w[static_cast<size_t>(r) * K], &s->f16[static_cast<size_t>(sr) * K], static_cast<size_t>(K) * 2);
        }
        B3_TRY(upload(L.w, w.data(), w.size() * 2, c->stream));
        B3_CUDA(cudaStreamSynchronize(c->stream));
    }
    return gemm_make_b_map(&L.map_b, L.w.p, lut, N, K);
}

// ───────────────────────────── GEMM helper ─────────────────────────────

// Algorithmic DRAM bytes of one GEMM: A once, W once (codes + tables or f16),
// the output once (read + write for the residual update).
double gemm_bytes(int M, int N, int K, bool lut, int epi) {
    const double a = 2.0 * M * K;
    const double w = lut ? (0.5 * N * K + 32.0 * N) : 2.0 * N * K;
    double o;
    switch (epi) {
        case EPI_F32: o = 4.0 * M * N; break;
        case EPI_RESID: o = 8.0 * M * N; break;
        case EPI_GLU_F16: o = 1.0 * M * N; break;
        case EPI_QKV: o = 2.0 * M * N + 2.0 * M * 1024; break;
        default: o = 2.0 * M * N; break;
    }
    return a + w + o;
}

int k_layernorm(b3_ctx* c, const float* x, int rows, const float* w1, const float* b1, float* y32,
                const float* w2, const float* b2, __half* y16) {
    ProfScope ps(c, B3_K_LAYERNORM, 0.0, rows * (4096.0 + (y32 ? 4096.0 : 0.0) + (y16 ? 2048.0 : 0.0)));
    return launch_layernorm(x, rows, w1, b1, y32, w2, b2, y16, c->stream);
}

int k_dwconv(b3_ctx* c, const __half* src, int rows, const float* dw_t, const float* bn_a, const float* bn_b,
             __half* dst) {
    ProfScope ps(c, B3_K_DWCONV, 2.0 * 9 * 1024 * rows, rows * 4096.0);
    return launch_dwconv(src, c->seg_d.as<int2>(), rows, dw_t, bn_a, bn_b, dst, c->stream);
}

int k_convert(b3_ctx* c, const float* src, __half* dst, int64_t n) {
    ProfScope ps(c, B3_K_CONVERT, 0.0, 6.0 * n);
    return launch_f32_to_f16(src, dst, n, c->stream);
}

int run_gemm(b3_ctx* c, const Linear& W, const __half* a, int M, int lda, int epi, GemmParams p) {
    GemmOp op;
    B3_TRY(gemm_make_a_map(&op.map_a, a, M, W.K, lda));
    op.map_b = W.map_b;
    p.M = M;
    p.N = W.N;
    p.K = W.K;
    p.lut = W.lut ? W.lut16.as<uint16_t>() : nullptr;
    op.p = p;
    op.lut = W.lut;
    op.epi = epi;
    ProfScope ps(c, W.lut ? B3_K_GEMM_LUT4 : B3_K_GEMM_F16, 2.0 * M * W.N * W.K,
                 gemm_bytes(M, W.N, W.K, W.lut, epi));
    return gemm_launch(op, c->stream);
}

GemmParams params_f32(float* out, int ldo, const float* bias) {
    GemmParams p{};
    p.out_f32 = out;
    p.ldo = ldo;
    p.bias = bias;
    return p;
}

GemmParams params_resid(float* x, float alpha) {
    GemmParams p{};
    p.out_f32 = x;
    p.ldo = kHidden;
    p.alpha = alpha;
    return p;
}

GemmParams params_f16(__half* out, int ldo) {
    GemmParams p{};
    p.out_f16 = out;
    p.ldo = ldo;
    return p;
}

// ───────────────────────────── planning ─────────────────────────────

int ensure_arena(b3_ctx* c, int M) {
    if (M <= c->mcap) return 0;
    int mcap = ((M + 255) / 256) * 256;
    const size_t m = static_cast<size_t>(mcap);
    B3_TRY(c->x.ensure(m * kHidden * 4));
    B3_TRY(c->a16.ensure(m * kHidden * 2));
    B3_TRY(c->h16.ensure(m * kFfn * 2));
    B3_TRY(c->qkv16.ensure(m * 4096 * 2));
    B3_TRY(c->g16.ensure(m * kHidden * 2));
    B3_TRY(c->sub16.ensure(m * kSubIn * 2));
    B3_TRY(c->seg_d.ensure(m * sizeof(int2)));
    B3_TRY(c->work_d.ensure((m / 64 + 1024) * sizeof(int4)));
    c->mcap = mcap;
    return 0;
}

int ensure_pos(b3_ctx* c, int tmax) {
    if (tmax <= c->tcap) return 0;
    int tcap = ((tmax + 511) / 512) * 512;
    const int rows = 2 * tcap - 1;
    B3_TRY(c->pos16.ensure(static_cast<size_t>(rows + 1) * kHidden * 2));
    B3_TRY(c->R16.ensure(static_cast<size_t>(rows + 1) * kHidden * 2));
    {
        ProfScope ps(c, B3_K_OTHER, 0.0, rows * 2048.0);
        B3_TRY(launch_pos_table(c->inv_freq.as<float>(), tcap, rows, c->pos16.as<__half>(), c->stream));
    }
    c->tcap = tcap;
    return 0;
}

int make_plan(b3_ctx* c, const int32_t* cu, int n_utt) {
    if (n_utt <= 0) return set_error(B3_EINVAL, "batch needs at least one utterance");
    if (cu[0] != 0) return set_error(B3_EINVAL, "cu_seqlens[0] must be 0");
    int tmax = 0;
    for (int i = 0; i < n_utt; ++i) {
        const int t = cu[i + 1] - cu[i];
        if (t <= 0) return set_error(B3_EINVAL, "utterance %d has %d frames", i, t);
        if (t > tmax) tmax = t;
    }
    const int M = cu[n_utt];
    std::vector<int32_t> key(cu, cu + n_utt + 1);
    if (key == c->plan.cu && c->mcap >= M && c->tcap >= tmax) return 0;
    ++c->plan_gen;
    B3_TRY(ensure_arena(c, M));
    B3_TRY(ensure_pos(c, tmax));
    const int bq = attention_tc_block_rows();
    // attention work entries: (first row of the utterance, its frames, first
    // query, 0), every value an item needs in one load
    std::vector<int4> work;
    std::vector<int2> seg(M);
    for (int i = 0; i < n_utt; ++i) {
        for (int q = 0; q < cu[i + 1] - cu[i]; q += bq) work.push_back(make_int4(cu[i], cu[i + 1] - cu[i], q, 0));
        for (int r = cu[i]; r < cu[i + 1]; ++r) seg[r] = make_int2(cu[i], cu[i + 1]);
    }
    // attention CTAs of the longest utterances first (their key loops are
    // longest), so the last wave is made of short ones
    std::stable_sort(work.begin(), work.end(), [](const int4& a, const int4& b) { return a.y > b.y; });
    B3_TRY(c->work_d.ensure(work.size() * sizeof(int4)));
    B3_TRY(c->cu_d.ensure(key.size() * sizeof(int32_t)));
    B3_CUDA(cudaMemcpyAsync(c->work_d.p, work.data(), work.size() * sizeof(int4), cudaMemcpyHostToDevice, c->stream));
    B3_CUDA(cudaMemcpyAsync(c->seg_d.p, seg.data(), seg.size() * sizeof(int2), cudaMemcpyHostToDevice, c->stream));
    B3_CUDA(cudaMemcpyAsync(c->cu_d.p, key.data(), key.size() * sizeof(int32_t), cudaMemcpyHostToDevice, c->stream));
    B3_CUDA(cudaStreamSynchronize(c->stream));
    c->plan.cu = key;
    c->plan.M = M;
    c->plan.tmax = tmax;
    c->plan.n_work = static_cast<int>(work.size());
    return 0;
}

// ───────────────────────────── forward ─────────────────────────────

// Attention section of block L: x += o_proj(MHSA(LN_att(x))).
int attention_section(b3_ctx* c, const Layer& L, int M) {
    float* x = c->x.as<float>();
    __half* a16 = c->a16.as<__half>();
    __half* qkv = c->qkv16.as<__half>();
    const int tmax = c->plan.tmax;
    B3_TRY(k_layernorm(c, x, M, L.ln_w(1), L.ln_b(1), nullptr, nullptr, nullptr, a16));
    GemmParams pq = params_f16(qkv, 4096);
    pq.bias_u = L.bu();
    pq.bias_v = L.bv();
    B3_TRY(run_gemm(c, L.qkv, a16, M, kHidden, EPI_QKV, pq));
    // R = pos[positions tmax-1 .. -(tmax-1)] . W_relk^T  (rounded to f16)
    const int prow0 = c->tcap - tmax;
    const int prows = 2 * tmax - 1;
    const __half* pos = c->pos16.as<__half>() + static_cast<size_t>(prow0) * kHidden;
    B3_TRY(run_gemm(c, L.relk, pos, prows, kHidden, EPI_F16, params_f16(c->R16.as<__half>(), kHidden)));
    AttnParams ap;
    ap.qkv = qkv;
    ap.R = c->R16.as<__half>();
    ap.r_center = tmax - 1;
    ap.r_rows = prows;
    ap.work = c->work_d.as<int4>();
    ap.out = a16;
    ap.scale_log2 = 1.4426950408889634f / std::sqrt(128.0f);
    {
        double fl = 0.0, by = 0.0;
        for (size_t i = 0; i + 1 < c->plan.cu.size(); ++i) {
            const double t = c->plan.cu[i + 1] - c->plan.cu[i];
            fl += 6144.0 * t * t;                       // 8 heads x (QK + band + PV), 2*128 each
            by += t * 1024 * 2 * 5 + (2 * t - 1) * 2048; // qu qv k v in, out; R band
        }
        ProfScope ps(c, B3_K_ATTENTION, fl, by);
        B3_TRY(launch_attention_tc(ap, M, c->plan.n_work, c->stream));
    }
    return run_gemm(c, L.o, a16, M, kHidden, EPI_RESID, params_resid(x, 1.0f));
}

// Conv section of block L: x += pw2(SiLU(BN(dwconv(GLU(pw1(LN_conv(x))))))).
int conv_section(b3_ctx* c, const Layer& L, int M) {
    float* x = c->x.as<float>();
    __half* a16 = c->a16.as<__half>();
    __half* g16 = c->g16.as<__half>();
    B3_TRY(k_layernorm(c, x, M, L.ln_w(2), L.ln_b(2), nullptr, nullptr, nullptr, a16));
    B3_TRY(run_gemm(c, L.pw1, a16, M, kHidden, EPI_GLU_F16, params_f16(g16, kHidden)));
    B3_TRY(k_dwconv(c, g16, M, L.dw_t(), L.bn_a(), L.bn_b(), a16));
    return run_gemm(c, L.pw2, a16, M, kHidden, EPI_RESID, params_resid(x, 1.0f));
}

// FFN half: x += 0.5 * W2 SiLU(W1 a16), a16 already holding LN(x).
int ffn_half(b3_ctx* c, const Linear& w1, const Linear& w2, int M) {
    B3_TRY(run_gemm(c, w1, c->a16.as<__half>(), M, kHidden, EPI_SILU_F16, params_f16(c->h16.as<__half>(), kFfn)));
    return run_gemm(c, w2, c->h16.as<__half>(), M, kFfn, EPI_RESID, params_resid(c->x.as<float>(), 0.5f));
}

// sub16 holds the f16 input; runs `layers` blocks.  After the call:
//   layers == n_layers: a16 = f16(norm_out(x)) of the last block, x = norm_out(x)
//   otherwise:          x = pre-norm_out residual of block layers-1
// `subw` is the subsampling linear matching sub16's column order (the
// reference's (channel, freq) order, or (freq, channel) from the GPU front end).
int forward_blocks(b3_ctx* c, int M, int layers, const Linear* subw = nullptr) {
    float* x = c->x.as<float>();
    __half* a16 = c->a16.as<__half>();
    B3_TRY(run_gemm(c, subw ? *subw : c->sub_w, c->sub16.as<__half>(), M, kSubIn, EPI_F32,
                    params_f32(x, kHidden, c->sub_b.as<float>())));
    const int upto = layers < c->n_layers ? layers : c->n_layers;
    if (upto > 0) {
        const Layer& L0 = c->layers[0];
        B3_TRY(k_layernorm(c, x, M, L0.ln_w(0), L0.ln_b(0), nullptr, nullptr, nullptr, a16));
    }
    for (int i = 0; i < upto; ++i) {
        const Layer& L = c->layers[i];
        // a16 = LN_ff1(x) on entry
        B3_TRY(ffn_half(c, L.ff1a, L.ff1b, M));
        B3_TRY(attention_section(c, L, M));
        B3_TRY(conv_section(c, L, M));
        B3_TRY(k_layernorm(c, x, M, L.ln_w(3), L.ln_b(3), nullptr, nullptr, nullptr, a16));
        B3_TRY(ffn_half(c, L.ff2a, L.ff2b, M));
        const bool last = (i + 1 == upto);
        if (!last) {
            const Layer& N = c->layers[i + 1];
            B3_TRY(k_layernorm(c, x, M, L.ln_w(4), L.ln_b(4), x, N.ln_w(0), N.ln_b(0), a16));
        } else if (upto == c->n_layers) {
            B3_TRY(k_layernorm(c, x, M, L.ln_w(4), L.ln_b(4), x, nullptr, nullptr, a16));
        }
    }
    if (upto == 0 && c->n_layers == 0)
        return set_error(B3_ESTATE, "encoder has no blocks");
    return 0;
}

int check_finalized(b3_ctx* c) {
    if (!c) return set_error(B3_EINVAL, "null context");
    if (!c->finalized) return set_error(B3_ESTATE, "b3_finalize has not been called");
    return 0;
}

// Waits for the context stream, then reads and clears the device error words
// of every module with bounded waits (K1 GEMM, attention, decoder): any set
// bit means a wait ran out and the call's results are not valid.
int sync_and_check(b3_ctx* c) {
    B3_CUDA(cudaStreamSynchronize(c->stream));
    unsigned int flag = 0, aflag = 0, dflag = 0;
    B3_TRY(gemm_take_dev_error(c->stream, &flag));
    B3_TRY(attention_take_dev_error(c->stream, &aflag));
    B3_TRY(decoder_take_dev_error(c->stream, &dflag));
    if (flag | aflag | dflag)
        return set_error(B3_ETIMEOUT, "device wait ran out (gemm 0x%x, attention 0x%x, decoder 0x%x)", flag, aflag,
                         dflag);
    return 0;
}

// Encode rows already in device memory: sub (f32 [M][4096]) -> out.
int encode_device(b3_ctx* c, const float* sub, int M, int layers, float* out) {
    B3_TRY(k_convert(c, sub, c->sub16.as<__half>(), static_cast<int64_t>(M) * kSubIn));
    B3_TRY(forward_blocks(c, M, layers));
    if (layers >= c->n_layers) {
        B3_TRY(run_gemm(c, c->proj_w, c->a16.as<__half>(), M, kHidden, EPI_F32,
                        params_f32(out, kProj, c->proj_b.as<float>())));
    } else {
        B3_CUDA(cudaMemcpyAsync(out, c->x.p, static_cast<size_t>(M) * kHidden * 4, cudaMemcpyDeviceToDevice, c->stream));
    }
    return 0;
}

// Rows up to which a repeated encode replays a graph (above it the kernels
// outweigh the launches by far).
constexpr int kGraphRows = 8192;

// encode_device, replayed from a CUDA graph when the same call (rows, input
// and output buffers, block count, plan) comes again.  The first call of a
// key runs eagerly (it also does the kernels' one-time set-up), the second
// captures and replays, later ones replay.  Off while profiling (the
// per-launch events are host-side bookkeeping) and for large batches.
int encode_rows(b3_ctx* c, const float* sub, int M, int layers, float* out) {
    auto& G = c->enc_graph;
    if (c->prof.on || M > kGraphRows) return encode_device(c, sub, M, layers, out);
    const bool same = G.sub == sub && G.out == out && G.M == M && G.layers == layers && G.gen == c->plan_gen;
    if (!same) {
        G.reset();
        G.sub = sub;
        G.out = out;
        G.M = M;
        G.layers = layers;
        G.gen = c->plan_gen;
    }
    if (G.exec) {
        B3_CUDA(cudaGraphLaunch(G.exec, c->stream));
        return 0;
    }
    if (!G.seen || G.no_graph) {
        G.seen = true;
        return encode_device(c, sub, M, layers, out);
    }
    cudaGraph_t graph = nullptr;
    B3_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = encode_device(c, sub, M, layers, out);
    cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
    if (rc == 0 && e == cudaSuccess) e = cudaGraphInstantiate(&G.exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (rc != 0 || e != cudaSuccess) {
        // nothing was launched while capturing: run the call eagerly, and keep
        // this key eager from now on
        cudaGetLastError();
        G.exec = nullptr;
        G.no_graph = true;
        return encode_device(c, sub, M, layers, out);
    }
    B3_CUDA(cudaGraphLaunch(G.exec, c->stream));
    return 0;
}

int encode_any(b3_ctx* c, const float* sub, const int32_t* cu, int n_utt, int layers, float* out,
               unsigned flags) {
    B3_TRY(check_finalized(c));
    if (!sub || !out || !cu) return set_error(B3_EINVAL, "null buffer");
    DeviceGuard g(c->device);
    B3_TRY(make_plan(c, cu, n_utt));
    const int M = c->plan.M;
    const int out_cols = layers >= c->n_layers ? kProj : kHidden;
    if (flags & B3_DEVICE_PTRS) return encode_rows(c, sub, M, layers, out);
    const size_t in_bytes = static_cast<size_t>(M) * kSubIn * 4;
    const size_t out_bytes = static_cast<size_t>(M) * out_cols * 4;
    B3_TRY(c->io_in.ensure(in_bytes));
    B3_TRY(c->io_out.ensure(out_bytes));
    B3_CUDA(cudaMemcpyAsync(c->io_in.p, sub, in_bytes, cudaMemcpyHostToDevice, c->stream));
    B3_TRY(encode_rows(c, c->io_in.as<float>(), M, layers, c->io_out.as<float>()));
    B3_CUDA(cudaMemcpyAsync(out, c->io_out.p, out_bytes, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

// ───────────────────────────── TDT decoder ─────────────────────────────

int build_dense(b3_ctx* c, Linear& L, const std::vector<uint16_t>& w, int N, int K) {
    L.present = true;
    L.lut = false;
    L.N = N;
    L.K = K;
    B3_TRY(upload(L.w, w.data(), w.size() * 2, c->stream));
    B3_CUDA(cudaStreamSynchronize(c->stream));
    return gemm_make_b_map(&L.map_b, L.w.p, false, N, K);
}

// A (rows, 640) dense matrix staged under `name`, rounded to f16 (pack16,
// src/tdt.rs:49-55).
int dec_matrix(b3_ctx* c, const std::string& name, int rows, const std::vector<uint16_t>** out) {
    const Staged* s = find(c, name);
    if (!s) return set_error(B3_ENOTFOUND, "tensor %s was not loaded", name.c_str());
    if (s->lowbit || numel(*s) != static_cast<int64_t>(rows) * 640)
        return set_error(B3_EINVAL, "tensor %s: expected (%d, 640)", name.c_str(), rows);
    *out = &s->f16;
    return 0;
}

// Builds the decoder from the staged tensors (TdtDecoder::from_source,
// src/tdt.rs:142-163).  Every GEMM weight is repeated along K so the f16
// hi | lo halves of an activation meet the same weight.
int build_decoder(b3_ctx* c) {
    auto& D = c->dec;
    const Staged* e = find(c, "decoder.embedding.weight");
    if (!e) return 0;  // encoder-only checkpoint
    if (e->lowbit || e->shape.size() != 2 || e->shape[1] != 640 || e->shape[0] < 2)
        return set_error(B3_EINVAL, "decoder.embedding.weight must be (vocab, 640)");
    const int V = static_cast<int>(e->shape[0]);
    const int H = 640, G = 2560;
    D.vocab = V;
    D.npad = (V + 5 + 127) / 128 * 128;
    std::vector<float> bias(2 * G + H + D.npad, 0.f), v1, v2;
    std::vector<float> bias0(G);
    Linear wih0;   // [2560][1280] = W_ih0 | W_ih0, used once for the E0 table
    for (int l = 0; l < 2; ++l) {
        const std::string sl = std::to_string(l);
        const std::vector<uint16_t>*wih, *whh;
        B3_TRY(dec_matrix(c, "decoder.lstm.weight_ih_l" + sl, G, &wih));
        B3_TRY(dec_matrix(c, "decoder.lstm.weight_hh_l" + sl, G, &whh));
        const int parts = l == 0 ? 2 : 4;   // layer 0: W_hh | W_hh only
        std::vector<uint16_t> w(static_cast<size_t>(G) * parts * H);
        for (int r = 0; r < G; ++r) {
            uint16_t* dst = &w[static_cast<size_t>(r) * parts * H];
            const uint16_t* src_ih = &(*wih)[static_cast<size_t>(r) * H];
            const uint16_t* src_hh = &(*whh)[static_cast<size_t>(r) * H];
            if (l == 1) {
                memcpy(dst, src_ih, H * 2);
                memcpy(dst + H, src_ih, H * 2);
                dst += 2 * H;
            }
            memcpy(dst, src_hh, H * 2);
            memcpy(dst + H, src_hh, H * 2);
        }
        B3_TRY(build_dense(c, D.lstm[l], w, G, parts * H));
        if (l == 0) {
            std::vector<uint16_t> wi(static_cast<size_t>(G) * 2 * H);
            for (int r = 0; r < G; ++r) {
                memcpy(&wi[static_cast<size_t>(r) * 2 * H], &(*wih)[static_cast<size_t>(r) * H], H * 2);
                memcpy(&wi[static_cast<size_t>(r) * 2 * H + H], &(*wih)[static_cast<size_t>(r) * H], H * 2);
            }
            B3_TRY(build_dense(c, wih0, wi, G, 2 * H));
        }
        B3_TRY(get_vec(c, "decoder.lstm.bias_ih_l" + sl, G, v1));
        B3_TRY(get_vec(c, "decoder.lstm.bias_hh_l" + sl, G, v2));
        for (int r = 0; r < G; ++r) (l == 0 ? bias0[r] : bias[l * G + r]) = v1[r] + v2[r];
    }
    {
        // E0 = [emb_hi | emb_lo] . [W_ih0 | W_ih0]^T + b0 on the tensor cores
        DevBuf tmp, hl, b0;
        B3_TRY(upload(tmp, e->f32.data(), e->f32.size() * 4, c->stream));
        B3_TRY(upload(b0, bias0.data(), bias0.size() * 4, c->stream));
        B3_TRY(hl.ensure(static_cast<size_t>(V) * 2 * H * 2));
        __half* hi = hl.as<__half>();
        DevBuf lo;
        B3_TRY(lo.ensure(static_cast<size_t>(V) * H * 2));
        B3_TRY(dec_launch_split(tmp.as<float>(), hi, lo.as<__half>(), static_cast<int64_t>(V) * H, c->stream));
        // hi rows were written densely [V][640]: spread them to [V][1280] and put lo beside them
        DevBuf packed;
        B3_TRY(packed.ensure(static_cast<size_t>(V) * 2 * H * 2));
        B3_CUDA(cudaMemcpy2DAsync(packed.p, 2 * H * 2, hi, H * 2, H * 2, V, cudaMemcpyDeviceToDevice, c->stream));
        B3_CUDA(cudaMemcpy2DAsync(packed.as<__half>() + H, 2 * H * 2, lo.p, H * 2, H * 2, V, cudaMemcpyDeviceToDevice,
                                  c->stream));
        B3_TRY(D.e0.ensure(static_cast<size_t>(V) * G * 4));
        B3_TRY(run_gemm(c, wih0, packed.as<__half>(), V, 2 * H, EPI_F32, params_f32(D.e0.as<float>(), G, b0.as<float>())));
        B3_CUDA(cudaStreamSynchronize(c->stream));
        wih0.w.release();
        wih0.lut16.release();
    }
    auto doubled = [&](const std::vector<uint16_t>& src, int rows, int out_rows) {
        std::vector<uint16_t> w(static_cast<size_t>(out_rows) * 2 * H, 0);
        for (int r = 0; r < rows; ++r) {
            memcpy(&w[static_cast<size_t>(r) * 2 * H], &src[static_cast<size_t>(r) * H], H * 2);
            memcpy(&w[static_cast<size_t>(r) * 2 * H + H], &src[static_cast<size_t>(r) * H], H * 2);
        }
        return w;
    };
    const std::vector<uint16_t>* wp;
    B3_TRY(dec_matrix(c, "decoder.decoder_projector.weight", H, &wp));
    B3_TRY(build_dense(c, D.proj, doubled(*wp, H, H), H, 2 * H));
    B3_TRY(get_vec(c, "decoder.decoder_projector.bias", H, v1));
    memcpy(&bias[2 * G], v1.data(), H * 4);
    const std::vector<uint16_t>* wh;
    B3_TRY(dec_matrix(c, "joint.head.weight", V + 5, &wh));
    B3_TRY(build_dense(c, D.head, doubled(*wh, V + 5, D.npad), D.npad, 2 * H));
    B3_TRY(get_vec(c, "joint.head.bias", V + 5, v1));
    memcpy(&bias[2 * G + H], v1.data(), (V + 5) * 4);
    B3_TRY(upload(D.bias, bias.data(), bias.size() * 4, c->stream));
    {
        // weight-stationary tiles (DecWs): head rows, then the three LSTM
        // matrices with 32 channels x 4 gates per tile, then the projector
        const int ht = (V + 5 + 127) / 128;
        const int n_roles = ht + 3 * kWsLstmTiles + kWsProjTiles;
        std::vector<uint16_t> wt(static_cast<size_t>(n_roles) * 128 * H, 0);
        auto put = [&](int dst_row, const std::vector<uint16_t>& src, int src_row) {
            memcpy(&wt[static_cast<size_t>(dst_row) * H], &src[static_cast<size_t>(src_row) * H], H * 2);
        };
        for (int r = 0; r < V + 5; ++r) put(r, *wh, r);
        const std::vector<uint16_t>*whh0, *whh1, *wih1;
        B3_TRY(dec_matrix(c, "decoder.lstm.weight_hh_l0", G, &whh0));
        B3_TRY(dec_matrix(c, "decoder.lstm.weight_hh_l1", G, &whh1));
        B3_TRY(dec_matrix(c, "decoder.lstm.weight_ih_l1", G, &wih1));
        const std::vector<uint16_t>* lstm[3] = {whh0, whh1, wih1};
        for (int m = 0; m < 3; ++m)
            for (int t = 0; t < kWsLstmTiles; ++t)
                for (int q = 0; q < 4; ++q)
                    for (int ch = 0; ch < 32; ++ch)
                        put((ht + m * kWsLstmTiles + t) * 128 + q * 32 + ch, *lstm[m], q * H + 32 * t + ch);
        for (int r = 0; r < H; ++r) put((ht + 3 * kWsLstmTiles) * 128 + r, *wp, r);
        std::vector<float> wb(static_cast<size_t>(ht) * 128 + G + H, 0.f);
        memcpy(wb.data(), v1.data(), (V + 5) * 4);                  // head bias
        memcpy(wb.data() + ht * 128, &bias[G], G * 4);               // b_ih1 + b_hh1
        memcpy(wb.data() + ht * 128 + G, &bias[2 * G], H * 4);       // projector bias
        B3_TRY(upload(D.ws_w, wt.data(), wt.size() * 2, c->stream));
        B3_TRY(upload(D.ws_bias, wb.data(), wb.size() * 4, c->stream));
        B3_TRY(make_map_2d(&D.ws_wmap, D.ws_w.p, kMapF16, H, static_cast<uint64_t>(n_roles) * 128, 2 * H, 64, 128,
                           true));
        D.ws_ht = ht;
    }
    B3_CUDA(cudaStreamSynchronize(c->stream));
    D.present = true;
    return 0;
}

// Greedy decode with the weight-stationary kernel (DecWs): batches of up to
// 2 x 128 rows on n_roles x nsplit CTAs.  Tokens and counts land where
// decode_collect reads them.
int decode_ws(b3_ctx* c, const float* pooler, const std::vector<int32_t>& rows, int B, int tmax, int max_tokens,
              int nsplit, int grid) {
    auto& D = c->dec;
    const int ntile = ((B + nsplit - 1) / nsplit + 31) / 32 * 32;
    const int bpad = ntile * nsplit;
    const size_t act_bytes = static_cast<size_t>(bpad) * 1280 * 2;
    B3_TRY(D.a0.ensure(act_bytes));
    B3_TRY(D.ap.ensure(act_bytes));
    B3_TRY(D.aj.ensure(act_bytes));
    B3_TRY(D.cstate.ensure(static_cast<size_t>(B) * 2 * 640 * 4));
    B3_TRY(D.gates.ensure(static_cast<size_t>(bpad) * 2560 * 4));
    B3_TRY(D.ws_keys.ensure(static_cast<size_t>(B) * 4 * 8));
    B3_TRY(D.ints.ensure(static_cast<size_t>(B) * 6 * 4));
    B3_TRY(D.tokens.ensure(static_cast<size_t>(B) * max_tokens * 12));
    B3_TRY(D.rows.ensure(static_cast<size_t>(B) * 2 * 4));
    B3_TRY(D.sync.ensure(32));
    ProfScope ps(c, B3_K_DECODER, 0.0, 0.0);
    c->prof.launches[B3_K_DECODER]++;
    // frame | count | guard (0) | alive of steps 0 and -1 (utterances with frames)
    std::vector<int32_t> ints(static_cast<size_t>(B) * 5, 0);
    for (int b = 0; b < B; ++b) ints[3 * B + b] = ints[4 * B + b] = rows[B + b] > 0 ? 1 : 0;
    B3_CUDA(cudaMemcpyAsync(D.rows.p, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice, c->stream));
    B3_CUDA(cudaMemcpyAsync(D.ints.p, ints.data(), ints.size() * 4, cudaMemcpyHostToDevice, c->stream));
    B3_CUDA(cudaMemsetAsync(D.a0.p, 0, act_bytes, c->stream));
    B3_CUDA(cudaMemsetAsync(D.ap.p, 0, act_bytes, c->stream));
    B3_CUDA(cudaMemsetAsync(D.aj.p, 0, act_bytes, c->stream));
    B3_CUDA(cudaMemsetAsync(D.cstate.p, 0, static_cast<size_t>(B) * 2 * 640 * 4, c->stream));
    B3_CUDA(cudaMemsetAsync(D.ws_keys.p, 0, static_cast<size_t>(B) * 4 * 8, c->stream));
    B3_CUDA(cudaMemsetAsync(D.sync.p, 0, 32, c->stream));
    DecWs p{};
    p.B = B;
    p.vocab = D.vocab;
    p.blank = D.vocab - 1;
    p.max_tokens = max_tokens;
    p.head_tiles = D.ws_ht;
    p.n_roles = D.ws_ht + 3 * kWsLstmTiles + kWsProjTiles;
    p.ntile = ntile;
    p.bpad = bpad;
    // k-blocks per TMA box: the largest divisor of the 10 k-blocks that keeps
    // two ring stages in the 64 KB ring (so no box reaches past the panels)
    p.kc = 1;
    for (int d : {10, 5, 2})
        if (d * 2 * ntile * 128 <= 32768) {
            p.kc = d;
            break;
        }
    p.max_steps = tmax * 14 + 64;
    p.row0 = D.rows.as<int>();
    p.len = D.rows.as<int>() + B;
    p.pooler = pooler;
    p.e0 = D.e0.as<float>();
    p.bias = D.ws_bias.as<float>();
    p.act0 = D.a0.as<__half>();
    p.act1 = D.ap.as<__half>();
    p.aj = D.aj.as<__half>();
    p.c = D.cstate.as<float>();
    p.g1p = D.gates.as<float>();
    p.keys = D.ws_keys.as<unsigned long long>();
    int* ip = D.ints.as<int>();
    p.frame = ip;
    p.count = ip + B;
    p.guard = ip + 2 * B;
    p.alive = ip + 3 * B;   // [0] step-0 parity, [1] the first pass (step -1)
    p.tokens = D.tokens.as<uint32_t>();
    p.sync = D.sync.as<unsigned int>();
    p.grid_wait_ns = c->grid_wait_ns;
    DecWsMaps maps;
    maps.w = D.ws_wmap;
    const uint64_t dims[3] = {64, static_cast<uint64_t>(bpad), 20};
    const uint64_t strides[2] = {128, static_cast<uint64_t>(bpad) * 128};
    const uint32_t box[3] = {64, static_cast<uint32_t>(ntile), static_cast<uint32_t>(2 * p.kc)};
    B3_TRY(make_map_3d(&maps.act0, D.a0.p, kMapF16, dims, strides, box, true));
    B3_TRY(make_map_3d(&maps.act1, D.ap.p, kMapF16, dims, strides, box, true));
    B3_TRY(make_map_3d(&maps.aj, D.aj.p, kMapF16, dims, strides, box, true));
    return dec_ws_launch(maps, p, grid, c->stream);
}

// Greedy-decodes n_utt utterances of a device pooler [total][640] with one
// cooperative launch of the persistent decoder; the tokens and counts are
// left in the decoder's buffers (row b = utterance b).
int decode_device(b3_ctx* c, const float* pooler, const int32_t* cu, int n_utt, int max_tokens) {
    auto& D = c->dec;
    if (!D.present) return set_error(B3_ESTATE, "no decoder weights were loaded");
    if (n_utt <= 0 || max_tokens <= 0) return set_error(B3_EINVAL, "bad decode batch");
    const int B = n_utt;
    std::vector<int32_t> rows(2 * B);
    int tmax = 0;
    for (int b = 0; b < B; ++b) {
        rows[b] = cu[b];
        rows[B + b] = cu[b + 1] - cu[b];
        if (rows[B + b] < 0) return set_error(B3_EINVAL, "cu_seqlens must be non-decreasing");
        tmax = std::max(tmax, rows[B + b]);
    }
    // up to 128 rows: the weight-stationary kernel (two halves of at most 64
    // columns above 64 rows), when its CTAs fit; its epilogues do per-column
    // work, so wider halves run slower than the split-K kernel
    {
        const int n_roles = D.ws_ht + 3 * kWsLstmTiles + kWsProjTiles;
        int nsplit = B <= 64 ? 1 : (B <= 128 ? 2 : 0);
        if (nsplit == 1 && B > 32 && 2 * n_roles <= device_sms()) nsplit = 2;
        const int ws_grid = nsplit ? dec_ws_grid(c->device, n_roles, nsplit) : 0;
        if (ws_grid > 0 && !c->dec_split_k_only) return decode_ws(c, pooler, rows, B, tmax, max_tokens, nsplit, ws_grid);
    }
    const int grid = dec_persistent_grid(c->device);
    if (grid <= 0) return set_error(B3_ECUDA, "the persistent decoder does not fit on this device");
    int bn[4], ks[4];
    dec_plan_persistent(B, D.npad, grid, bn, ks);
    const size_t b = static_cast<size_t>(B);
    const size_t prow = static_cast<size_t>(gemm_split_rows(B));
    B3_TRY(D.a0.ensure(b * 1280 * 2));
    B3_TRY(D.a1.ensure(b * 2560 * 2));
    B3_TRY(D.ap.ensure(b * 1280 * 2));
    B3_TRY(D.aj.ensure(b * 1280 * 2));
    B3_TRY(D.gates.ensure(std::max(ks[kDecLstm0], ks[kDecLstm1]) * prow * 2560 * 4));
    B3_TRY(D.cstate.ensure(b * 2 * 640 * 4));
    B3_TRY(D.dec.ensure(ks[kDecProj] * prow * 640 * 4));
    B3_TRY(D.scores.ensure(ks[kDecHead] * prow * D.npad * 4));
    B3_TRY(D.ints.ensure(b * 6 * 4));
    B3_TRY(D.tokens.ensure(b * static_cast<size_t>(max_tokens) * 12));
    B3_TRY(D.rows.ensure(b * 2 * 4));
    B3_TRY(D.sync.ensure(32));
    ProfScope ps(c, B3_K_DECODER, 0.0, 0.0);
    c->prof.launches[B3_K_DECODER]++;   // init + the persistent kernel
    B3_CUDA(cudaMemcpyAsync(D.rows.p, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice, c->stream));
    B3_CUDA(cudaMemsetAsync(D.sync.p, 0, 32, c->stream));

    DecPersist p{};
    DecState& s = p.s;
    s.B = B;
    s.vocab = D.vocab;
    s.blank = D.vocab - 1;
    s.max_tokens = max_tokens;
    s.row0 = D.rows.as<int>();
    s.len = D.rows.as<int>() + B;
    s.pooler = pooler;
    s.e0 = D.e0.as<float>();
    s.a0 = D.a0.as<__half>();
    s.a1 = D.a1.as<__half>();
    s.ap = D.ap.as<__half>();
    s.aj = D.aj.as<__half>();
    s.gates = D.gates.as<float>();
    s.c = D.cstate.as<float>();
    s.dec = D.dec.as<float>();
    s.scores = D.scores.as<float>();
    s.ld_scores = D.npad;
    s.prow = static_cast<int>(prow);
    s.ks_g0 = ks[kDecLstm0];
    s.ks_g1 = ks[kDecLstm1];
    s.ks_p = ks[kDecProj];
    s.ks_h = ks[kDecHead];
    int* ints = D.ints.as<int>();
    s.frame = ints;
    s.count = ints + B;
    s.guard = ints + 2 * B;
    s.emit = ints + 3 * B;
    s.active = ints + 4 * B;
    s.tok = ints + 5 * B;
    s.tokens = D.tokens.as<uint32_t>();
    const float* bias = D.bias.as<float>();
    const Linear* w[4] = {&D.head, &D.lstm[0], &D.lstm[1], &D.proj};
    __half* acts[4] = {s.aj, s.a0, s.a1, s.ap};
    float* outs[4] = {s.scores, s.gates, s.gates, s.dec};
    const int ldos[4] = {D.npad, 2560, 2560, 640};
    const float* biases[4] = {bias + 5120 + 640, nullptr, bias + 2560, bias + 5120};
    DecMaps maps;
    for (int i = 0; i < 4; ++i) {
        B3_TRY(gemm_make_a_map(&maps.a[i], acts[i], B, w[i]->K, w[i]->K));
        maps.b[i] = w[i]->map_b;
        B3_TRY(make_map_2d(&maps.c[i], outs[i], kMapF32, static_cast<uint64_t>(ldos[i]),
                           static_cast<uint64_t>(ks[i]) * prow, static_cast<uint64_t>(ldos[i]) * 4, 32, 32, true));
        DecGemm& g = p.g[i];
        g.m_tiles = (B + 127) / 128;
        g.bn = bn[i];
        g.n_tiles = w[i]->N / bn[i];
        g.ks = ks[i];
        g.nkb = w[i]->K / 2 / 64 / ks[i];
        g.out = outs[i];
        g.ldo = ldos[i];
        g.bias = biases[i];
    }
    p.sync = D.sync.as<unsigned int>();
    p.max_steps = tmax * 14 + 64;
    p.grid_wait_ns = c->grid_wait_ns;
    B3_TRY(dec_launch_init(s, c->stream));
    return dec_launch_persistent(maps, p, grid, c->stream);
}

// Copies the decoder's tokens / counts out (device or host destination).
int decode_collect(b3_ctx* c, int n_utt, b3_token* tokens, int32_t* counts, int max_tokens, bool dev) {
    auto& D = c->dec;
    const cudaMemcpyKind k = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
    B3_CUDA(cudaMemcpyAsync(tokens, D.tokens.p, static_cast<size_t>(n_utt) * max_tokens * sizeof(b3_token), k,
                            c->stream));
    B3_CUDA(cudaMemcpyAsync(counts, D.ints.as<int>() + n_utt, n_utt * sizeof(int32_t), k, c->stream));
    return 0;
}

// ───────────────────────────── front end ─────────────────────────────

int conv_len_h(int l) { return (l - 1) / 2 + 1; }

// Slaney mel filterbank (norm "slaney", mel scale "slaney"; the published
// librosa / transformers definition the reference's data/mel_filters.f32
// holds): 128 area-normalised triangles over 0..8000 Hz on the 257 bins of a
// 512-point FFT at 16 kHz, computed in double and stored as f32.
void slaney_filterbank(std::vector<float>& fb) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    const double logstep = std::log(6.4) / 27.0;
    auto hz_to_mel = [&](double f) { return f >= min_log_hz ? min_log_mel + std::log(f / min_log_hz) / logstep : f / f_sp; };
    auto mel_to_hz = [&](double m) { return m >= min_log_mel ? min_log_hz * std::exp(logstep * (m - min_log_mel)) : m * f_sp; };
    const int n_mels = 128, n_bins = 257;
    const double mlo = hz_to_mel(0.0), mhi = hz_to_mel(8000.0);
    std::vector<double> pts(n_mels + 2);
    for (int i = 0; i < n_mels + 2; ++i) pts[i] = mel_to_hz(mlo + (mhi - mlo) * i / (n_mels + 1));
    fb.assign(static_cast<size_t>(n_mels) * n_bins, 0.f);
    for (int m = 0; m < n_mels; ++m) {
        const double enorm = 2.0 / (pts[m + 2] - pts[m]);
        for (int k = 0; k < n_bins; ++k) {
            const double f = k * 8000.0 / 256.0;
            const double lower = (f - pts[m]) / (pts[m + 1] - pts[m]);
            const double upper = (pts[m + 2] - f) / (pts[m + 2] - pts[m + 1]);
            const double w = std::max(0.0, std::min(lower, upper));
            fb[static_cast<size_t>(m) * n_bins + k] = static_cast<float>(w * enorm);
        }
    }
}

// Window, twiddles and filterbank, uploaded once per context.
int build_fe_tables(b3_ctx* c) {
    std::vector<float> fb;
    slaney_filterbank(fb);
    // each filter's nonzero span [lo, hi), and the spans packed end to end
    // (fb_off: start of filter m in the packed weights)
    std::vector<int32_t> lo_hi(256, 0), off(129, 0);
    for (int m = 0; m < 128; ++m) {
        int lo = 257, hi = 0;
        for (int k = 0; k < 257; ++k)
            if (fb[m * 257 + k] != 0.f) {
                lo = std::min(lo, k);
                hi = k + 1;
            }
        lo_hi[m] = lo < hi ? lo : 0;
        lo_hi[128 + m] = lo < hi ? hi : 0;
        off[m + 1] = off[m] + (lo_hi[128 + m] - lo_hi[m]);
    }
    // window [512] | twiddle [256][2] | fb [128][257] | fb_lo [128] | fb_hi [128] | fb_off [129]
    // (+ 3 pad) | packed weights [fb_off[128]]
    const size_t pack0 = 1024 + fb.size() + 256 + 132;
    std::vector<float> t(pack0 + off[128], 0.f);
    for (int i = 0; i < 400; ++i)  // symmetric Hann(400) centred in 512 (src/mel.rs:27-36)
        t[56 + i] = 0.5f * (1.0f - cosf(6.2831855f * static_cast<float>(i) / 399.0f));
    for (int k = 0; k < 256; ++k) {
        t[512 + 2 * k] = static_cast<float>(std::cos(-2.0 * M_PI * k / 512.0));
        t[512 + 2 * k + 1] = static_cast<float>(std::sin(-2.0 * M_PI * k / 512.0));
    }
    memcpy(&t[1024], fb.data(), fb.size() * 4);
    memcpy(&t[1024 + fb.size()], lo_hi.data(), 256 * 4);
    memcpy(&t[1024 + fb.size() + 256], off.data(), 129 * 4);
    for (int m = 0; m < 128; ++m)
        for (int k = lo_hi[m]; k < lo_hi[128 + m]; ++k) t[pack0 + off[m] + (k - lo_hi[m])] = fb[m * 257 + k];
    c->fe.fb_packed = off[128];
    B3_TRY(upload(c->fe.tables, t.data(), t.size() * 4, c->stream));
    B3_CUDA(cudaStreamSynchronize(c->stream));
    return 0;
}

// Conv-subsampling weights (SubsamplingWeights, src/sub.rs:56-103) and the
// encoder's subsampling linear with its input columns permuted from
// (channel c, freq m) -> c*16 + m to (m, c) -> m*256 + c, the order the GPU
// front end writes.
int build_frontend(b3_ctx* c) {
    auto& F = c->fe;
    if (!find(c, "encoder.subsampling.layers.0.weight")) return 0;
    const std::string p = "encoder.subsampling.layers.";
    std::vector<float> conv, v;
    for (const char* l : {"0", "2", "5"}) {
        B3_TRY(get_vec(c, p + l + ".weight", 256 * 9, v));
        conv.insert(conv.end(), v.begin(), v.end());
        B3_TRY(get_vec(c, p + l + ".bias", 256, v));
        conv.insert(conv.end(), v.begin(), v.end());
    }
    B3_TRY(upload(F.conv, conv.data(), conv.size() * 4, c->stream));
    std::vector<float> pb;
    for (const char* l : {"3", "6"}) {
        const Staged* s = find(c, p + l + ".weight");
        if (!s) return set_error(B3_ENOTFOUND, "tensor %s.weight was not loaded", (p + l).c_str());
        if (s->lowbit || numel(*s) != 256 * 256) return set_error(B3_EINVAL, "%s.weight must be (256, 256, 1, 1)", (p + l).c_str());
        B3_TRY(build_dense(c, l[0] == '3' ? F.pw1 : F.pw2, s->f16, 256, 256));
        B3_TRY(get_vec(c, p + l + ".bias", 256, v));
        pb.insert(pb.end(), v.begin(), v.end());
    }
    B3_TRY(upload(F.pw_bias, pb.data(), pb.size() * 4, c->stream));
    // permuted subsampling linear
    const Staged* s = find(c, "encoder.subsampling.linear.weight");
    if (!s) return set_error(B3_ENOTFOUND, "tensor encoder.subsampling.linear.weight was not loaded");
    Linear& L = F.sub_w_perm;
    L.present = true;
    L.lut = s->lowbit;
    L.N = kHidden;
    L.K = kSubIn;
    auto src_col = [](int col) { return (col % 256) * 16 + col / 256; };  // new (m, c) -> old c*16 + m
    if (s->lowbit) {
        std::vector<uint8_t> codes(static_cast<size_t>(kHidden) * kSubIn / 2, 0);
        for (int r = 0; r < kHidden; ++r) {
            const uint8_t* old = &s->codes[static_cast<size_t>(r) * kSubIn / 2];
            uint8_t* dst = &codes[static_cast<size_t>(r) * kSubIn / 2];
            for (int col = 0; col < kSubIn; ++col) {
                const int oc = src_col(col);
                const uint8_t code = (oc & 1) ? (old[oc / 2] >> 4) : (old[oc / 2] & 0xF);
                dst[col / 2] |= (col & 1) ? static_cast<uint8_t>(code << 4) : code;
            }
        }
        B3_TRY(upload(L.w, codes.data(), codes.size(), c->stream));
        B3_TRY(upload(L.lut16, s->lut16.data(), s->lut16.size() * 2, c->stream));
    } else {
        std::vector<uint16_t> w(static_cast<size_t>(kHidden) * kSubIn);
        for (int r = 0; r < kHidden; ++r)
            for (int col = 0; col < kSubIn; ++col)
                w[static_cast<size_t>(r) * kSubIn + col] = s->f16[static_cast<size_t>(r) * kSubIn + src_col(col)];
        B3_TRY(upload(L.w, w.data(), w.size() * 2, c->stream));
    }
    B3_CUDA(cudaStreamSynchronize(c->stream));
    B3_TRY(gemm_make_b_map(&L.map_b, L.w.p, L.lut, kHidden, kSubIn));
    F.present = true;
    return 0;
}

void fe_shape_from_frames(FeShape& s, const std::vector<int32_t>& frames, const std::vector<int32_t>& nvalid) {
    const int n = static_cast<int>(frames.size());
    s.foff.assign(n + 1, 0);
    s.x2off.assign(n + 1, 0);
    s.x4off.assign(n + 1, 0);
    s.nvalid = nvalid;
    s.work.clear();
    s.rows3.clear();
    s.woff.assign(n + 1, 0);
    const int rows = sub_work_rows(), groups = 256 / sub_work_channels();
    for (int u = 0; u < n; ++u) {
        const int f2 = conv_len_h(conv_len_h(frames[u]));
        const int t = conv_len_h(f2);
        s.foff[u + 1] = s.foff[u] + frames[u];
        s.x2off[u + 1] = s.x2off[u] + f2;
        s.x4off[u + 1] = s.x4off[u] + t;
        // two int4 per item: (first mel row, mel frames, valid frames, first
        // t2 row), (first x2 row, channel group, 0, 0): every table value the
        // item needs, so the kernel's per-item reads have no dependent chain
        for (int t2 = 0; t2 < f2; t2 += rows)
            for (int g = 0; g < groups; ++g) {
                s.work.push_back(make_int4(s.foff[u], frames[u], nvalid[u], t2));
                s.work.push_back(make_int4(s.x2off[u], g, 0, 0));
            }
        s.woff[u + 1] = static_cast<int32_t>(s.work.size() / 2);
        // the second depthwise conv's rows: every table value a row needs
        const int v3 = conv_len_h(conv_len_h(conv_len_h(nvalid[u] > 1 ? nvalid[u] : 1)));
        for (int t3 = 0; t3 < t; ++t3) s.rows3.push_back(make_int4(s.x2off[u], f2, v3, t3));
    }
}

// mel [frames][128] (device, in c->fe.mel) -> c->sub16 [sum T][4096] in
// (freq, channel) column order.  fe_sub_setup sizes the buffers, uploads the
// batch tables and sets up the encoder plan for the T offsets; fe_sub_run
// subsamples utterances [u0, u1).
int fe_sub_setup(b3_ctx* c, const FeShape& s, SubParams& sp) {
    auto& F = c->fe;
    const int n = static_cast<int>(s.nvalid.size());
    const int rows2 = s.x2off[n], T = s.x4off[n];
    B3_TRY(make_plan(c, s.x4off.data(), n));
    B3_TRY(F.x2.ensure(static_cast<size_t>(rows2) * 32 * 256 * 2 + 16));
    B3_TRY(F.x3.ensure(static_cast<size_t>(rows2) * 32 * 256 * 2 + 16));
    B3_TRY(F.x4.ensure(static_cast<size_t>(T) * 16 * 256 * 2 + 16));
    // the per-batch tables go up once per batch shape
    std::vector<int32_t> key(s.foff);
    key.insert(key.end(), s.nvalid.begin(), s.nvalid.end());
    int32_t* ints = nullptr;
    if (key != F.sub_key) {
        B3_TRY(F.ints.ensure((3 * n + 2) * sizeof(int32_t)));
        B3_TRY(F.work.ensure(s.work.size() * sizeof(int4) + 16));
        B3_TRY(F.rows3.ensure(s.rows3.size() * sizeof(int4) + 16));
        ints = F.ints.as<int32_t>();
        B3_CUDA(cudaMemcpyAsync(ints, s.nvalid.data(), n * 4, cudaMemcpyHostToDevice, c->stream));
        B3_CUDA(cudaMemcpyAsync(ints + n, s.x2off.data(), (n + 1) * 4, cudaMemcpyHostToDevice, c->stream));
        B3_CUDA(cudaMemcpyAsync(ints + 2 * n + 1, s.x4off.data(), (n + 1) * 4, cudaMemcpyHostToDevice, c->stream));
        B3_CUDA(cudaMemcpyAsync(F.work.p, s.work.data(), s.work.size() * sizeof(int4), cudaMemcpyHostToDevice, c->stream));
        B3_CUDA(cudaMemcpyAsync(F.rows3.p, s.rows3.data(), s.rows3.size() * sizeof(int4), cudaMemcpyHostToDevice,
                                c->stream));
        F.sub_key = key;
    }
    ints = F.ints.as<int32_t>();
    sp.n_utt = n;
    sp.mel = F.mel.as<float>();
    sp.mel_off = F.frame_off.as<int>();
    sp.n_valid = ints;
    sp.work = F.work.as<int4>();
    sp.rows3 = F.rows3.as<int4>();
    const float* cv = F.conv.as<float>();
    sp.w0 = cv;
    sp.b0 = cv + 2304;
    sp.w2 = cv + 2560;
    sp.b2 = cv + 4864;
    sp.w5 = cv + 5120;
    sp.b5 = cv + 7424;
    sp.x2 = F.x2.as<__half>();
    sp.x3 = F.x3.as<__half>();
    sp.x4 = F.x4.as<__half>();
    sp.x2_off = ints + n;
    sp.x4_off = ints + 2 * n + 1;
    return 0;
}

int fe_sub_run(b3_ctx* c, const FeShape& s, const SubParams& sp, int u0, int u1) {
    auto& F = c->fe;
    {
        ProfScope ps(c, B3_K_FRONTEND, 0.0, 0.0);
        B3_TRY(launch_sub_conv0_dw1(sp, s.woff[u0], s.woff[u1], c->stream));
    }
    const size_t r2 = static_cast<size_t>(s.x2off[u0]) * 32, n2 = static_cast<size_t>(s.x2off[u1]) * 32 - r2;
    if (n2 > 0) {
        GemmParams p1 = params_f16(F.x3.as<__half>() + r2 * 256, 256);
        p1.bias = F.pw_bias.as<float>();
        B3_TRY(run_gemm(c, F.pw1, F.x2.as<__half>() + r2 * 256, static_cast<int>(n2), 256, EPI_RELU_F16, p1));
    }
    {
        ProfScope ps(c, B3_K_FRONTEND, 0.0, 0.0);
        B3_TRY(launch_sub_dw2(sp, s.x4off[u0], s.x4off[u1], c->stream));
    }
    const size_t r4 = static_cast<size_t>(s.x4off[u0]) * 16, n4 = static_cast<size_t>(s.x4off[u1]) * 16 - r4;
    if (n4 == 0) return 0;
    GemmParams p2 = params_f16(c->sub16.as<__half>() + r4 * 256, 256);
    p2.bias = F.pw_bias.as<float>() + 256;
    return run_gemm(c, F.pw2, F.x4.as<__half>() + r4 * 256, static_cast<int>(n4), 256, EPI_RELU_F16, p2);
}

int fe_subsample(b3_ctx* c, const FeShape& s) {
    SubParams sp;
    B3_TRY(fe_sub_setup(c, s, sp));
    return fe_sub_run(c, s, sp, 0, static_cast<int>(s.nvalid.size()));
}

// Padded waves (device, concatenated at woff) -> c->fe.mel: fe_mel_setup
// fills s, uploads the batch's offset tables (once per shape) and the kernel
// parameters; fe_mel_run computes a range of utterances.
int fe_mel_setup(b3_ctx* c, const float* wave, const std::vector<int64_t>& woff, int lead, FeShape& s,
                 MelParams& mp) {
    auto& F = c->fe;
    const int n = static_cast<int>(woff.size()) - 1;
    std::vector<int64_t> key(woff);
    key.push_back(lead);
    if (key == F.mel_key) {
        s = F.mel_shape;  // same batch shape as the previous call: tables are on the device
    } else {
        std::vector<int32_t> frames(n), nvalid(n);
        for (int u = 0; u < n; ++u) {
            const int64_t len = woff[u + 1] - woff[u] + lead;
            if (len < lead) return set_error(B3_EINVAL, "sample offsets must be non-decreasing");
            frames[u] = static_cast<int32_t>(1 + len / 160);
            nvalid[u] = static_cast<int32_t>(len / 160);
        }
        fe_shape_from_frames(s, frames, nvalid);
        B3_TRY(F.wave_off.ensure((n + 1) * 8));
        B3_TRY(F.frame_off.ensure((n + 1) * 4));
        B3_TRY(F.mel.ensure(static_cast<size_t>(s.foff[n]) * 128 * 4 + 16));
        B3_CUDA(cudaMemcpyAsync(F.wave_off.p, woff.data(), (n + 1) * 8, cudaMemcpyHostToDevice, c->stream));
        B3_CUDA(cudaMemcpyAsync(F.frame_off.p, s.foff.data(), (n + 1) * 4, cudaMemcpyHostToDevice, c->stream));
        F.mel_key = key;
        F.mel_shape = s;
    }
    const float* t = F.tables.as<float>();
    mp.n_utt = n;
    mp.lead = lead;
    mp.wave = wave;
    mp.wave_off = F.wave_off.as<int64_t>();
    mp.frame_off = F.frame_off.as<int>();
    mp.window = t;
    mp.twiddle = reinterpret_cast<const float2*>(t + 512);
    mp.fb = t + 1024;
    mp.fb_lo = reinterpret_cast<const int*>(t + 1024 + 128 * 257);
    mp.fb_hi = mp.fb_lo + 128;
    mp.fb_off = mp.fb_hi + 128;
    mp.fb_pack = t + 1024 + 128 * 257 + 256 + 132;
    mp.fb_total = F.fb_packed;
    mp.mel = F.mel.as<float>();
    return 0;
}

// Mel of utterances [u0, u1) (frames and per-utterance normalisation).
int fe_mel_run(b3_ctx* c, const FeShape& s, const MelParams& mp, int u0, int u1) {
    const int f0 = s.foff[u0], f1 = s.foff[u1];
    ProfScope ps(c, B3_K_FRONTEND, 0.0, (f1 - f0) * (160.0 * 4 + 512.0));
    return launch_mel(mp, f0, f1, u0, u1, c->stream);
}

int fe_mel(b3_ctx* c, const float* wave, const std::vector<int64_t>& woff, FeShape& s) {
    MelParams mp;
    B3_TRY(fe_mel_setup(c, wave, woff, 0, s, mp));
    return fe_mel_run(c, s, mp, 0, static_cast<int>(woff.size()) - 1);
}

// The whole front end of an audio batch (device waves at woff, each
// utterance behind the reference's 0.25 s of silence -> c->sub16), chunk by
// chunk: with host input each chunk starts as soon as its own waves are on the
// device, so the upload of later chunks overlaps the mel and subsampling of
// earlier ones.  max_rows < 0: no limit on the subsampled rows; else a batch
// with more rows is an error before any launch.
int fe_front(b3_ctx* c, const float* wave, const std::vector<int64_t>& woff, FeShape& s, int64_t max_rows) {
    auto& F = c->fe;
    const int n = static_cast<int>(woff.size()) - 1;
    MelParams mp;
    B3_TRY(fe_mel_setup(c, wave, woff, kLeadSamples, s, mp));
    if (max_rows >= 0 && s.x4off[n] > max_rows)
        return set_error(B3_EINVAL, "pooler needs %d rows, capacity is %lld", s.x4off[n], static_cast<long long>(max_rows));
    SubParams sp;
    B3_TRY(fe_sub_setup(c, s, sp));
    const bool chunked = F.chunk_wait && F.chunk_u.size() >= 2 && F.chunk_u.back() == n;
    const std::vector<int> one = {0, n};
    const std::vector<int>& cu = chunked ? F.chunk_u : one;
    for (size_t k = 0; k + 1 < cu.size(); ++k) {
        if (chunked) B3_CUDA(cudaStreamWaitEvent(c->stream, F.chunk_ev[k], 0));
        B3_TRY(fe_mel_run(c, s, mp, cu[k], cu[k + 1]));
        B3_TRY(fe_sub_run(c, s, sp, cu[k], cu[k + 1]));
    }
    F.chunk_wait = false;
    return 0;
}

// Samples (host or device, one utterance per offset range) for the audio
// front end.  Device samples are read where they are.  Host samples go up
// into c->fe.wave (same offsets) in up to kChunks chunks, one copy each, on
// the front end's copy stream, which first waits for every earlier use of that
// buffer; fe_front waits for each chunk only.  The first chunk is small (1/32
// of the samples) so the front end starts early; the front end then consumes
// samples more slowly than the copies deliver them.  The
// reference's 0.25 s of leading silence (src/transcription.rs:48-52) is never
// stored: the mel reads it as zeros.
int fe_upload(b3_ctx* c, const float* samples, const int64_t* off, int n, bool dev, std::vector<int64_t>& woff,
              const float** wave) {
    auto& F = c->fe;
    woff.assign(off, off + n + 1);
    for (int u = 0; u < n; ++u)
        if (off[u + 1] < off[u]) return set_error(B3_EINVAL, "sample offsets must be non-decreasing");
    F.chunk_wait = false;
    if (dev) {
        *wave = samples;
        return 0;
    }
    B3_TRY(F.wave.ensure(static_cast<size_t>(off[n]) * 4 + 16));
    float* w = F.wave.as<float>();
    *wave = w;
    constexpr int kChunks = 8;
    if (!F.copy_st) B3_CUDA(cudaStreamCreateWithFlags(&F.copy_st, cudaStreamNonBlocking));
    if (!F.wave_free) B3_CUDA(cudaEventCreateWithFlags(&F.wave_free, cudaEventDisableTiming));
    while (F.chunk_ev.size() < static_cast<size_t>(kChunks)) {
        cudaEvent_t e;
        B3_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        F.chunk_ev.push_back(e);
    }
    B3_CUDA(cudaEventRecord(F.wave_free, c->stream));
    B3_CUDA(cudaStreamWaitEvent(F.copy_st, F.wave_free, 0));
    F.chunk_u.assign(1, 0);
    const int64_t total = off[n];
    // cumulative sample fractions (in 32nds) at which chunks 0 .. kChunks-2 end
    static constexpr int kEnd32[kChunks - 1] = {1, 4, 8, 12, 16, 20, 24};
    for (int u = 0; u < n; ++u) {
        const int k = static_cast<int>(F.chunk_u.size()) - 1;
        if (u + 1 == n || (k + 1 < kChunks && off[u + 1] * 32 >= total * kEnd32[k])) {
            const int64_t a = off[F.chunk_u.back()], b = off[u + 1];
            if (b > a)
                B3_CUDA(cudaMemcpyAsync(w + a, samples + a, static_cast<size_t>(b - a) * 4, cudaMemcpyHostToDevice,
                                        F.copy_st));
            B3_CUDA(cudaEventRecord(F.chunk_ev[k], F.copy_st));
            F.chunk_u.push_back(u + 1);
        }
    }
    F.chunk_wait = true;
    return 0;
}

// Single linear (configs 1 / lbtest): c = a . W^T (+ bias), W given per call.
int linear_any(b3_ctx* c, const float* a, const void* w, const uint16_t* lut16, bool lut,
               const float* bias, float* out, int m, int n, int k, unsigned flags) {
    if (!c) return set_error(B3_EINVAL, "null context");
    if (!a || !w || !out || (lut && !lut16)) return set_error(B3_EINVAL, "null buffer");
    if (m <= 0 || n <= 0 || k <= 0 || k % 64 || n % 128)
        return set_error(B3_EINVAL, "linear shape m=%d n=%d k=%d (need k %% 64 == 0, n %% 128 == 0)", m, n, k);
    DeviceGuard g(c->device);
    const bool dev = flags & B3_DEVICE_PTRS;
    const size_t a_bytes = static_cast<size_t>(m) * k * 4;
    const size_t w_bytes = lut ? static_cast<size_t>(n) * k / 2 : static_cast<size_t>(n) * k * 2;
    const size_t lut_bytes = lut ? static_cast<size_t>(n) * 32 : 0;
    const size_t bias_bytes = bias ? static_cast<size_t>(n) * 4 : 0;
    const size_t c_bytes = static_cast<size_t>(m) * n * 4;
    const float* da = a;
    const void* dw = w;
    const uint16_t* dl = lut16;
    const float* db = bias;
    float* dc = out;
    if (!dev) {
        // one staging block: a | w | lut | bias | c (each 256-byte aligned)
        auto al = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
        const size_t total = al(a_bytes) + al(w_bytes) + al(lut_bytes) + al(bias_bytes) + al(c_bytes);
        B3_TRY(c->io_in.ensure(total));
        char* base = c->io_in.as<char>();
        size_t off = 0;
        auto put = [&](const void* src, size_t bytes) -> char* {
            char* d = base + off;
            off += al(bytes);
            if (src && bytes) cudaMemcpyAsync(d, src, bytes, cudaMemcpyHostToDevice, c->stream);
            return d;
        };
        da = reinterpret_cast<const float*>(put(a, a_bytes));
        dw = put(w, w_bytes);
        dl = lut ? reinterpret_cast<const uint16_t*>(put(lut16, lut_bytes)) : nullptr;
        db = bias ? reinterpret_cast<const float*>(put(bias, bias_bytes)) : nullptr;
        dc = reinterpret_cast<float*>(put(nullptr, c_bytes));
    }
    B3_TRY(c->scratch16.ensure(static_cast<size_t>(m) * k * 2));
    B3_TRY(k_convert(c, da, c->scratch16.as<__half>(), static_cast<int64_t>(m) * k));
    GemmOp op;
    B3_TRY(gemm_make_a_map(&op.map_a, c->scratch16.as<__half>(), m, k, k));
    B3_TRY(gemm_make_b_map(&op.map_b, dw, lut, n, k));
    op.p = params_f32(dc, n, db);
    op.p.M = m;
    op.p.N = n;
    op.p.K = k;
    op.p.lut = dl;
    op.lut = lut;
    op.epi = EPI_F32;
    {
        ProfScope ps(c, lut ? B3_K_GEMM_LUT4 : B3_K_GEMM_F16, 2.0 * m * n * k, gemm_bytes(m, n, k, lut, EPI_F32));
        B3_TRY(gemm_launch(op, c->stream));
    }
    if (dev) return 0;
    B3_CUDA(cudaMemcpyAsync(out, dc, c_bytes, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

}  // namespace

// ───────────────────────────── C ABI ─────────────────────────────

extern "C" {

const char* b3_last_error(void) { return b3::g_last_error; }

int b3_version(void) { return 100; }

b3_ctx* b3_create(int device) {
    clear_error();
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || device < 0 || device >= n) {
        set_error(B3_ECUDA, "no CUDA device %d (%s)", device, cudaGetErrorString(e));
        return nullptr;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) {
        set_error(B3_ECUDA, "device %d is not an sm_100 (Blackwell B200) GPU", device);
        return nullptr;
    }
    DeviceGuard g(device);
    b3_ctx* c = new (std::nothrow) b3_ctx();
    if (!c) {
        set_error(B3_ENOMEM, "out of host memory");
        return nullptr;
    }
    c->device = device;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_error(B3_ECUDA, "cudaStreamCreate failed");
        delete c;
        return nullptr;
    }
    // inverse frequencies exactly as src/encoder.rs:231-234 computes them (f32)
    float inv[512];
    for (int i = 0; i < 512; ++i) inv[i] = 1.0f / powf(10000.0f, (2.0f * static_cast<float>(i)) / 1024.0f);
    if (upload(c->inv_freq, inv, sizeof(inv), c->stream) || cudaStreamSynchronize(c->stream) != cudaSuccess ||
        build_fe_tables(c)) {
        delete c;
        return nullptr;
    }
    return c;
}

void b3_destroy(b3_ctx* ctx) {
    if (!ctx) return;
    DeviceGuard g(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    delete ctx;
}

int b3_sync(b3_ctx* ctx) {
    if (!ctx) return set_error(B3_EINVAL, "null context");
    DeviceGuard g(ctx->device);
    return sync_and_check(ctx);
}

void* b3_stream(b3_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int b3_set_decoder(b3_ctx* ctx, int kind) {
    if (!ctx) return set_error(B3_EINVAL, "null context");
    if (kind != B3_DECODER_AUTO && kind != B3_DECODER_SPLIT_K) return set_error(B3_EINVAL, "unknown decoder kind %d", kind);
    ctx->dec_split_k_only = kind == B3_DECODER_SPLIT_K;
    return 0;
}

int b3_set_wait_limit(b3_ctx* ctx, int64_t grid_barrier_ns) {
    if (!ctx) return set_error(B3_EINVAL, "null context");
    ctx->grid_wait_ns = grid_barrier_ns > 0 ? static_cast<uint64_t>(grid_barrier_ns) : kDefaultWaitNs;
    return 0;
}

int b3_load_tensor(b3_ctx* ctx, const char* name, int dtype, const int64_t* shape, int ndim,
                   const void* data) {
    if (!ctx || !name || !data || (ndim > 0 && !shape) || ndim < 0 || ndim > 8)
        return set_error(B3_EINVAL, "b3_load_tensor: bad arguments");
    if (ctx->finalized) return set_error(B3_ESTATE, "weights are already finalized");
    Staged s;
    s.shape.assign(shape, shape + ndim);
    int64_t n = 1;
    for (int i = 0; i < ndim; ++i) {
        if (shape[i] < 0) return set_error(B3_EINVAL, "%s: negative dimension", name);
        n *= shape[i];
    }
    s.f32.resize(n);
    s.f16.resize(n);
    for (int64_t i = 0; i < n; ++i) {
        float v;
        switch (dtype) {
            case B3_DTYPE_F32: v = static_cast<const float*>(data)[i]; break;
            case B3_DTYPE_F16: v = f16_bits_to_f32(static_cast<const uint16_t*>(data)[i]); break;
            case B3_DTYPE_BF16: v = bf16_bits_to_f32(static_cast<const uint16_t*>(data)[i]); break;
            default: return set_error(B3_EINVAL, "%s: unknown dtype %d", name, dtype);
        }
        s.f32[i] = v;
        s.f16[i] = dtype == B3_DTYPE_F16 ? static_cast<const uint16_t*>(data)[i] : f32_to_f16_bits(v);
    }
    ctx->staged[name] = std::move(s);
    return 0;
}

int b3_load_lowbit(b3_ctx* ctx, const char* name, const uint8_t* codes, const uint16_t* lut16, int rows,
                   int cols) {
    if (!ctx || !name || !codes || !lut16 || rows <= 0 || cols <= 0 || (cols & 1))
        return set_error(B3_EINVAL, "b3_load_lowbit: bad arguments");
    if (ctx->finalized) return set_error(B3_ESTATE, "weights are already finalized");
    Staged s;
    s.lowbit = true;
    s.rows = rows;
    s.cols = cols;
    s.shape = {rows, cols};
    s.codes.assign(codes, codes + static_cast<size_t>(rows) * cols / 2);
    s.lut16.assign(lut16, lut16 + static_cast<size_t>(rows) * 16);
    ctx->staged[name] = std::move(s);
    return 0;
}

int b3_load_lowbit_levels(b3_ctx* ctx, const char* name, const uint32_t* code_words, const uint16_t* levels,
                          int k, int rows, int cols) {
    if (!ctx || !name || !code_words || !levels || rows <= 0 || cols <= 0 || (cols & 1))
        return set_error(B3_EINVAL, "b3_load_lowbit_levels: bad arguments");
    if (k < 1 || k > 3) return set_error(B3_EINVAL, "%s: unsupported level count %d", name, k);
    const int ld = (cols + 7) / 8;
    std::vector<uint8_t> codes(static_cast<size_t>(rows) * cols / 2);
    std::vector<uint16_t> tab(static_cast<size_t>(rows) * 16, 0);
    for (int r = 0; r < rows; ++r) {
        const uint8_t* wb = reinterpret_cast<const uint8_t*>(code_words + static_cast<size_t>(r) * ld);
        memcpy(&codes[static_cast<size_t>(r) * cols / 2], wb, cols / 2);
        const uint16_t* lev = levels + static_cast<size_t>(r) * 4;
        for (int code = 1; code <= 2 * k; ++code) {
            const bool neg = code > k;
            const uint16_t mag = lev[neg ? code - k - 1 : code - 1];
            tab[static_cast<size_t>(r) * 16 + code] = neg ? static_cast<uint16_t>(mag ^ 0x8000u) : mag;
        }
    }
    return b3_load_lowbit(ctx, name, codes.data(), tab.data(), rows, cols);
}

int b3_finalize(b3_ctx* ctx, int n_layers) {
    if (!ctx) return set_error(B3_EINVAL, "null context");
    if (ctx->finalized) return set_error(B3_ESTATE, "already finalized");
    if (n_layers < 1 || n_layers > 64) return set_error(B3_EINVAL, "n_layers %d out of range", n_layers);
    DeviceGuard g(ctx->device);
    std::vector<float> v;
    B3_TRY(build_linear(ctx, ctx->sub_w, {"encoder.subsampling.linear.weight"}, kHidden, kSubIn, false));
    B3_TRY(get_vec(ctx, "encoder.subsampling.linear.bias", kHidden, v));
    B3_TRY(upload(ctx->sub_b, v.data(), v.size() * 4, ctx->stream));
    B3_TRY(build_linear(ctx, ctx->proj_w, {"encoder_projector.weight"}, kProj, kHidden, false));
    B3_TRY(get_vec(ctx, "encoder_projector.bias", kProj, v));
    B3_TRY(upload(ctx->proj_b, v.data(), v.size() * 4, ctx->stream));
    ctx->layers.resize(n_layers);
    for (int l = 0; l < n_layers; ++l) {
        Layer& L = ctx->layers[l];
        const std::string p = "encoder.layers." + std::to_string(l) + ".";
        B3_TRY(build_linear(ctx, L.qkv, {p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                                         p + "self_attn.v_proj.weight"}, kHidden, kHidden, false));
        B3_TRY(build_linear(ctx, L.relk, {p + "self_attn.relative_k_proj.weight"}, kHidden, kHidden, false));
        B3_TRY(build_linear(ctx, L.o, {p + "self_attn.o_proj.weight"}, kHidden, kHidden, false));
        B3_TRY(build_linear(ctx, L.ff1a, {p + "feed_forward1.linear1.weight"}, kFfn, kHidden, false));
        B3_TRY(build_linear(ctx, L.ff1b, {p + "feed_forward1.linear2.weight"}, kHidden, kFfn, false));
        B3_TRY(build_linear(ctx, L.ff2a, {p + "feed_forward2.linear1.weight"}, kFfn, kHidden, false));
        B3_TRY(build_linear(ctx, L.ff2b, {p + "feed_forward2.linear2.weight"}, kHidden, kFfn, false));
        B3_TRY(build_linear(ctx, L.pw1, {p + "conv.pointwise_conv1.weight"}, 2 * kHidden, kHidden, true));
        B3_TRY(build_linear(ctx, L.pw2, {p + "conv.pointwise_conv2.weight"}, kHidden, kHidden, false));
        std::vector<float> prm(Layer::kParamFloats, 0.f);
        // depthwise taps rounded through f16 like every other weight
        // (src/cpu/mod.rs:101), stored tap-major for coalesced loads
        B3_TRY(get_vec(ctx, p + "conv.depthwise_conv.weight", kHidden * 9, v));
        for (int c = 0; c < kHidden; ++c)
            for (int i = 0; i < 9; ++i) prm[i * kHidden + c] = f16_bits_to_f32(f32_to_f16_bits(v[c * 9 + i]));
        std::vector<float> gam, bet, mu, var;
        B3_TRY(get_vec(ctx, p + "conv.norm.weight", kHidden, gam));
        B3_TRY(get_vec(ctx, p + "conv.norm.bias", kHidden, bet));
        B3_TRY(get_vec(ctx, p + "conv.norm.running_mean", kHidden, mu));
        B3_TRY(get_vec(ctx, p + "conv.norm.running_var", kHidden, var));
        for (int c = 0; c < kHidden; ++c) {  // BN fold, src/cpu/mod.rs:113-119
            const float a = gam[c] / sqrtf(var[c] + 1e-5f);
            prm[9 * kHidden + c] = a;
            prm[10 * kHidden + c] = bet[c] - mu[c] * a;
        }
        const char* norms[5] = {"norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out"};
        for (int i = 0; i < 5; ++i) {
            B3_TRY(get_vec(ctx, p + norms[i] + ".weight", kHidden, v));
            memcpy(&prm[(11 + i) * kHidden], v.data(), kHidden * 4);
            B3_TRY(get_vec(ctx, p + norms[i] + ".bias", kHidden, v));
            memcpy(&prm[(16 + i) * kHidden], v.data(), kHidden * 4);
        }
        B3_TRY(get_vec(ctx, p + "self_attn.bias_u", kHidden, v));
        memcpy(&prm[21 * kHidden], v.data(), kHidden * 4);
        B3_TRY(get_vec(ctx, p + "self_attn.bias_v", kHidden, v));
        memcpy(&prm[22 * kHidden], v.data(), kHidden * 4);
        B3_TRY(upload(L.params, prm.data(), prm.size() * 4, ctx->stream));
        B3_CUDA(cudaStreamSynchronize(ctx->stream));
    }
    B3_TRY(build_decoder(ctx));
    B3_TRY(build_frontend(ctx));
    ctx->n_layers = n_layers;
    ctx->finalized = true;
    ++ctx->plan_gen;
    ctx->staged.clear();
    return 0;
}

int b3_decode_batch(b3_ctx* ctx, const float* pooler, const int32_t* cu_seqlens, int n_utt, b3_token* tokens,
                    int32_t* counts, int max_tokens, unsigned flags) {
    B3_TRY(check_finalized(ctx));
    if (!pooler || !cu_seqlens || !tokens || !counts) return set_error(B3_EINVAL, "null buffer");
    if (n_utt <= 0 || cu_seqlens[0] != 0) return set_error(B3_EINVAL, "bad cu_seqlens");
    DeviceGuard g(ctx->device);
    const bool dev = flags & B3_DEVICE_PTRS;
    const float* p = pooler;
    // the decoder reads pooler rows as float4: host buffers and unaligned
    // device buffers go through the context's own copy
    if (!dev || (reinterpret_cast<uintptr_t>(pooler) & 15)) {
        const size_t bytes = static_cast<size_t>(cu_seqlens[n_utt]) * 640 * 4;
        B3_TRY(ctx->dec.pooler.ensure(bytes > 0 ? bytes : 4));
        B3_CUDA(cudaMemcpyAsync(ctx->dec.pooler.p, pooler, bytes, dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                ctx->stream));
        p = ctx->dec.pooler.as<float>();
    }
    B3_TRY(decode_device(ctx, p, cu_seqlens, n_utt, max_tokens));
    B3_TRY(decode_collect(ctx, n_utt, tokens, counts, max_tokens, dev));
    return dev ? 0 : sync_and_check(ctx);
}

int b3_transcribe_batch(b3_ctx* ctx, const float* sub, const int32_t* cu_seqlens, int n_utt, b3_token* tokens,
                        int32_t* counts, int max_tokens, unsigned flags) {
    B3_TRY(check_finalized(ctx));
    if (!ctx->dec.present) return set_error(B3_ESTATE, "no decoder weights were loaded");
    if (!sub || !cu_seqlens || !tokens || !counts) return set_error(B3_EINVAL, "null buffer");
    DeviceGuard g(ctx->device);
    B3_TRY(make_plan(ctx, cu_seqlens, n_utt));
    const int M = ctx->plan.M;
    const bool dev = flags & B3_DEVICE_PTRS;
    B3_TRY(ctx->dec.pooler.ensure(static_cast<size_t>(M) * 640 * 4));
    const float* in = sub;
    if (!dev) {
        const size_t in_bytes = static_cast<size_t>(M) * kSubIn * 4;
        B3_TRY(ctx->io_in.ensure(in_bytes));
        B3_CUDA(cudaMemcpyAsync(ctx->io_in.p, sub, in_bytes, cudaMemcpyHostToDevice, ctx->stream));
        in = ctx->io_in.as<float>();
    }
    B3_TRY(encode_device(ctx, in, M, ctx->n_layers, ctx->dec.pooler.as<float>()));
    B3_TRY(decode_device(ctx, ctx->dec.pooler.as<float>(), cu_seqlens, n_utt, max_tokens));
    B3_TRY(decode_collect(ctx, n_utt, tokens, counts, max_tokens, dev));
    return dev ? 0 : sync_and_check(ctx);
}

int b3_mel_filters(float* out) {
    if (!out) return set_error(B3_EINVAL, "null buffer");
    std::vector<float> fb;
    slaney_filterbank(fb);
    memcpy(out, fb.data(), fb.size() * 4);
    return 0;
}

int b3_mel(b3_ctx* ctx, const float* wave, const int64_t* offsets, int n_utt, float* mel, int32_t* frame_offsets,
           unsigned flags) {
    if (!ctx) return set_error(B3_EINVAL, "null context");
    if (!wave || !offsets || !mel || !frame_offsets || n_utt <= 0) return set_error(B3_EINVAL, "bad arguments");
    if (offsets[0] != 0) return set_error(B3_EINVAL, "offsets[0] must be 0");
    DeviceGuard g(ctx->device);
    const bool dev = flags & B3_DEVICE_PTRS;
    std::vector<int64_t> woff(offsets, offsets + n_utt + 1);
    const float* w = wave;
    if (!dev) {
        B3_TRY(ctx->fe.wave.ensure(static_cast<size_t>(woff[n_utt]) * 4 + 16));
        B3_CUDA(cudaMemcpyAsync(ctx->fe.wave.p, wave, static_cast<size_t>(woff[n_utt]) * 4, cudaMemcpyHostToDevice, ctx->stream));
        w = ctx->fe.wave.as<float>();
    }
    FeShape s;
    B3_TRY(fe_mel(ctx, w, woff, s));
    memcpy(frame_offsets, s.foff.data(), (n_utt + 1) * 4);
    B3_CUDA(cudaMemcpyAsync(mel, ctx->fe.mel.p, static_cast<size_t>(s.foff[n_utt]) * 128 * 4,
                            dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, ctx->stream));
    return dev ? 0 : sync_and_check(ctx);
}

int b3_subsample(b3_ctx* ctx, const float* mel, const int32_t* frame_offsets, const int32_t* n_valid, int n_utt,
                 float* sub, int32_t* row_offsets, unsigned flags) {
    B3_TRY(check_finalized(ctx));
    if (!ctx->fe.present) return set_error(B3_ESTATE, "no conv subsampling weights were loaded");
    if (!mel || !frame_offsets || !n_valid || !sub || !row_offsets || n_utt <= 0)
        return set_error(B3_EINVAL, "bad arguments");
    DeviceGuard g(ctx->device);
    const bool dev = flags & B3_DEVICE_PTRS;
    std::vector<int32_t> frames(n_utt), nv(n_valid, n_valid + n_utt);
    for (int u = 0; u < n_utt; ++u) {
        frames[u] = frame_offsets[u + 1] - frame_offsets[u];
        if (frames[u] <= 0) return set_error(B3_EINVAL, "utterance %d has no frames", u);
    }
    FeShape s;
    fe_shape_from_frames(s, frames, nv);
    auto& F = ctx->fe;
    F.mel_key.clear();  // frame_off is rewritten below: the cached mel shape is stale
    const int nf = s.foff[n_utt];
    B3_TRY(F.frame_off.ensure((n_utt + 1) * 4));
    B3_TRY(F.mel.ensure(static_cast<size_t>(nf) * 128 * 4 + 16));
    B3_CUDA(cudaMemcpyAsync(F.frame_off.p, s.foff.data(), (n_utt + 1) * 4, cudaMemcpyHostToDevice, ctx->stream));
    B3_CUDA(cudaMemcpyAsync(F.mel.p, mel, static_cast<size_t>(nf) * 128 * 4,
                            dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream));
    B3_TRY(fe_subsample(ctx, s));
    const int T = s.x4off[n_utt];
    memcpy(row_offsets, s.x4off.data(), (n_utt + 1) * 4);
    float* out = sub;
    if (!dev) {
        B3_TRY(ctx->io_out.ensure(static_cast<size_t>(T) * 4096 * 4));
        out = ctx->io_out.as<float>();
    }
    B3_TRY(launch_sub_to_ref(ctx->sub16.as<__half>(), out, T, ctx->stream));
    if (dev) return 0;
    B3_CUDA(cudaMemcpyAsync(sub, out, static_cast<size_t>(T) * 4096 * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return sync_and_check(ctx);
}

int b3_transcribe_audio(b3_ctx* ctx, const float* samples, const int64_t* offsets, int n_utt, b3_token* tokens,
                        int32_t* counts, int max_tokens, unsigned flags) {
    B3_TRY(check_finalized(ctx));
    if (!ctx->fe.present) return set_error(B3_ESTATE, "no conv subsampling weights were loaded");
    if (!ctx->dec.present) return set_error(B3_ESTATE, "no decoder weights were loaded");
    if (!samples || !offsets || !tokens || !counts || n_utt <= 0) return set_error(B3_EINVAL, "bad arguments");
    if (offsets[0] != 0) return set_error(B3_EINVAL, "offsets[0] must be 0");
    DeviceGuard g(ctx->device);
    const bool dev = flags & B3_DEVICE_PTRS;
    std::vector<int64_t> woff;
    const float* wave = nullptr;
    B3_TRY(fe_upload(ctx, samples, offsets, n_utt, dev, woff, &wave));
    FeShape s;
    B3_TRY(fe_front(ctx, wave, woff, s, -1));
    const int M = s.x4off[n_utt];
    B3_TRY(forward_blocks(ctx, M, ctx->n_layers, &ctx->fe.sub_w_perm));
    B3_TRY(ctx->dec.pooler.ensure(static_cast<size_t>(M) * 640 * 4));
    B3_TRY(run_gemm(ctx, ctx->proj_w, ctx->a16.as<__half>(), M, kHidden, EPI_F32,
                    params_f32(ctx->dec.pooler.as<float>(), kProj, ctx->proj_b.as<float>())));
    B3_TRY(decode_device(ctx, ctx->dec.pooler.as<float>(), s.x4off.data(), n_utt, max_tokens));
    B3_TRY(decode_collect(ctx, n_utt, tokens, counts, max_tokens, dev));
    return dev ? 0 : sync_and_check(ctx);
}

int b3_encode_audio(b3_ctx* ctx, const float* samples, const int64_t* offsets, int n_utt, float* pooler,
                    int32_t* row_offsets, int64_t max_rows, unsigned flags) {
    B3_TRY(check_finalized(ctx));
    if (!ctx->fe.present) return set_error(B3_ESTATE, "no conv subsampling weights were loaded");
    if (ctx->n_layers <= 0) return set_error(B3_ESTATE, "no encoder layers were loaded");
    if (!samples || !offsets || !pooler || !row_offsets || n_utt <= 0) return set_error(B3_EINVAL, "bad arguments");
    if (offsets[0] != 0) return set_error(B3_EINVAL, "offsets[0] must be 0");
    DeviceGuard g(ctx->device);
    const bool dev = flags & B3_DEVICE_PTRS;
    std::vector<int64_t> woff;
    const float* wave = nullptr;
    B3_TRY(fe_upload(ctx, samples, offsets, n_utt, dev, woff, &wave));
    FeShape s;
    B3_TRY(fe_front(ctx, wave, woff, s, max_rows));
    const int M = s.x4off[n_utt];
    B3_TRY(forward_blocks(ctx, M, ctx->n_layers, &ctx->fe.sub_w_perm));
    float* dst = dev ? pooler : nullptr;
    if (!dev) {
        B3_TRY(ctx->dec.pooler.ensure(static_cast<size_t>(M) * kProj * 4 + 16));
        dst = ctx->dec.pooler.as<float>();
    }
    B3_TRY(run_gemm(ctx, ctx->proj_w, ctx->a16.as<__half>(), M, kHidden, EPI_F32,
                    params_f32(dst, kProj, ctx->proj_b.as<float>())));
    if (!dev)
        B3_CUDA(cudaMemcpyAsync(pooler, dst, static_cast<size_t>(M) * kProj * 4, cudaMemcpyDeviceToHost, ctx->stream));
    memcpy(row_offsets, s.x4off.data(), (n_utt + 1) * sizeof(int32_t));
    return dev ? 0 : sync_and_check(ctx);
}

int b3_shard_lpt(const int32_t* frames, int n_utt, int n_ranks, int32_t* rank_of) {
    if (!frames || !rank_of || n_utt < 0 || n_ranks <= 0) return set_error(B3_EINVAL, "b3_shard_lpt: bad arguments");
    std::vector<int> order(n_utt);
    std::vector<double> cost(n_utt);
    for (int i = 0; i < n_utt; ++i) {
        if (frames[i] <= 0) return set_error(B3_EINVAL, "utterance %d has %d frames", i, frames[i]);
        const double t = frames[i];
        cost[i] = 52.4e6 * t + 6144.0 * t * t;
        order[i] = i;
    }
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
    std::vector<double> load(n_ranks, 0.0);
    for (int i : order) {
        int best = 0;
        for (int r = 1; r < n_ranks; ++r)
            if (load[r] < load[best]) best = r;
        rank_of[i] = best;
        load[best] += cost[i];
    }
    return 0;
}

int b3_profile(b3_ctx* ctx, int enable) {
    if (!ctx) return set_error(B3_EINVAL, "null context");
    DeviceGuard g(ctx->device);
    Prof& p = ctx->prof;
    B3_CUDA(cudaStreamSynchronize(ctx->stream));
    if (enable && p.pool.empty()) {
        p.pool.resize(1 << 17);
        for (auto& e : p.pool) B3_CUDA(cudaEventCreate(&e));
    }
    p.on = enable != 0;
    p.recs.clear();
    p.next = 0;
    for (int k = 0; k < B3_K_COUNT; ++k) {
        p.launches[k] = p.timed[k] = 0;
        p.ms[k] = p.flops[k] = p.bytes[k] = 0.0;
    }
    return 0;
}

int b3_profile_read(b3_ctx* ctx, int kind, double* ms, double* flops, double* bytes, int64_t* launches) {
    if (!ctx || kind < 0 || kind >= B3_K_COUNT) return set_error(B3_EINVAL, "bad profile query");
    DeviceGuard g(ctx->device);
    B3_TRY(prof_collect(ctx));
    const Prof& p = ctx->prof;
    if (ms) *ms = p.ms[kind];
    if (flops) *flops = p.flops[kind];
    if (bytes) *bytes = p.bytes[kind];
    if (launches) *launches = p.launches[kind];
    return 0;
}

int b3_encode(b3_ctx* ctx, const float* sub, int t, int layers, float* out, unsigned flags) {
    if (t <= 0) return set_error(B3_EINVAL, "t must be positive");
    if (layers < 0) return set_error(B3_EINVAL, "layers must be >= 0");
    int32_t cu[2] = {0, t};
    return encode_any(ctx, sub, cu, 1, layers, out, flags);
}

int b3_encode_batch(b3_ctx* ctx, const float* sub, const int32_t* cu_seqlens, int n_utt, float* pooler,
                    unsigned flags) {
    if (!ctx) return set_error(B3_EINVAL, "null context");
    return encode_any(ctx, sub, cu_seqlens, n_utt, ctx->n_layers, pooler, flags);
}

int b3_linear_lut4(b3_ctx* ctx, const float* a, const uint8_t* codes, const uint16_t* lut16, const float* bias,
                   float* c, int m, int n, int k, unsigned flags) {
    return linear_any(ctx, a, codes, lut16, true, bias, c, m, n, k, flags);
}

int b3_linear_f16(b3_ctx* ctx, const float* a, const uint16_t* w16, const float* bias, float* c, int m, int n,
                  int k, unsigned flags) {
    return linear_any(ctx, a, w16, nullptr, false, bias, c, m, n, k, flags);
}

int b3_attn_conv(b3_ctx* ctx, int layer, float* x, int t, unsigned flags) {
    B3_TRY(check_finalized(ctx));
    if (layer < 0 || layer >= ctx->n_layers) return set_error(B3_EINVAL, "layer %d out of range", layer);
    if (!x || t <= 0) return set_error(B3_EINVAL, "bad input");
    DeviceGuard g(ctx->device);
    int32_t cu[2] = {0, t};
    B3_TRY(make_plan(ctx, cu, 1));
    const size_t bytes = static_cast<size_t>(t) * kHidden * 4;
    const Layer& L = ctx->layers[layer];
    if (flags & B3_DEVICE_PTRS) {
        B3_CUDA(cudaMemcpyAsync(ctx->x.p, x, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
    } else {
        B3_CUDA(cudaMemcpyAsync(ctx->x.p, x, bytes, cudaMemcpyHostToDevice, ctx->stream));
    }
    B3_TRY(attention_section(ctx, L, t));
    B3_TRY(conv_section(ctx, L, t));
    if (flags & B3_DEVICE_PTRS) {
        B3_CUDA(cudaMemcpyAsync(x, ctx->x.p, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
        return 0;
    }
    B3_CUDA(cudaMemcpyAsync(x, ctx->x.p, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    return sync_and_check(ctx);
}

}  // extern "C"
