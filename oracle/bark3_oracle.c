/*
 * bark3_oracle.c — CPU restatement of bark3-wgpu's CPU encoder path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline ("port" of the reference's AVX2 backend).  Only tests/, the smoke
 * check in __graft_entry__.py and bench.py's cpu_baseline / --impl reference
 * legs load it.  The product path (bark3-wgpu_b200/) never links or calls it.
 *
 * It restates, in C, the arithmetic of the reference's Rust CPU encoder
 * (reference paths are relative to the bark3-wgpu crate):
 *   - src/cpu/gemm.rs     PackW 16-column panels (f16 storage), the 6x16
 *                         FMA micro-kernel with k ascending, the TM=192/TN=128
 *                         task tiling and the split-k A.V product.
 *   - src/cpu/ops.rs      layer_norm (256 strided lanes + tree sum),
 *                         silu, glu, add_scaled, add_bias, rel_softmax_rows,
 *                         dwconv_bn_silu, pack_attention_inputs.
 *   - src/cpu/layer.rs    CpuLayer::forward (FF1 -> MHSA -> conv -> FF2 ->
 *                         norm_out), 256-row query blocks.
 *   - src/cpu/mod.rs      CpuEncoder::encode (sub linear, per-layer
 *                         truncation, projector), BN fold.
 *   - src/encoder.rs      pos_embed_f32 (228-246), pad128 (34-36).
 *   - src/bark.rs         expand (597-611): sign-magnitude level codes.
 *   - src/raw.rs          bf16 -> f32, f32 -> f16 (round to nearest even).
 *
 * Numerics follow the reference exactly where it is deterministic: every GEMM
 * output is one fused multiply-add chain over k in ascending order starting
 * from +0 (tile_avx2_half, src/cpu/gemm.rs:633-698); element-wise ops are
 * unfused multiply / add as Rust writes them (build with -ffp-contract=off);
 * exp/sin/cos/pow are the C library's expf/sinf/cosf/powf, which is what Rust's
 * f32 methods lower to on Linux.  The split-k reduction depends on the worker
 * count, which is an explicit argument here.
 */
#define _GNU_SOURCE
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define PANEL 16
#define MR 6
#define TM 192
#define TN 128
#define HIDDEN 1024
#define HEADS 8
#define HDIM 128
#define BQ 256

static int g_threads = 1;

void or_set_threads(int n) { g_threads = n > 0 ? n : 1; }
int or_get_threads(void) { return g_threads; }

/* ───────────────────────── f16 / bf16 conversions ───────────────────────── */

/* IEEE-754 binary32 -> binary16, round to nearest even (half::f16::from_f32). */
uint16_t or_f32_to_f16_bits(float v) {
    uint32_t x;
    memcpy(&x, &v, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) {                      /* inf / nan */
        if (man == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | (man >> 13));
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);   /* overflow -> inf */
    if (e <= 0) {                                      /* subnormal / zero */
        if (e < -10) return (uint16_t)sign;
        uint32_t m = man | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half_m = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (half_m & 1u))) half_m++;
        return (uint16_t)(sign | half_m);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;  /* carry may bump exp */
    return (uint16_t)h;
}

float or_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)h & 0x3FFu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {                                  /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            man &= 0x3FFu;
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1Fu) {
        x = sign | 0x7F800000u | (man << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

float or_round_f16(float v) { return or_f16_bits_to_f32(or_f32_to_f16_bits(v)); }

/* bf16 -> f32 bit pattern (src/raw.rs:126-128). */
float or_bf16_bits_to_f32(uint16_t b) {
    uint32_t x = (((uint32_t)b & 0x8000u) << 16) | (((uint32_t)b & 0x7FFFu) << 16);
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void or_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = or_f32_to_f16_bits(src[i]);
}

void or_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = or_f16_bits_to_f32(src[i]);
}

/* ───────────────────────────── 4-bit codes ───────────────────────────── */

/* `expand` (src/bark.rs:597-611): 0 -> 0, 1..=k -> +lev[c-1],
 * k+1..=2k -> -lev[c-k-1], anything else reads past the level list -> 0. */
float or_expand_code(int code, int k, const uint16_t* levels) {
    if (code == 0) return 0.0f;
    int mag, neg;
    if (code <= k) { mag = code - 1; neg = 0; } else { mag = code - k - 1; neg = 1; }
    float v = mag < k ? or_f16_bits_to_f32(levels[mag]) : 0.0f;
    return neg ? -v : v;
}

/* Codes packed two per byte (low nibble = even column) + a per-row 16-entry
 * f16 table -> dense f32 [rows][cols].  The reference's u32 words with eight
 * nibbles low-first along k are the same bytes (src/bark.rs:352-358). */
void or_expand_lut4(const uint8_t* codes, const uint16_t* lut16, float* dst,
                    int rows, int cols) {
    int ld = (cols + 1) / 2;
    for (int r = 0; r < rows; r++) {
        for (int c = 0; c < cols; c++) {
            uint8_t b = codes[(int64_t)r * ld + c / 2];
            int code = (c & 1) ? (b >> 4) : (b & 0xF);
            dst[(int64_t)r * cols + c] = or_f16_bits_to_f32(lut16[r * 16 + code]);
        }
    }
}

/* ─────────────────────────────── PackW ─────────────────────────────── */

typedef struct {
    int n, k;
    int half;
    float* d32;
    uint16_t* d16;
} PackW;

static void packw_free(PackW* p) {
    free(p->d32);
    free(p->d16);
    p->d32 = NULL;
    p->d16 = NULL;
    p->n = p->k = 0;
}

/* `refill_rows` / `refill_rows_half` (src/cpu/gemm.rs:107-167): w is (n, k)
 * row-major; panel p holds columns p*16..p*16+15, laid out [k][16]. */
static void packw_rows(PackW* p, const float* w, int n, int k, int half, int round_f16) {
    packw_free(p);
    p->n = n;
    p->k = k;
    p->half = half;
    int panels = (n + PANEL - 1) / PANEL;
    size_t sz = (size_t)panels * k * PANEL;
    if (half) p->d16 = (uint16_t*)calloc(sz, 2);
    else p->d32 = (float*)calloc(sz, 4);
#pragma omp parallel for schedule(static) num_threads(g_threads) if (panels >= 16)
    for (int pi = 0; pi < panels; pi++) {
        size_t base = (size_t)pi * k * PANEL;
        for (int j = 0; j < PANEL; j++) {
            int row = pi * PANEL + j;
            if (row >= n) break;
            for (int kk = 0; kk < k; kk++) {
                float v = w[(size_t)row * k + kk];
                if (half) p->d16[base + (size_t)kk * PANEL + j] = or_f32_to_f16_bits(v);
                else p->d32[base + (size_t)kk * PANEL + j] = round_f16 ? or_round_f16(v) : v;
            }
        }
    }
}

/* `refill_cols` (src/cpu/gemm.rs:169-202): source is (k, n) with row stride
 * ld starting at row k_off; output column j of panel p is src[..][p*16+j]. */
static void packw_cols(PackW* p, const float* src, int ld, int k_off, int n, int k, int round_f16) {
    packw_free(p);
    p->n = n;
    p->k = k;
    p->half = 0;
    int panels = (n + PANEL - 1) / PANEL;
    p->d32 = (float*)calloc((size_t)panels * k * PANEL, 4);
    for (int pi = 0; pi < panels; pi++) {
        size_t base = (size_t)pi * k * PANEL;
        int cols = n - pi * PANEL < PANEL ? n - pi * PANEL : PANEL;
        for (int kk = 0; kk < k; kk++) {
            const float* srow = src + (size_t)(k_off + kk) * ld + pi * PANEL;
            for (int j = 0; j < cols; j++) {
                float v = srow[j];
                p->d32[base + (size_t)kk * PANEL + j] = round_f16 ? or_round_f16(v) : v;
            }
        }
    }
}

/* ───────────────────────────── micro-kernels ───────────────────────────── */

static int have_avx2(void) {
#if defined(__x86_64__)
    static int v = -1;
    if (v < 0) {
        __builtin_cpu_init();
        v = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") &&
            __builtin_cpu_supports("f16c");
    }
    return v;
#else
    return 0;
#endif
}

#if defined(__x86_64__)
/* N rows x 16 columns, k ascending, one FMA per (row, lane) per k: the shape
 * of tile_avx2 / tile_avx2_half (src/cpu/gemm.rs:555-698). */
__attribute__((target("avx2,fma,f16c")))
static void micro_avx2(const float* a, int lda, int nrows, const PackW* w, size_t panel_off,
                       int k0, int k1, float* buf) {
    __m256 acc[MR * 2];
    for (int i = 0; i < MR * 2; i++) acc[i] = _mm256_setzero_ps();
    if (w->half) {
        const uint16_t* wp = w->d16 + panel_off;
        for (int kk = k0; kk < k1; kk++) {
            const uint16_t* wpk = wp + (size_t)kk * PANEL;
            __m256 w0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)wpk));
            __m256 w1 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(wpk + 8)));
            for (int r = 0; r < nrows; r++) {
                __m256 av = _mm256_broadcast_ss(a + (size_t)r * lda + kk);
                acc[2 * r] = _mm256_fmadd_ps(av, w0, acc[2 * r]);
                acc[2 * r + 1] = _mm256_fmadd_ps(av, w1, acc[2 * r + 1]);
            }
        }
    } else {
        const float* wp = w->d32 + panel_off;
        for (int kk = k0; kk < k1; kk++) {
            const float* wpk = wp + (size_t)kk * PANEL;
            __m256 w0 = _mm256_loadu_ps(wpk);
            __m256 w1 = _mm256_loadu_ps(wpk + 8);
            for (int r = 0; r < nrows; r++) {
                __m256 av = _mm256_broadcast_ss(a + (size_t)r * lda + kk);
                acc[2 * r] = _mm256_fmadd_ps(av, w0, acc[2 * r]);
                acc[2 * r + 1] = _mm256_fmadd_ps(av, w1, acc[2 * r + 1]);
            }
        }
    }
    for (int r = 0; r < nrows; r++) {
        _mm256_storeu_ps(buf + r * PANEL, acc[2 * r]);
        _mm256_storeu_ps(buf + r * PANEL + 8, acc[2 * r + 1]);
    }
}

/* Fully unrolled 6-row variant: the compiler keeps all 12 accumulators in
 * registers (the loop form above spills).  Same arithmetic order. */
__attribute__((target("avx2,fma,f16c")))
static void micro6_avx2(const float* a, int lda, const PackW* w, size_t panel_off,
                        int k0, int k1, float* buf) {
    __m256 c00 = _mm256_setzero_ps(), c01 = _mm256_setzero_ps();
    __m256 c10 = _mm256_setzero_ps(), c11 = _mm256_setzero_ps();
    __m256 c20 = _mm256_setzero_ps(), c21 = _mm256_setzero_ps();
    __m256 c30 = _mm256_setzero_ps(), c31 = _mm256_setzero_ps();
    __m256 c40 = _mm256_setzero_ps(), c41 = _mm256_setzero_ps();
    __m256 c50 = _mm256_setzero_ps(), c51 = _mm256_setzero_ps();
    const float* a0 = a;
    const float* a1 = a + lda;
    const float* a2 = a + 2 * (size_t)lda;
    const float* a3 = a + 3 * (size_t)lda;
    const float* a4 = a + 4 * (size_t)lda;
    const float* a5 = a + 5 * (size_t)lda;
#define OR_STEP(W0, W1, KK)                                                     \
    do {                                                                        \
        __m256 av;                                                              \
        av = _mm256_broadcast_ss(a0 + KK); c00 = _mm256_fmadd_ps(av, W0, c00); c01 = _mm256_fmadd_ps(av, W1, c01); \
        av = _mm256_broadcast_ss(a1 + KK); c10 = _mm256_fmadd_ps(av, W0, c10); c11 = _mm256_fmadd_ps(av, W1, c11); \
        av = _mm256_broadcast_ss(a2 + KK); c20 = _mm256_fmadd_ps(av, W0, c20); c21 = _mm256_fmadd_ps(av, W1, c21); \
        av = _mm256_broadcast_ss(a3 + KK); c30 = _mm256_fmadd_ps(av, W0, c30); c31 = _mm256_fmadd_ps(av, W1, c31); \
        av = _mm256_broadcast_ss(a4 + KK); c40 = _mm256_fmadd_ps(av, W0, c40); c41 = _mm256_fmadd_ps(av, W1, c41); \
        av = _mm256_broadcast_ss(a5 + KK); c50 = _mm256_fmadd_ps(av, W0, c50); c51 = _mm256_fmadd_ps(av, W1, c51); \
    } while (0)
    if (w->half) {
        const uint16_t* wp = w->d16 + panel_off;
        for (int kk = k0; kk < k1; kk++) {
            const uint16_t* wpk = wp + (size_t)kk * PANEL;
            __m256 w0 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)wpk));
            __m256 w1 = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(wpk + 8)));
            OR_STEP(w0, w1, kk);
        }
    } else {
        const float* wp = w->d32 + panel_off;
        for (int kk = k0; kk < k1; kk++) {
            const float* wpk = wp + (size_t)kk * PANEL;
            __m256 w0 = _mm256_loadu_ps(wpk);
            __m256 w1 = _mm256_loadu_ps(wpk + 8);
            OR_STEP(w0, w1, kk);
        }
    }
#undef OR_STEP
    _mm256_storeu_ps(buf + 0 * PANEL, c00); _mm256_storeu_ps(buf + 0 * PANEL + 8, c01);
    _mm256_storeu_ps(buf + 1 * PANEL, c10); _mm256_storeu_ps(buf + 1 * PANEL + 8, c11);
    _mm256_storeu_ps(buf + 2 * PANEL, c20); _mm256_storeu_ps(buf + 2 * PANEL + 8, c21);
    _mm256_storeu_ps(buf + 3 * PANEL, c30); _mm256_storeu_ps(buf + 3 * PANEL + 8, c31);
    _mm256_storeu_ps(buf + 4 * PANEL, c40); _mm256_storeu_ps(buf + 4 * PANEL + 8, c41);
    _mm256_storeu_ps(buf + 5 * PANEL, c50); _mm256_storeu_ps(buf + 5 * PANEL + 8, c51);
}
#endif

/* Scalar twin with the identical per-element order (fmaf, k ascending). */
static void micro_scalar(const float* a, int lda, int nrows, const PackW* w, size_t panel_off,
                         int k0, int k1, float* buf) {
    for (int r = 0; r < nrows; r++) {
        for (int j = 0; j < PANEL; j++) {
            float acc = 0.0f;
            for (int kk = k0; kk < k1; kk++) {
                float wv = w->half ? or_f16_bits_to_f32(w->d16[panel_off + (size_t)kk * PANEL + j])
                                   : w->d32[panel_off + (size_t)kk * PANEL + j];
                acc = fmaf(a[(size_t)r * lda + kk], wv, acc);
            }
            buf[r * PANEL + j] = acc;
        }
    }
}

/* `tile` (src/cpu/gemm.rs:456-494): rows x [n0, n0+ncols) over k in [k0, k1). */
static void tile(const float* a, int lda, const PackW* w, int n0, int ncols, float* c, int ldc,
                 int rows, int k0, int k1) {
    int k = w->k;
    int first = n0 / PANEL;
    int panels = (ncols + PANEL - 1) / PANEL;
    int simd = have_avx2();
    float buf[MR * PANEL];
    for (int row = 0; row < rows;) {
        int tr = rows - row < MR ? rows - row : MR;
        for (int p = 0; p < panels; p++) {
            int cols = ncols - p * PANEL < PANEL ? ncols - p * PANEL : PANEL;
            size_t off = (size_t)(first + p) * k * PANEL;
#if defined(__x86_64__)
            if (simd && tr == MR) micro6_avx2(a + (size_t)row * lda, lda, w, off, k0, k1, buf);
            else if (simd) micro_avx2(a + (size_t)row * lda, lda, tr, w, off, k0, k1, buf);
            else
#endif
                micro_scalar(a + (size_t)row * lda, lda, tr, w, off, k0, k1, buf);
            for (int r = 0; r < tr; r++)
                memcpy(c + (size_t)(row + r) * ldc + p * PANEL, buf + r * PANEL, cols * sizeof(float));
        }
        row += tr;
    }
    (void)simd;
}

static int mr_floor(int v) { int x = v / MR * MR; return x < MR ? MR : x; }
static int panel_floor(int v) { int x = v / PANEL * PANEL; return x < PANEL ? PANEL : x; }

/* `gemm` (src/cpu/gemm.rs:220-311): C[0..m, n0..n0+ncols] = A[m,k] W^T.
 * The task grid only changes which thread computes an element, never the
 * arithmetic of that element. */
static void gemm_packed(const float* a, const PackW* w, float* c, int m, int n0, int ncols) {
    int k = w->k;
    if (m == 0 || ncols == 0 || k == 0) return;
    int threads = g_threads;
    int tm = mr_floor(TM < (m > MR ? m : MR) ? TM : (m > MR ? m : MR));
    int tn = panel_floor((TN < ncols ? TN : ncols) > PANEL ? (TN < ncols ? TN : ncols) : PANEL);
    for (;;) {
        if (((m + tm - 1) / tm) * ((ncols + tn - 1) / tn) >= threads * 2) break;
        int can_m = tm > MR, can_n = tn > PANEL;
        if (!can_m && !can_n) break;
        if ((can_m && tm >= tn) || !can_n) tm = mr_floor(tm / 2 > MR ? tm / 2 : MR);
        else tn = panel_floor(tn / 2);
    }
    int mt = (m + tm - 1) / tm, nt = (ncols + tn - 1) / tn;
    int ntasks = mt * nt;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
    for (int t = 0; t < ntasks; t++) {
        int mi = t / nt, ni = t % nt;
        int m0 = mi * tm;
        int rows = m - m0 < tm ? m - m0 : tm;
        int tn0 = n0 + ni * tn;
        int cols = ncols - ni * tn < tn ? ncols - ni * tn : tn;
        tile(a + (size_t)m0 * k, k, w, tn0, cols, c + (size_t)m0 * ncols + (tn0 - n0), ncols, rows, 0, k);
    }
}

/* `gemm_split_k` (src/cpu/gemm.rs:348-415).  `workers` partial products over
 * contiguous k chunks, reduced in worker order with plain adds. */
static void gemm_split_k(const float* a, const PackW* w, float* c, float* parts, int m, int n0,
                         int ncols) {
    int k = w->k;
    int threads = g_threads;
    int workers = (k + 63) / 64;
    if (workers > threads) workers = threads;
    if (workers < 1) workers = 1;
    if (workers <= 1) { gemm_packed(a, w, c, m, n0, ncols); return; }
    int chunk = (k + workers - 1) / workers;
#pragma omp parallel for schedule(static, 1) num_threads(threads)
    for (int wi = 0; wi < workers; wi++) {
        int k0 = wi * chunk;
        int k1 = k0 + chunk < k ? k0 + chunk : k;
        if (k0 >= k1) continue;
        tile(a, k, w, n0, ncols, parts + (size_t)wi * m * ncols, ncols, m, k0, k1);
    }
    int total = m * ncols;
    for (int i = 0; i < total; i++) {
        float acc = 0.0f;
        for (int wi = 0; wi < workers; wi++) {
            int k0 = wi * chunk;
            if (k0 >= k) continue;           /* an idle worker's slice is never written */
            acc += parts[(size_t)wi * m * ncols + i];
        }
        c[i] = acc;
    }
}

/* Public single-call GEMM for tests: w is (n, k) row-major f32 values; `half`
 * selects the f16 panel storage the reference uses for static weights. */
void or_gemm(const float* a, const float* w, float* c, int m, int n, int k, int half) {
    PackW p = {0};
    packw_rows(&p, w, n, k, half, 0);
    gemm_packed(a, &p, c, m, 0, n);
    packw_free(&p);
}

/* Opaque packed weight for timing loops (the pack happens at load time). */
void* or_packw_new(const float* w, int n, int k, int half) {
    PackW* p = (PackW*)calloc(1, sizeof(PackW));
    packw_rows(p, w, n, k, half, 0);
    return p;
}

void or_packw_free(void* p) {
    if (!p) return;
    packw_free((PackW*)p);
    free(p);
}

void or_gemm_packed(const float* a, const void* pw, float* c, int m) {
    const PackW* p = (const PackW*)pw;
    gemm_packed(a, p, c, m, 0, p->n);
}

/* ──────────────────────────────── ops ──────────────────────────────── */

/* `layer_norm` (src/cpu/ops.rs:15-56): 256 lanes of 4 strided elements,
 * tree-summed; var = E[x^2] - mean^2. */
void or_layer_norm(const float* src, float* dst, const float* w, const float* b, int rows, int dim) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (rows >= 8)
    for (int r = 0; r < rows; r++) {
        const float* x = src + (size_t)r * dim;
        float* y = dst + (size_t)r * dim;
        float rs[256], rq[256];
        for (int lane = 0; lane < 256; lane++) {
            float e0 = x[lane], e1 = x[lane + 256], e2 = x[lane + 512], e3 = x[lane + 768];
            rs[lane] = (e0 + e2) + (e1 + e3);
            rq[lane] = (e0 * e0 + e2 * e2) + (e1 * e1 + e3 * e3);
        }
        for (int s = 128; s > 0; s >>= 1)
            for (int i = 0; i < s; i++) {
                rs[i] += rs[i + s];
                rq[i] += rq[i + s];
            }
        float inv_n = 1.0f / (float)dim;
        float mean = rs[0] * inv_n;
        float var = rq[0] * inv_n - mean * mean;
        float inv_std = 1.0f / sqrtf(var + 1e-5f);
        for (int i = 0; i < dim; i++) y[i] = (x[i] - mean) * inv_std * w[i] + b[i];
    }
}

void or_silu(float* x, int64_t n) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (n >= 4096)
    for (int64_t i = 0; i < n; i++) x[i] = x[i] / (1.0f + expf(-x[i]));
}

/* `glu` (src/cpu/ops.rs:74-95): dst[r][i] = a / (1 + exp(-b)). */
void or_glu(const float* src, float* dst, int rows, int c) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (rows >= 8)
    for (int r = 0; r < rows; r++)
        for (int i = 0; i < c; i++) {
            float a = src[(size_t)r * 2 * c + i], bb = src[(size_t)r * 2 * c + c + i];
            dst[(size_t)r * c + i] = a / (1.0f + expf(-bb));
        }
}

void or_add_scaled(float* a, const float* b, float scale, int64_t n) {
    for (int64_t i = 0; i < n; i++) a[i] += scale * b[i];
}

void or_add_bias(float* x, const float* bias, int rows, int dim) {
    for (int r = 0; r < rows; r++)
        for (int i = 0; i < dim; i++) x[(size_t)r * dim + i] += bias[i];
}

/* `rel_softmax_rows` (src/cpu/ops.rs:133-189). */
void or_rel_softmax_rows(float* probs, const float* bd, int win, int rows, int t, int q0, int j0,
                         float scale) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (rows >= 8)
    for (int qi = 0; qi < rows; qi++) {
        float* prow = probs + (size_t)qi * t;
        int shift = t - 1 - (q0 + qi) - j0;
        const float* brow = bd + (size_t)qi * win;
        float m = -INFINITY;
        for (int k = 0; k < t; k++) {
            float s = scale * (prow[k] + brow[shift + k]);
            prow[k] = s;
            if (s > m) m = s;
        }
        float part[256];
        for (int lane = 0; lane < 256; lane++) {
            float acc = 0.0f;
            for (int j = lane; j < t; j += 256) {
                float e = expf(prow[j] - m);
                prow[j] = e;
                acc += e;
            }
            part[lane] = acc;
        }
        for (int s = 128; s > 0; s >>= 1)
            for (int i = 0; i < s; i++) part[i] += part[i + s];
        float sum = part[0];
        for (int k = 0; k < t; k++) prow[k] /= sum;
    }
}

/* `dwconv_bn_silu` (src/cpu/ops.rs:195-233): taps 0..8 over frames t-4..t+4,
 * frames outside [0, rows) skipped. */
void or_dwconv_bn_silu(const float* src, const float* dw, const float* bn_a, const float* bn_b,
                       float* dst, int rows, int dim) {
#pragma omp parallel for schedule(static) num_threads(g_threads) if (rows >= 8)
    for (int t = 0; t < rows; t++)
        for (int c = 0; c < dim; c++) {
            float acc = 0.0f;
            for (int i = 0; i < 9; i++) {
                int tt = t + i - 4;
                if (tt < 0 || tt >= rows) continue;
                acc += src[(size_t)tt * dim + c] * dw[c * 9 + i];
            }
            float y = acc * bn_a[c] + bn_b[c];
            dst[(size_t)t * dim + c] = y / (1.0f + expf(-y));
        }
}

/* `pos_embed_f32` (src/encoder.rs:228-246): row j is position T-1-j,
 * [sin, cos] interleaved, inv_freq = 1 / 10000^(2i/1024). */
void or_pos_embed(int t, float* out) {
    int p = 2 * t - 1;
    float inv_freq[HIDDEN / 2];
    for (int i = 0; i < HIDDEN / 2; i++)
        inv_freq[i] = 1.0f / powf(10000.0f, (2.0f * (float)i) / (float)HIDDEN);
    for (int pi = 0; pi < p; pi++) {
        float pos = (float)((p - 1) / 2 - pi);
        for (int i = 0; i < HIDDEN / 2; i++) {
            float f = pos * inv_freq[i];
            out[(size_t)pi * HIDDEN + 2 * i] = sinf(f);
            out[(size_t)pi * HIDDEN + 2 * i + 1] = cosf(f);
        }
    }
}

/* ─────────────────────────────── encoder ─────────────────────────────── */

typedef struct {
    PackW qkv, o, ff1a, ff1b, ff2a, ff2b, pw1, pw2;
    float* relk;   /* (1024, 1024) f16-rounded values, used as the A operand */
    float* dw;     /* (1024, 9) f16-rounded */
    float bn_a[HIDDEN], bn_b[HIDDEN];
    float ln_w[5][HIDDEN], ln_b[5][HIDDEN];
    float bu[HIDDEN], bv[HIDDEN];
} OrLayer;

typedef struct {
    int n_layers;
    int half;
    PackW sub_w, proj_w;
    float sub_b[HIDDEN];
    float proj_b[640];
    OrLayer* layers;
} OrEncoder;

static float* dup_round(const float* src, size_t n) {
    float* d = (float*)malloc(n * 4);
    for (size_t i = 0; i < n; i++) d[i] = or_round_f16(src[i]);
    return d;
}

/* Weight set as the reference's CpuEncoder::load_with sees it
 * (src/cpu/mod.rs:47-152): every matrix is given as f32 values (bf16
 * checkpoints widened, 4-bit layers expanded); they are rounded to f16 here
 * (f16v, src/cpu/mod.rs:35-37) before packing.  BN is folded on load. */
void* or_encoder_new(int n_layers, int half, const float* sub_w, const float* sub_b,
                     const float* proj_w, const float* proj_b) {
    OrEncoder* e = (OrEncoder*)calloc(1, sizeof(OrEncoder));
    e->n_layers = n_layers;
    e->half = half;
    float* r = dup_round(sub_w, (size_t)HIDDEN * 4096);
    packw_rows(&e->sub_w, r, HIDDEN, 4096, half, 0);
    free(r);
    memcpy(e->sub_b, sub_b, sizeof(e->sub_b));
    r = dup_round(proj_w, (size_t)640 * HIDDEN);
    packw_rows(&e->proj_w, r, 640, HIDDEN, half, 0);
    free(r);
    memcpy(e->proj_b, proj_b, sizeof(e->proj_b));
    e->layers = (OrLayer*)calloc((size_t)n_layers, sizeof(OrLayer));
    return e;
}

static void pack_round(PackW* p, const float* w, int n, int k, int half) {
    float* r = dup_round(w, (size_t)n * k);
    packw_rows(p, r, n, k, half, 0);
    free(r);
}

/* ln_w/ln_b: 5 x 1024 in the order norm_feed_forward1, norm_self_att,
 * norm_conv, norm_feed_forward2, norm_out.  bn: gamma, beta, mean, var. */
int or_encoder_set_layer(void* enc, int l, const float* wq, const float* wk, const float* wv,
                         const float* relk, const float* o, const float* ff1a, const float* ff1b,
                         const float* ff2a, const float* ff2b, const float* pw1, const float* pw2,
                         const float* dw, const float* bn_gamma, const float* bn_beta,
                         const float* bn_mean, const float* bn_var, const float* ln_w,
                         const float* ln_b, const float* bu, const float* bv) {
    OrEncoder* e = (OrEncoder*)enc;
    if (l < 0 || l >= e->n_layers) return -1;
    OrLayer* L = &e->layers[l];
    float* cat = (float*)malloc((size_t)3 * HIDDEN * HIDDEN * 4);
    memcpy(cat, wq, (size_t)HIDDEN * HIDDEN * 4);
    memcpy(cat + (size_t)HIDDEN * HIDDEN, wk, (size_t)HIDDEN * HIDDEN * 4);
    memcpy(cat + (size_t)2 * HIDDEN * HIDDEN, wv, (size_t)HIDDEN * HIDDEN * 4);
    pack_round(&L->qkv, cat, 3072, HIDDEN, e->half);
    free(cat);
    L->relk = dup_round(relk, (size_t)HIDDEN * HIDDEN);
    pack_round(&L->o, o, HIDDEN, HIDDEN, e->half);
    pack_round(&L->ff1a, ff1a, 4096, HIDDEN, e->half);
    pack_round(&L->ff1b, ff1b, HIDDEN, 4096, e->half);
    pack_round(&L->ff2a, ff2a, 4096, HIDDEN, e->half);
    pack_round(&L->ff2b, ff2b, HIDDEN, 4096, e->half);
    pack_round(&L->pw1, pw1, 2048, HIDDEN, e->half);
    pack_round(&L->pw2, pw2, HIDDEN, HIDDEN, e->half);
    L->dw = dup_round(dw, (size_t)HIDDEN * 9);
    for (int c = 0; c < HIDDEN; c++) {       /* BN fold, src/cpu/mod.rs:113-119 */
        float a = bn_gamma[c] / sqrtf(bn_var[c] + 1e-5f);
        L->bn_a[c] = a;
        L->bn_b[c] = bn_beta[c] - bn_mean[c] * a;
    }
    memcpy(L->ln_w, ln_w, sizeof(L->ln_w));
    memcpy(L->ln_b, ln_b, sizeof(L->ln_b));
    memcpy(L->bu, bu, sizeof(L->bu));
    memcpy(L->bv, bv, sizeof(L->bv));
    return 0;
}

void or_encoder_free(void* enc) {
    OrEncoder* e = (OrEncoder*)enc;
    if (!e) return;
    packw_free(&e->sub_w);
    packw_free(&e->proj_w);
    for (int l = 0; l < e->n_layers; l++) {
        OrLayer* L = &e->layers[l];
        packw_free(&L->qkv); packw_free(&L->o);
        packw_free(&L->ff1a); packw_free(&L->ff1b); packw_free(&L->ff2a); packw_free(&L->ff2b);
        packw_free(&L->pw1); packw_free(&L->pw2);
        free(L->relk); free(L->dw);
    }
    free(e->layers);
    free(e);
}

static int pad128(int n) { return (n + 127) & ~127; }

typedef struct {
    int t, pp;
    float *normed, *ffb, *tmp, *tmp2, *qkv, *qu, *qv, *kh, *vh, *relk_t, *attnout, *cb1, *cb2;
    float *probs, *bd, *attn_h, *av_parts;
    PackW kh_pack[HEADS], vh_pack[HEADS], rkh_pack[HEADS];
} Scratch;

static void scratch_init(Scratch* s, int t) {
    memset(s, 0, sizeof(*s));
    s->t = t;
    s->pp = pad128(2 * t - 1);
    s->normed = (float*)calloc((size_t)t * HIDDEN, 4);
    s->ffb = (float*)calloc((size_t)t * 4096, 4);
    s->tmp = (float*)calloc((size_t)t * HIDDEN, 4);
    s->tmp2 = (float*)calloc((size_t)t * HIDDEN, 4);
    s->qkv = (float*)calloc((size_t)t * 3072, 4);
    s->qu = (float*)calloc((size_t)HEADS * t * HDIM, 4);
    s->qv = (float*)calloc((size_t)HEADS * t * HDIM, 4);
    s->kh = (float*)calloc((size_t)HEADS * t * HDIM, 4);
    s->vh = (float*)calloc((size_t)HEADS * t * HDIM, 4);
    s->relk_t = (float*)calloc((size_t)HIDDEN * s->pp, 4);
    s->attnout = (float*)calloc((size_t)t * HIDDEN, 4);
    s->cb1 = (float*)calloc((size_t)t * 2048, 4);
    s->cb2 = (float*)calloc((size_t)t * HIDDEN, 4);
    s->probs = (float*)calloc((size_t)BQ * t, 4);
    s->bd = (float*)calloc((size_t)BQ * (t + BQ + 2 * PANEL), 4);
    s->attn_h = (float*)calloc((size_t)BQ * HDIM, 4);
    s->av_parts = (float*)calloc((size_t)g_threads * BQ * HDIM, 4);
}

static void scratch_free(Scratch* s) {
    free(s->normed); free(s->ffb); free(s->tmp); free(s->tmp2); free(s->qkv);
    free(s->qu); free(s->qv); free(s->kh); free(s->vh); free(s->relk_t); free(s->attnout);
    free(s->cb1); free(s->cb2); free(s->probs); free(s->bd); free(s->attn_h); free(s->av_parts);
    for (int h = 0; h < HEADS; h++) {
        packw_free(&s->kh_pack[h]); packw_free(&s->vh_pack[h]); packw_free(&s->rkh_pack[h]);
    }
}

/* `pack_attention_inputs` (src/cpu/ops.rs:238-279). */
static void pack_attention_inputs(const float* qkv, int rows, const float* bu, const float* bv,
                                  float* qu, float* qv, float* kh, float* vh) {
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int i = 0; i < HEADS * rows; i++) {
        int h = i / rows, q = i % rows;
        for (int j = 0; j < HDIM; j++) {
            int b = h * HDIM + j;
            const float* row = qkv + (size_t)q * 3072;
            qu[(size_t)i * HDIM + j] = row[b] + bu[b];
            qv[(size_t)i * HDIM + j] = row[b] + bv[b];
            kh[(size_t)i * HDIM + j] = or_round_f16(row[1024 + b]);
            vh[(size_t)i * HDIM + j] = or_round_f16(row[2048 + b]);
        }
    }
}

/* `CpuLayer::forward` (src/cpu/layer.rs:157-327). */
static void layer_forward(const OrLayer* L, float* x, Scratch* s, const PackW* pos) {
    int t = s->t, pp = s->pp;
    float scale = powf((float)HDIM, -0.5f);

    /* FF1 */
    or_layer_norm(x, s->normed, L->ln_w[0], L->ln_b[0], t, HIDDEN);
    gemm_packed(s->normed, &L->ff1a, s->ffb, t, 0, 4096);
    or_silu(s->ffb, (int64_t)t * 4096);
    gemm_packed(s->ffb, &L->ff1b, s->tmp, t, 0, HIDDEN);
    or_add_scaled(x, s->tmp, 0.5f, (int64_t)t * HIDDEN);

    /* attention */
    or_layer_norm(x, s->normed, L->ln_w[1], L->ln_b[1], t, HIDDEN);
    gemm_packed(s->normed, &L->qkv, s->qkv, t, 0, 3072);
    pack_attention_inputs(s->qkv, t, L->bu, L->bv, s->qu, s->qv, s->kh, s->vh);
    for (int h = 0; h < HEADS; h++) {
        packw_rows(&s->kh_pack[h], s->kh + (size_t)h * t * HDIM, t, HDIM, 0, 0);
        packw_cols(&s->vh_pack[h], s->vh + (size_t)h * t * HDIM, HDIM, 0, HDIM, t, 0);
    }
    /* relk_t[d][p] = relk[d] . pos[p], then rounded through f16 when packed. */
    gemm_packed(L->relk, pos, s->relk_t, HIDDEN, 0, pp);
    for (int h = 0; h < HEADS; h++)
        packw_cols(&s->rkh_pack[h], s->relk_t + (size_t)h * HDIM * pp, pp, 0, pp, HDIM, 1);

    for (int q0 = 0; q0 < t;) {
        int rows = t - q0 < BQ ? t - q0 : BQ;
        int jmin = t - 1 - (q0 + rows - 1);
        int jmax = 2 * t - 2 - q0;
        if (jmax > pp - 1) jmax = pp - 1;
        int j0 = (jmin / PANEL) * PANEL;
        int j1 = (jmax + PANEL) / PANEL * PANEL;
        if (j1 > pp) j1 = pp;
        int win = j1 - j0;
        for (int h = 0; h < HEADS; h++) {
            gemm_packed(s->qu + (size_t)h * t * HDIM + (size_t)q0 * HDIM, &s->kh_pack[h], s->probs,
                        rows, 0, t);
            gemm_packed(s->qv + (size_t)h * t * HDIM + (size_t)q0 * HDIM, &s->rkh_pack[h], s->bd,
                        rows, j0, win);
            or_rel_softmax_rows(s->probs, s->bd, win, rows, t, q0, j0, scale);
            gemm_split_k(s->probs, &s->vh_pack[h], s->attn_h, s->av_parts, rows, 0, HDIM);
            for (int qi = 0; qi < rows; qi++)
                memcpy(s->attnout + (size_t)(q0 + qi) * HIDDEN + h * HDIM, s->attn_h + (size_t)qi * HDIM,
                       HDIM * 4);
        }
        q0 += rows;
    }
    gemm_packed(s->attnout, &L->o, s->tmp, t, 0, HIDDEN);
    or_add_scaled(x, s->tmp, 1.0f, (int64_t)t * HIDDEN);

    /* conv module */
    or_layer_norm(x, s->normed, L->ln_w[2], L->ln_b[2], t, HIDDEN);
    gemm_packed(s->normed, &L->pw1, s->cb1, t, 0, 2048);
    or_glu(s->cb1, s->cb2, t, HIDDEN);
    or_dwconv_bn_silu(s->cb2, L->dw, L->bn_a, L->bn_b, s->tmp, t, HIDDEN);
    gemm_packed(s->tmp, &L->pw2, s->tmp2, t, 0, HIDDEN);
    or_add_scaled(x, s->tmp2, 1.0f, (int64_t)t * HIDDEN);

    /* FF2 */
    or_layer_norm(x, s->normed, L->ln_w[3], L->ln_b[3], t, HIDDEN);
    gemm_packed(s->normed, &L->ff2a, s->ffb, t, 0, 4096);
    or_silu(s->ffb, (int64_t)t * 4096);
    gemm_packed(s->ffb, &L->ff2b, s->tmp, t, 0, HIDDEN);
    or_add_scaled(x, s->tmp, 0.5f, (int64_t)t * HIDDEN);

    /* norm_out into the scratch; the caller decides whether to adopt it. */
    or_layer_norm(x, s->normed, L->ln_w[4], L->ln_b[4], t, HIDDEN);
}

/* `CpuEncoder::encode` (src/cpu/mod.rs:156-189).  Returns the (t, 640)
 * pooler when layers >= n_layers, else the last block's pre-norm residual
 * (t, 1024).  `out` must hold the matching size.  When `dump` is given and
 * every block runs, it receives the pre-norm_out residual after each block
 * (n_layers x t x 1024 floats) from the same single pass: block l's entry
 * equals what a call with layers = l + 1 returns. */
static int encode_impl(OrEncoder* e, const float* sub, int t, int layers, float* out, float* dump) {
    if (t <= 0) return -1;
    Scratch s;
    scratch_init(&s, t);
    float* pos_pad = (float*)calloc((size_t)s.pp * HIDDEN, 4);
    or_pos_embed(t, pos_pad);
    PackW pos = {0};
    packw_rows(&pos, pos_pad, s.pp, HIDDEN, 0, 0);
    free(pos_pad);

    float* x = (float*)calloc((size_t)t * HIDDEN, 4);
    gemm_packed(sub, &e->sub_w, x, t, 0, HIDDEN);
    or_add_bias(x, e->sub_b, t, HIDDEN);
    int upto = layers < e->n_layers ? layers : e->n_layers;
    for (int i = 0; i < upto; i++) {
        layer_forward(&e->layers[i], x, &s, &pos);
        if (dump) memcpy(dump + (size_t)i * t * HIDDEN, x, (size_t)t * HIDDEN * 4);
        if (i + 1 < upto || upto == e->n_layers) memcpy(x, s.normed, (size_t)t * HIDDEN * 4);
    }
    if (upto == e->n_layers) {
        gemm_packed(x, &e->proj_w, out, t, 0, 640);
        or_add_bias(out, e->proj_b, t, 640);
    } else {
        memcpy(out, x, (size_t)t * HIDDEN * 4);
    }
    free(x);
    packw_free(&pos);
    scratch_free(&s);
    return 0;
}

int or_encode(void* enc, const float* sub, int t, int layers, float* out) {
    return encode_impl((OrEncoder*)enc, sub, t, layers, out, NULL);
}

/* Every block's pre-norm_out residual (dump: n_layers x t x 1024) and the
 * pooler (out: t x 640) in one pass over all blocks. */
int or_encode_layers(void* enc, const float* sub, int t, float* dump, float* out) {
    OrEncoder* e = (OrEncoder*)enc;
    return encode_impl(e, sub, t, e->n_layers, out, dump);
}

/* Attention + conv sections of one block in isolation:
 * x (t, 1024) -> x + MHSA(LN(x)) then + conv(LN(x)), same code as the layer. */
int or_attn_conv(void* enc, int l, float* x, int t) {
    OrEncoder* e = (OrEncoder*)enc;
    if (l < 0 || l >= e->n_layers || t <= 0) return -1;
    const OrLayer* L = &e->layers[l];
    Scratch s;
    scratch_init(&s, t);
    int pp = s.pp;
    float* pos_pad = (float*)calloc((size_t)pp * HIDDEN, 4);
    or_pos_embed(t, pos_pad);
    PackW pos = {0};
    packw_rows(&pos, pos_pad, pp, HIDDEN, 0, 0);
    free(pos_pad);
    float scale = powf((float)HDIM, -0.5f);

    or_layer_norm(x, s.normed, L->ln_w[1], L->ln_b[1], t, HIDDEN);
    gemm_packed(s.normed, &L->qkv, s.qkv, t, 0, 3072);
    pack_attention_inputs(s.qkv, t, L->bu, L->bv, s.qu, s.qv, s.kh, s.vh);
    for (int h = 0; h < HEADS; h++) {
        packw_rows(&s.kh_pack[h], s.kh + (size_t)h * t * HDIM, t, HDIM, 0, 0);
        packw_cols(&s.vh_pack[h], s.vh + (size_t)h * t * HDIM, HDIM, 0, HDIM, t, 0);
    }
    gemm_packed(L->relk, &pos, s.relk_t, HIDDEN, 0, pp);
    for (int h = 0; h < HEADS; h++)
        packw_cols(&s.rkh_pack[h], s.relk_t + (size_t)h * HDIM * pp, pp, 0, pp, HDIM, 1);
    for (int q0 = 0; q0 < t;) {
        int rows = t - q0 < BQ ? t - q0 : BQ;
        int jmin = t - 1 - (q0 + rows - 1);
        int jmax = 2 * t - 2 - q0;
        if (jmax > pp - 1) jmax = pp - 1;
        int j0 = (jmin / PANEL) * PANEL;
        int j1 = (jmax + PANEL) / PANEL * PANEL;
        if (j1 > pp) j1 = pp;
        int win = j1 - j0;
        for (int h = 0; h < HEADS; h++) {
            gemm_packed(s.qu + (size_t)h * t * HDIM + (size_t)q0 * HDIM, &s.kh_pack[h], s.probs, rows, 0, t);
            gemm_packed(s.qv + (size_t)h * t * HDIM + (size_t)q0 * HDIM, &s.rkh_pack[h], s.bd, rows, j0, win);
            or_rel_softmax_rows(s.probs, s.bd, win, rows, t, q0, j0, scale);
            gemm_split_k(s.probs, &s.vh_pack[h], s.attn_h, s.av_parts, rows, 0, HDIM);
            for (int qi = 0; qi < rows; qi++)
                memcpy(s.attnout + (size_t)(q0 + qi) * HIDDEN + h * HDIM, s.attn_h + (size_t)qi * HDIM, HDIM * 4);
        }
        q0 += rows;
    }
    gemm_packed(s.attnout, &L->o, s.tmp, t, 0, HIDDEN);
    or_add_scaled(x, s.tmp, 1.0f, (int64_t)t * HIDDEN);

    or_layer_norm(x, s.normed, L->ln_w[2], L->ln_b[2], t, HIDDEN);
    gemm_packed(s.normed, &L->pw1, s.cb1, t, 0, 2048);
    or_glu(s.cb1, s.cb2, t, HIDDEN);
    or_dwconv_bn_silu(s.cb2, L->dw, L->bn_a, L->bn_b, s.tmp, t, HIDDEN);
    gemm_packed(s.tmp, &L->pw2, s.tmp2, t, 0, HIDDEN);
    or_add_scaled(x, s.tmp2, 1.0f, (int64_t)t * HIDDEN);
    packw_free(&pos);
    scratch_free(&s);
    return 0;
}

/* Standalone attention core for kernel-level parity: head-major inputs as
 * the reference packs them (qu/qv f32, k/v already f16-rounded), relk_t is
 * (1024, pp) before its f16 rounding.  out is (t, 1024). */
int or_attention_core(const float* qu, const float* qv, const float* kh, const float* vh,
                      const float* relk_t, int t, float* out) {
    int pp = pad128(2 * t - 1);
    float scale = powf((float)HDIM, -0.5f);
    PackW kp = {0}, vp = {0}, rp = {0};
    float* probs = (float*)calloc((size_t)BQ * t, 4);
    float* bd = (float*)calloc((size_t)BQ * (t + BQ + 2 * PANEL), 4);
    float* attn_h = (float*)calloc((size_t)BQ * HDIM, 4);
    float* parts = (float*)calloc((size_t)g_threads * BQ * HDIM, 4);
    for (int h = 0; h < HEADS; h++) {
        packw_rows(&kp, kh + (size_t)h * t * HDIM, t, HDIM, 0, 0);
        packw_cols(&vp, vh + (size_t)h * t * HDIM, HDIM, 0, HDIM, t, 0);
        packw_cols(&rp, relk_t + (size_t)h * HDIM * pp, pp, 0, pp, HDIM, 1);
        for (int q0 = 0; q0 < t;) {
            int rows = t - q0 < BQ ? t - q0 : BQ;
            int jmin = t - 1 - (q0 + rows - 1);
            int jmax = 2 * t - 2 - q0;
            if (jmax > pp - 1) jmax = pp - 1;
            int j0 = (jmin / PANEL) * PANEL;
            int j1 = (jmax + PANEL) / PANEL * PANEL;
            if (j1 > pp) j1 = pp;
            int win = j1 - j0;
            gemm_packed(qu + (size_t)h * t * HDIM + (size_t)q0 * HDIM, &kp, probs, rows, 0, t);
            gemm_packed(qv + (size_t)h * t * HDIM + (size_t)q0 * HDIM, &rp, bd, rows, j0, win);
            or_rel_softmax_rows(probs, bd, win, rows, t, q0, j0, scale);
            gemm_split_k(probs, &vp, attn_h, parts, rows, 0, HDIM);
            for (int qi = 0; qi < rows; qi++)
                memcpy(out + (size_t)(q0 + qi) * HIDDEN + h * HDIM, attn_h + (size_t)qi * HDIM, HDIM * 4);
            q0 += rows;
        }
    }
    packw_free(&kp); packw_free(&vp); packw_free(&rp);
    free(probs); free(bd); free(attn_h); free(parts);
    return 0;
}

/* ───────────────────────────── TDT decoder ─────────────────────────────
 * Restates TdtDecoder (src/tdt.rs:19-535): 2-layer LSTM prediction net
 * (hidden 640, gate order i, f, g, o), projector 640 -> 640, joint
 * ReLU(enc + dec) . head^T + bias over vocab + 5 duration rows, greedy loop
 * with blank forcing at least one frame and the step guard
 * T * (MAX_SYMBOLS + 4) + 64.  Matrices are stored f16 (pack16), the
 * embedding stays f32, as in the reference. */

#define DEC_H 640
#define DEC_GS (4 * DEC_H)
#define N_DUR 5
#define MAX_SYMBOLS 10

/* dot16 (src/tdt.rs:57-97): two 8-lane FMA accumulators over 16-element
 * blocks, then an 8-lane block, lanes summed 0..7, scalar tail.  `w` holds
 * the f16 weights widened to f32 (exact), as vcvtph2ps produces them. */
#if defined(__x86_64__)
__attribute__((target("avx2,fma")))
static float dot16_avx2(const float* w, const float* x, int n) {
    __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(w + i), _mm256_loadu_ps(x + i), a0);
        a1 = _mm256_fmadd_ps(_mm256_loadu_ps(w + i + 8), _mm256_loadu_ps(x + i + 8), a1);
    }
    __m256 acc = _mm256_add_ps(a0, a1);
    for (; i + 8 <= n; i += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(w + i), _mm256_loadu_ps(x + i), acc);
    float tmp[8];
    _mm256_storeu_ps(tmp, acc);
    float sum = 0.0f;
    for (int l = 0; l < 8; l++) sum += tmp[l];
    for (; i < n; i++) sum += w[i] * x[i];
    return sum;
}
#endif

static float dot16(const float* w, const float* x, int n) {
#if defined(__x86_64__)
    if (have_avx2()) return dot16_avx2(w, x, n);
#endif
    float a0[8] = {0}, a1[8] = {0}, acc[8];
    int i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 8; l++) {
            a0[l] = fmaf(w[i + l], x[i + l], a0[l]);
            a1[l] = fmaf(w[i + 8 + l], x[i + 8 + l], a1[l]);
        }
    for (int l = 0; l < 8; l++) acc[l] = a0[l] + a1[l];
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(w[i + l], x[i + l], acc[l]);
    float sum = 0.0f;
    for (int l = 0; l < 8; l++) sum += acc[l];
    for (; i < n; i++) sum += w[i] * x[i];
    return sum;
}

typedef struct {
    int vocab;            /* token rows incl. blank; blank = vocab - 1 */
    float* embed;         /* [vocab][640] f32 */
    float* w_ih;          /* [2][2560][640] f16 values (widened) */
    float* w_hh;
    float* b_ih;          /* [2][2560] */
    float* b_hh;
    float* proj_w;        /* [640][640] f16 values */
    float* proj_b;
    float* head_w;        /* [vocab + 5][640] f16 values */
    float* head_b;
} OrTdt;

/* pack16 (src/tdt.rs:49-55): round to f16, kept widened to f32 */
static float* pack16(const float* v, size_t n) {
    float* o = (float*)malloc(n * 4);
    for (size_t i = 0; i < n; i++) o[i] = or_round_f16(v[i]);
    return o;
}

static float* dupf(const float* v, size_t n) {
    float* o = (float*)malloc(n * 4);
    memcpy(o, v, n * 4);
    return o;
}

void* or_tdt_new(int vocab, const float* embed, const float* w_ih, const float* w_hh, const float* b_ih,
                 const float* b_hh, const float* proj_w, const float* proj_b, const float* head_w,
                 const float* head_b) {
    OrTdt* d = (OrTdt*)calloc(1, sizeof(OrTdt));
    d->vocab = vocab;
    d->embed = dupf(embed, (size_t)vocab * DEC_H);
    d->w_ih = pack16(w_ih, (size_t)2 * DEC_GS * DEC_H);
    d->w_hh = pack16(w_hh, (size_t)2 * DEC_GS * DEC_H);
    d->b_ih = dupf(b_ih, 2 * DEC_GS);
    d->b_hh = dupf(b_hh, 2 * DEC_GS);
    d->proj_w = pack16(proj_w, (size_t)DEC_H * DEC_H);
    d->proj_b = dupf(proj_b, DEC_H);
    d->head_w = pack16(head_w, (size_t)(vocab + N_DUR) * DEC_H);
    d->head_b = dupf(head_b, (size_t)vocab + N_DUR);
    return d;
}

void or_tdt_free(void* p) {
    OrTdt* d = (OrTdt*)p;
    if (!d) return;
    free(d->embed); free(d->w_ih); free(d->w_hh); free(d->b_ih); free(d->b_hh);
    free(d->proj_w); free(d->proj_b); free(d->head_w); free(d->head_b);
    free(d);
}

static float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

/* lstm_step (src/tdt.rs:179-214) */
static void lstm_step(const OrTdt* d, const float* x, float h[2][DEC_H], float c[2][DEC_H]) {
    float gates[DEC_GS];
    for (int layer = 0; layer < 2; layer++) {
        const float* wih = d->w_ih + (size_t)layer * DEC_GS * DEC_H;
        const float* whh = d->w_hh + (size_t)layer * DEC_GS * DEC_H;
        const float* bih = d->b_ih + layer * DEC_GS;
        const float* bhh = d->b_hh + layer * DEC_GS;
        const float* xin = layer == 0 ? x : h[0];
        const float* hin = h[layer];
        for (int row = 0; row < DEC_GS; row++)
            gates[row] = bih[row] + bhh[row] + dot16(wih + (size_t)row * DEC_H, xin, DEC_H) +
                         dot16(whh + (size_t)row * DEC_H, hin, DEC_H);
        for (int ch = 0; ch < DEC_H; ch++) {
            float in = sigm(gates[ch]);
            float fg = sigm(gates[DEC_H + ch]);
            float cand = tanhf(gates[2 * DEC_H + ch]);
            c[layer][ch] = fg * c[layer][ch] + in * cand;
            float out = sigm(gates[3 * DEC_H + ch]);
            h[layer][ch] = out * tanhf(c[layer][ch]);
        }
    }
}

static void project(const OrTdt* d, const float* x, float* out) {
    for (int r = 0; r < DEC_H; r++) out[r] = d->proj_b[r] + dot16(d->proj_w + (size_t)r * DEC_H, x, DEC_H);
}

/* joint (src/tdt.rs:217-290): first maximum wins on ties.  When `gap` is
 * given it receives the decision margins of this step: gap[0] = best token
 * score - runner-up token score, gap[1] = the same over the durations. */
static void joint(const OrTdt* d, const float* enc, const float* dec, uint32_t* tok, uint32_t* dur, float* gap) {
    float s[DEC_H];
    for (int i = 0; i < DEC_H; i++) {
        float v = enc[i] + dec[i];
        s[i] = v > 0.0f ? v : 0.0f;
    }
    float bt = -INFINITY, bd = -INFINITY, st = -INFINITY, sd = -INFINITY;
    uint32_t it = 0, id = (uint32_t)d->vocab;
    int rows = d->vocab + N_DUR;
    for (int r = 0; r < rows; r++) {
        float score = d->head_b[r] + dot16(d->head_w + (size_t)r * DEC_H, s, DEC_H);
        if (r < d->vocab) {
            if (score > bt) { st = bt; bt = score; it = (uint32_t)r; }
            else if (score > st) st = score;
        } else if (score > bd) {
            sd = bd;
            bd = score;
            id = (uint32_t)r;
        } else if (score > sd) {
            sd = score;
        }
    }
    *tok = it;
    *dur = id - (uint32_t)d->vocab;
    if (gap) {
        gap[0] = bt - st;
        gap[1] = bd - sd;
    }
}

/* Greedy decode of one utterance (decode_rayon, src/tdt.rs:416-467).  out
 * receives (id, frame, dur) triples; returns the token count (capped at
 * max_tokens; the loop still runs to the end).  When `gaps` is given, step s
 * (s < max_gaps) writes its two decision margins to gaps[2s], gaps[2s+1] and
 * *n_steps receives the number of steps taken. */
static int tdt_decode_impl(const OrTdt* d, const float* pooler, int t_len, uint32_t* out, int max_tokens,
                           float* gaps, long max_gaps, long* n_steps) {
    const uint32_t blank = (uint32_t)d->vocab - 1;
    float h[2][DEC_H] = {{0}}, c[2][DEC_H] = {{0}}, dec[DEC_H];
    lstm_step(d, d->embed + (size_t)blank * DEC_H, h, c);
    project(d, h[1], dec);
    long max_steps = (long)t_len * (MAX_SYMBOLS + 4) + 64;
    long guard = 0;
    int n = 0, frame = 0;
    for (;;) {
        if (frame >= t_len) break;
        if (++guard > max_steps) break;
        uint32_t tok, dur;
        float* g = (gaps && guard <= max_gaps) ? gaps + 2 * (guard - 1) : NULL;
        joint(d, pooler + (size_t)frame * DEC_H, dec, &tok, &dur, g);
        if (tok == blank) {
            frame += dur > 0 ? (int)dur : 1;
        } else {
            if (n < max_tokens) {
                out[3 * n] = tok;
                out[3 * n + 1] = (uint32_t)frame;
                out[3 * n + 2] = dur;
            }
            n++;
            lstm_step(d, d->embed + (size_t)tok * DEC_H, h, c);
            project(d, h[1], dec);
            frame += (int)dur;
        }
    }
    if (n_steps) *n_steps = guard > max_steps ? max_steps : guard;
    return n;
}

int or_tdt_decode(const void* p, const float* pooler, int t_len, uint32_t* out, int max_tokens) {
    return tdt_decode_impl((const OrTdt*)p, pooler, t_len, out, max_tokens, NULL, 0, NULL);
}

/* The same decode, also recording each step's token and duration margins
 * (test statistics: how far every greedy decision is from a tie).  Returns
 * the token count; *n_steps receives the step count. */
int or_tdt_decode_margins(const void* p, const float* pooler, int t_len, uint32_t* out, int max_tokens,
                          float* gaps, long max_gaps, long* n_steps) {
    return tdt_decode_impl((const OrTdt*)p, pooler, t_len, out, max_tokens, gaps, max_gaps, n_steps);
}

/* Decodes n_utt utterances of a varlen pooler [total][640] (cu offsets), one
 * utterance per thread.  tokens: n_utt * max_tokens triples; counts: n_utt. */
void or_tdt_decode_batch(const void* p, const float* pooler, const int32_t* cu, int n_utt, uint32_t* tokens,
                         int32_t* counts, int max_tokens) {
#pragma omp parallel for schedule(dynamic, 1) num_threads(g_threads)
    for (int i = 0; i < n_utt; i++)
        counts[i] = or_tdt_decode(p, pooler + (size_t)cu[i] * DEC_H, cu[i + 1] - cu[i],
                                  tokens + (size_t)i * max_tokens * 3, max_tokens);
}

/* ───────────────────────────── front end ─────────────────────────────
 * Mel features (MelFrontend::compute, src/mel.rs:41-138) and the conv
 * subsampling (subsample, src/sub.rs:107-300), restated for parity tests
 * and the end-to-end CPU baseline. */

#define MEL_BINS 128
#define N_FFT 512
#define HOP 160
#define WIN 400

/* In-place radix-2 complex FFT of size 512 (double precision). */
static void fft512(double* re, double* im) {
    for (int i = 1, j = 0; i < N_FFT; i++) {
        int bit = N_FFT >> 1;
        for (; j & bit; bit >>= 1) j ^= bit;
        j ^= bit;
        if (i < j) {
            double t = re[i]; re[i] = re[j]; re[j] = t;
            t = im[i]; im[i] = im[j]; im[j] = t;
        }
    }
    for (int len = 2; len <= N_FFT; len <<= 1) {
        double ang = -2.0 * M_PI / len;
        for (int i = 0; i < N_FFT; i += len)
            for (int k = 0; k < len / 2; k++) {
                double wr = cos(ang * k), wi = sin(ang * k);
                double ur = re[i + k], ui = im[i + k];
                double vr = re[i + k + len / 2] * wr - im[i + k + len / 2] * wi;
                double vi = re[i + k + len / 2] * wi + im[i + k + len / 2] * wr;
                re[i + k] = ur + vr; im[i + k] = ui + vi;
                re[i + k + len / 2] = ur - vr; im[i + k + len / 2] = ui - vi;
            }
    }
}

/* wave: samples (the 0.25 s pad already prepended), fb: (128, 257) slaney
 * filterbank.  out: (n_frames, 128) normalised log-mel, frames >= n_valid
 * zero.  Returns n_frames; *n_valid_out = len / 160. */
int or_mel(const float* wave_in, int64_t len, const float* fb, float* out, int* n_valid_out) {
    float* wave = (float*)malloc((size_t)(len > 0 ? len : 1) * 4);
    for (int64_t i = 0; i < len; i++) wave[i] = i == 0 ? wave_in[0] : wave_in[i] - 0.97f * wave_in[i - 1];
    int n_frames = (int)(1 + len / HOP);
    int n_valid = (int)(len / HOP);
    float window[N_FFT] = {0};
    for (int i = 0; i < WIN; i++)
        window[(N_FFT - WIN) / 2 + i] = 0.5f * (1.0f - cosf(6.2831855f * (float)i / (float)(WIN - 1)));
    float* mel = (float*)malloc((size_t)MEL_BINS * n_frames * 4);
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int t = 0; t < n_frames; t++) {
        double re[N_FFT], im[N_FFT];
        int64_t start = (int64_t)t * HOP - N_FFT / 2;
        for (int i = 0; i < N_FFT; i++) {
            int64_t s = start + i;
            re[i] = (s >= 0 && s < len) ? (double)(wave[s] * window[i]) : 0.0;
            im[i] = 0.0;
        }
        fft512(re, im);
        float power[257];
        for (int k = 0; k < 257; k++) power[k] = (float)(re[k] * re[k] + im[k] * im[k]);
        for (int m = 0; m < MEL_BINS; m++) {
            const float* row = fb + m * 257;
            float s = 0.0f;
            for (int k = 0; k < 257; k++)
                if (row[k] != 0.0f) s += row[k] * power[k];
            mel[(size_t)m * n_frames + t] = logf(s + 5.9604645e-08f);
        }
    }
    int nv = n_valid > 1 ? n_valid : 1;
    for (int m = 0; m < MEL_BINS; m++) {
        float s = 0.0f;
        for (int t = 0; t < n_valid; t++) s += mel[(size_t)m * n_frames + t];
        float mean = s / (float)nv;
        float q = 0.0f;
        for (int t = 0; t < n_valid; t++) {
            float d = mel[(size_t)m * n_frames + t] - mean;
            q += d * d;
        }
        float sd = sqrtf(q / (float)(nv - 1 > 1 ? nv - 1 : 1) + 0.0f);
        for (int t = 0; t < n_frames; t++)
            out[(size_t)t * MEL_BINS + m] = t < n_valid ? (mel[(size_t)m * n_frames + t] - mean) / (sd + 1e-5f) : 0.0f;
    }
    free(mel);
    free(wave);
    if (n_valid_out) *n_valid_out = n_valid;
    return n_frames;
}

static int conv_len(int l) { return (l + 2 - 3) / 2 + 1; }

static void mask_time(float* x, int ch, int t, int m, int vlen) {
    if (vlen >= t) return;
    for (int c = 0; c < ch; c++)
        for (int i = vlen; i < t; i++)
            for (int j = 0; j < m; j++) x[((size_t)c * t + i) * m + j] = 0.0f;
}

/* depthwise 3x3 stride 2, padding 1 (src/sub.rs:173-201): s = b, then taps
 * ki, kj ascending, unfused, out-of-range taps skipped. */
static float* sub_dw(const float* x, const float* w, const float* b, int t_in, int m_in, int* t_out_p, int* m_out_p) {
    int t_out = conv_len(t_in), m_out = conv_len(m_in);
    float* out = (float*)malloc((size_t)256 * t_out * m_out * 4);
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int c = 0; c < 256; c++)
        for (int i = 0; i < t_out; i++)
            for (int j = 0; j < m_out; j++) {
                float s = b[c];
                for (int ki = 0; ki < 3; ki++) {
                    int ii = 2 * i + ki - 1;
                    if (ii < 0 || ii >= t_in) continue;
                    for (int kj = 0; kj < 3; kj++) {
                        int jj = 2 * j + kj - 1;
                        if (jj < 0 || jj >= m_in) continue;
                        s += w[c * 9 + ki * 3 + kj] * x[((size_t)c * t_in + ii) * m_in + jj];
                    }
                }
                out[((size_t)c * t_out + i) * m_out + j] = s;
            }
    *t_out_p = t_out;
    *m_out_p = m_out;
    return out;
}

/* pointwise 256 -> 256 (src/sub.rs:206-260): acc over ci ascending starting
 * at 0 (zero weights skipped), then (acc + b).max(0). */
static float* sub_pw(const float* x, const float* w, const float* b, int t, int m) {
    size_t p = (size_t)t * m;
    float* out = (float*)calloc((size_t)256 * p, 4);
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int co = 0; co < 256; co++) {
        float* o = out + (size_t)co * p;
        for (int ci = 0; ci < 256; ci++) {
            float wv = w[co * 256 + ci];
            if (wv == 0.0f) continue;
            const float* xr = x + (size_t)ci * p;
            for (size_t q = 0; q < p; q++) o[q] += wv * xr[q];
        }
        for (size_t q = 0; q < p; q++) {
            float v = o[q] + b[co];
            o[q] = v > 0.0f ? v : 0.0f;
        }
    }
    return out;
}

/* mel (f, 128) -> (T, 4096) with T = conv_len^3(f), row t = [c * 16 + m].
 * w0/w2/w5: (256, 9); w3/w6: (256, 256); b*: (256).  Returns T. */
int or_subsample(const float* mel, int f, int n_valid, const float* w0, const float* b0, const float* w2,
                 const float* b2, const float* w3, const float* b3, const float* w5, const float* b5,
                 const float* w6, const float* b6, float* out) {
    const int m0 = MEL_BINS;
    int f1 = conv_len(f), m1 = conv_len(m0);
    size_t p = (size_t)f1 * m1;
    float* x = (float*)malloc((size_t)256 * p * 4);
    /* layer 0 (src/sub.rs:110-167): bias, taps t = ki*3 + kj in order, ReLU */
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int co = 0; co < 256; co++)
        for (int i = 0; i < f1; i++)
            for (int j = 0; j < m1; j++) {
                float s = b0[co];
                for (int t = 0; t < 9; t++) {
                    int ki = t / 3, kj = t % 3;
                    int ii = 2 * i + ki, jj = 2 * j + kj;
                    float v = 0.0f;
                    if (ii > 0 && ii <= 2 * f && jj > 0 && jj <= 2 * m0) {
                        int si = ii - 1, sj = jj - 1;
                        if (si < f && sj < m0) v = mel[(size_t)si * m0 + sj];
                    }
                    s += w0[co * 9 + t] * v;
                }
                x[((size_t)co * f1 + i) * m1 + j] = s > 0.0f ? s : 0.0f;
            }
    int vlen = conv_len(n_valid > 1 ? n_valid : 1);
    mask_time(x, 256, f1, m1, vlen < f1 ? vlen : f1);
    int len, mlen;
    float* x2 = sub_dw(x, w2, b2, f1, m1, &len, &mlen);
    free(x);
    vlen = conv_len(vlen);
    mask_time(x2, 256, len, mlen, vlen < len ? vlen : len);
    float* x3 = sub_pw(x2, w3, b3, len, mlen);
    free(x2);
    int len2, mlen2;
    float* x4 = sub_dw(x3, w5, b5, len, mlen, &len2, &mlen2);
    free(x3);
    vlen = conv_len(vlen);
    mask_time(x4, 256, len2, mlen2, vlen < len2 ? vlen : len2);
    float* x5 = sub_pw(x4, w6, b6, len2, mlen2);
    free(x4);
    int t = len2;
    for (int c = 0; c < 256; c++)
        for (int i = 0; i < t; i++)
            for (int j = 0; j < mlen2; j++)
                out[(size_t)i * 256 * mlen2 + c * mlen2 + j] = x5[((size_t)c * t + i) * mlen2 + j];
    free(x5);
    return t;
}

/* ─────────────────────── .bark entropy coding (ANS) ───────────────────────
 * constriction 0.5.0, the crate src/bark.rs decodes the container with
 * (src/bark.rs:314-326, 398-421): `DefaultAnsCoder` = stack ANS over u32 words
 * with a u64 state; `DefaultContiguousCategoricalEntropyModel` = 24-bit
 * probabilities quantised by `from_floating_point_probabilities_fast`.  Its
 * published algorithm, restated: each symbol keeps one unit of mass and the
 * remaining 2^24 - n units follow the floor of the scaled running sum.  No
 * constriction-written stream or `.bark` file is available here, so these
 * restatements are checked only against each other and round trips
 * (parity unpinned).  The encoder exists to build test containers. */

int or_ans_cdf(const uint32_t* counts, int n, uint32_t* cdf) {
    if (n < 2 || n >= (1 << 24)) return -1;
    double total = 0.0, norm = 0.0, run = 0.0;
    for (int i = 0; i < n; i++) total += (double)counts[i];
    if (!(total > 0.0)) return -1;
    for (int i = 0; i < n; i++) norm += (double)counts[i] / total;
    if (!isnormal(norm) || norm < 0.0) return -1;
    double scale = (double)((1u << 24) - (uint32_t)n) / norm;
    for (int i = 0; i < n; i++) {
        cdf[i] = (uint32_t)(run * scale) + (uint32_t)i;
        run += (double)counts[i] / total;
    }
    cdf[n] = 1u << 24;
    return 0;
}

/* Pushes sym[n-1], ..., sym[0] (so a decoder pops them in order 0..n-1)
 * onto the coder (state, words[0..*n_words)).  Returns -1 when cap words
 * would be exceeded. */
int or_ans_push_reverse(uint64_t* state, uint32_t* words, int64_t* n_words, int64_t cap, const uint16_t* sym,
                        int64_t n, const uint32_t* cdf, int n_symbols) {
    uint64_t s = *state;
    int64_t w = *n_words;
    for (int64_t i = n - 1; i >= 0; i--) {
        int c = sym[i];
        if (c < 0 || c >= n_symbols) return -2;
        uint64_t lo = cdf[c], p = (uint64_t)cdf[c + 1] - lo;
        if ((s >> 40) >= p) {
            if (w >= cap) return -1;
            words[w++] = (uint32_t)s;
            s >>= 32;
        }
        s = ((s / p) << 24) | (s % p + lo);
    }
    *state = s;
    *n_words = w;
    return 0;
}

/* Final state onto the stack, low word first (the top word is never zero). */
int or_ans_flush(uint64_t* state, uint32_t* words, int64_t* n_words, int64_t cap) {
    uint64_t s = *state;
    int64_t w = *n_words;
    while (s) {
        if (w >= cap) return -1;
        words[w++] = (uint32_t)s;
        s >>= 32;
    }
    *state = 0;
    *n_words = w;
    return 0;
}

/* Decoder with a caller-held position: *top words are still on the stack.
 * or_ans_open returns -1 for a zero top word. */
int or_ans_open(const uint32_t* words, int64_t* top, uint64_t* state) {
    *state = 0;
    if (*top == 0) return 0;
    uint32_t first = words[--*top];
    if (first == 0) return -1;
    uint64_t s = first;
    while (*top > 0 && s < ((uint64_t)1 << 32)) s = (s << 32) | words[--*top];
    *state = s;
    return 0;
}

void or_ans_pop(const uint32_t* words, int64_t* top, uint64_t* state, const uint32_t* cdf, int n_symbols,
                uint16_t* out, int64_t n) {
    uint64_t s = *state;
    int64_t t = *top;
    for (int64_t i = 0; i < n; i++) {
        uint32_t q = (uint32_t)(s & 0xFFFFFF);
        int c = 0;
        while (c + 1 < n_symbols && cdf[c + 1] <= q) c++;
        s = (s >> 24) * (uint64_t)(cdf[c + 1] - cdf[c]) + (q - cdf[c]);
        if (s < ((uint64_t)1 << 32) && t > 0) s = (s << 32) | words[--t];
        out[i] = (uint16_t)c;
    }
    *state = s;
    *top = t;
}
