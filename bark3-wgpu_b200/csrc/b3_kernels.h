// b3_kernels.h — host launchers of the non-GEMM kernels.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b3 {

// K4: y = LN1(x) -> y32 (may alias x, may be null); then f16 output of
// LN2(y) (w2 non-null) or of y itself (w2 null) -> y16 (may be null).
int launch_layernorm(const float* x, int rows, const float* w1, const float* b1, float* y32,
                     const float* w2, const float* b2, __half* y16, cudaStream_t st);

// K3b: depthwise conv (taps dw_t [9][1024]) + folded BN + SiLU; seg[t] is the
// [start, end) row range of frame t's utterance.
int launch_dwconv(const __half* src, const int2* seg, int rows, const float* dw_t, const float* bn_a,
                  const float* bn_b, __half* dst, cudaStream_t st);

int launch_f32_to_f16(const float* src, __half* dst, int64_t n, cudaStream_t st);

// Relative-position table: `rows` rows, row j = position tcap - 1 - j.
int launch_pos_table(const float* inv_freq, int tcap, int rows, __half* out, cudaStream_t st);

struct AttnParams {
    const __half* qkv;   // [M][4096] = qu | qv | k | v (f16)
    const __half* R;     // [r_rows][1024] relative-position keys
    int r_center;        // row of R holding offset 0; row r_center - d holds offset d
    int r_rows;
    const int4* work;    // device (first row of the utterance, its frames, first query, 0) per work entry
    __half* out;         // [M][1024]
    float scale_log2;    // log2(e) / sqrt(128)
};

// attention_tc.cu: M rows in the qkv buffer.
int launch_attention_tc(const AttnParams& p, int M, int n_work, cudaStream_t st);
int attention_tc_block_rows();
int attention_take_dev_error(cudaStream_t st, unsigned int* out);

// Batched greedy TDT decoder state (tdt_decoder.cu).  B rows, one per
// utterance; GEMM inputs are f16 hi | lo pairs (see tdt_decoder.cu).
struct DecState {
    int B, vocab, blank, max_tokens;
    const int* row0;         // [B] first pooler row of each utterance
    const int* len;          // [B] encoder frames of each utterance
    const float* pooler;     // [total][640]
    const float* e0;         // [vocab][2560] W_ih0 . emb(token) + b_ih0 + b_hh0
    int* tok;                // [B] last emitted token (blank before the first)
    __half* a0;              // [B][1280] h0_hi | h0_lo                 (LSTM layer 0 input)
    __half* a1;              // [B][2560] h0_hi | h0_lo | h1_hi | h1_lo (layer 1 input)
    __half* ap;              // [B][1280] h1_hi | h1_lo                 (projector input)
    __half* aj;              // [B][1280] joint input hi | lo
    // split-K GEMM outputs: part p of a GEMM with output [B][n] sits at
    // rows [p * prow, p * prow + B); the consumer adds the parts in order
    float* gates;            // layer gates, n = 2560
    float* dec;              // projector output, n = 640
    float* scores;           // joint head, n = ld_scores
    float* c;                // [B][2][640]
    int prow;                // rows per part
    int ks_g0, ks_g1, ks_p, ks_h;  // parts of the layer 0 / layer 1 / projector / head GEMMs
    int ld_scores;
    int *frame, *count, *guard, *emit, *active;
    uint32_t* tokens;        // [B][max_tokens][3] (id, frame, duration)
};

// One GEMM of the persistent decoder: out[B][N] (+)= A[B][K] . W[N][K]^T,
// where A holds [hi | lo] f16 halves per 640-wide segment and W matches them
// ([W_seg | W_seg]), so the logical K is half the stored one.  128 x bn tiles
// (bn 128 or 256), the logical K cut into `ks` parts of `nkb` 64-wide
// k-blocks; part p lands at rows [p * prow, p * prow + B), part 0 adds `bias`.
struct DecGemm {
    int m_tiles, n_tiles, bn, ks, nkb;
    float* out;
    int ldo;
    const float* bias;
};

// Maps of the persistent decoder's GEMMs, indexed like DecPersist::g:
// A over the activation rows, B over the f16 weights (box 64 x 128 / 64 x 64),
// C over the f32 split-K parts (box 32 x 32, 128-byte swizzle).
struct alignas(64) DecMaps {
    CUtensorMap a[4];
    CUtensorMap b[4];
    CUtensorMap c[4];
};

// The whole greedy decode of one batch in one cooperative launch.
struct DecPersist {
    DecState s;
    DecGemm g[4];        // kDecHead, kDecLstm0, kDecLstm1, kDecProj
    unsigned int* sync;  // [0] barrier arrivals, [1] abort flag,
                         // [4..5] active-row counts of even / odd steps (8 words, host-zeroed)
    int max_steps;       // lock steps at most (every row is bounded on its own as well)
    unsigned long long grid_wait_ns;   // wall-time bound of each grid-barrier wait
};
constexpr int kDecHead = 0, kDecLstm0 = 1, kDecLstm1 = 2, kDecProj = 3;

// CTAs of the persistent decoder that fit on the device at once (0 if none).
int dec_persistent_grid(int device);
int dec_launch_persistent(const DecMaps& maps, const DecPersist& p, int grid, cudaStream_t st);
// Tile widths and splits of the four GEMMs for `grid` CTAs (DecPersist::g order).
void dec_plan_persistent(int B, int npad, int grid, int bn[4], int ks[4]);
int dec_launch_init(const DecState& s, cudaStream_t st);
int dec_launch_split(const float* src, __half* hi, __half* lo, int64_t n, cudaStream_t st);
// Reads and clears the decoder's device error word (stream-ordered).
int decoder_take_dev_error(cudaStream_t st, unsigned int* out);

// Weight-stationary lock-step decoder (batches up to 2 x 128 rows).  Every
// CTA owns one 128-row tile of one weight matrix for the whole decode, kept
// in shared memory; tiles are numbered head (head_tiles), layer-0 recurrent
// (20), layer-1 recurrent (20), layer-1 input (20), projector (5).  The LSTM
// tiles hold 32 channels x 4 gates (rows i | f | g | o of channels
// [32 t, 32 t + 32)), so a tile's owner applies the cell to its channels.
// With nsplit = 2 the batch rows are cut in two halves of `ntile` rows and
// every tile has one CTA per half.
constexpr int kWsLstmTiles = 20;
constexpr int kWsProjTiles = 5;
struct DecWs {
    int B, vocab, blank, max_tokens;
    int head_tiles, n_roles, ntile, bpad, kc, max_steps;   // kc: k-blocks per TMA box
    const int* row0;         // [B] first pooler row of each utterance
    const int* len;          // [B] encoder frames of each utterance
    const float* pooler;     // [total][640]
    const float* e0;         // [vocab][2560] W_ih0 . emb(token) + b_ih0 + b_hh0 (gate order i | f | g | o)
    const float* bias;       // head [head_tiles * 128] | layer 1 [2560] (b_ih1 + b_hh1) | projector [640]
    __half *act0, *act1, *aj;   // h0, h1 and the joint input as f16 hi | lo: [10 k-blocks][hi, lo][bpad][64]
    float* c;                // [B][2][640] cell states
    float* g1p;              // [bpad][2560] recurrent half of the layer-1 gates (W_hh1 . h1)
    unsigned long long* keys;   // [2 step parities][2: token, duration][B] argmax keys
    int *frame, *count, *guard;  // [B] each
    int* alive;              // [2 step parities][B]
    uint32_t* tokens;        // [B][max_tokens][3] (id, frame, duration)
    unsigned int* sync;      // [0] barrier arrivals, [1] abort flag, [4..5] alive counts by step parity
    unsigned long long grid_wait_ns;
};
struct alignas(64) DecWsMaps {
    CUtensorMap w;                 // [n_roles * 128][640] f16 weight tiles, box 64 x 128
    CUtensorMap act0, act1, aj;    // 3D (64, bpad, 20 panels) f16, box 64 x ntile x 2 kc
};
// CTAs of one weight-stationary decode (0 if it does not fit this device).
int dec_ws_grid(int device, int n_roles, int nsplit);
int dec_ws_launch(const DecWsMaps& maps, const DecWs& p, int grid, cudaStream_t st);

// Mel front end (frontend.cu).
struct MelParams {
    int n_utt;
    int lead;                 // zero samples before each utterance (not stored)
    const float* wave;        // waves, concatenated
    const int64_t* wave_off;  // [n_utt + 1] sample offsets
    const int* frame_off;     // [n_utt + 1] frame offsets (1 + len/160 frames each)
    const float* window;      // [512] Hann(400) centred
    const float2* twiddle;    // [256] exp(-2 pi i k / 512)
    const float* fb;          // [128][257] slaney filterbank
    const int* fb_lo;         // [128] first nonzero bin of each filter
    const int* fb_hi;         // [128] one past the last
    const int* fb_off;        // [129] start of filter m's span in fb_pack
    const float* fb_pack;     // the filters' nonzero spans, packed end to end
    int fb_total;             // fb_off[128]
    float* mel;               // [frames][128]
};

// Conv subsampling (frontend.cu); activations channels-last, f16.
struct SubParams {
    int n_utt;
    const float* mel;         // [frames][128]
    const int* mel_off;       // [n_utt + 1]
    const int* n_valid;       // [n_utt] valid mel frames
    const int4* work;         // per item: (first mel row, mel frames, valid frames, first t2 row),
                              // (first x2 row, channel group, 0, 0)
    const float *w0, *b0, *w2, *b2, *w5, *b5;  // conv0 and the two depthwise convs, [256][9] + [256]
    __half* x2;               // [sum F2][32][256]  after depthwise 1
    const __half* x3;         // [sum F2][32][256]  after pointwise 1
    __half* x4;               // [sum T][16][256]   after depthwise 2
    const int* x2_off;        // [n_utt + 1] row offsets of x2 / x3
    const int* x4_off;        // [n_utt + 1] row offsets of x4 (= encoder frames)
    const int4* rows3;        // per x4 row: (first x2 row of its utterance, depthwise-1 rows,
                              // valid x4 rows, row within the utterance)
};

// The front-end kernels over a range of the batch: mel frames [f0, f1) and
// the normalisation of utterances [u0, u1); conv work items [w0, w1); second
// depthwise-conv rows [r0, r1).
int launch_mel(const MelParams& p, int f0, int f1, int u0, int u1, cudaStream_t st);
int launch_sub_conv0_dw1(const SubParams& p, int w0, int w1, cudaStream_t st);
int launch_sub_dw2(const SubParams& p, int r0, int r1, cudaStream_t st);
int launch_sub_to_ref(const __half* src, float* dst, int rows, cudaStream_t st);
int sub_work_rows();
int sub_work_channels();

}  // namespace b3
