/*
 * bark3_b200.h — C ABI of the B200 (sm_100a) encoder for bark3-wgpu.
 *
 * This is the drop-in boundary for the reference crate's encoder seam.  A Rust
 * (or any FFI) host binds these `extern "C"` functions in place of the wgpu
 * encoder; everything is plain pointers, sizes and integer status codes.
 *
 * Conventions
 *   - Every function returns 0 (B3_OK) or a negative B3_E* code.  The message
 *     for the most recent failure on the calling thread is b3_last_error().
 *     Nothing aborts or throws across this boundary (the reference panics on a
 *     missing tensor, src/encoder.rs:419; this ABI returns B3_ENOTFOUND).
 *   - Host buffers are borrowed for the duration of the call.  Device weights
 *     and the activation arena belong to the context.
 *   - One context per GPU; calls on one context must be serialised (the
 *     reference AsrInference is effectively !Sync, src/encoder/prof.rs:22-28,
 *     src/gpu.rs:608).  Use one host thread per context for several GPUs.
 *   - With B3_DEVICE_PTRS the data pointers are device pointers on the
 *     context's GPU and the call only enqueues work on the context stream;
 *     b3_sync() waits for it.  Without the flag the pointers are host memory
 *     and the call returns when the results are in host memory.
 *   - Layouts: row-major, f32 unless stated.  f16 / bf16 are raw 16-bit
 *     patterns (uint16_t).
 */
#ifndef BARK3_B200_H
#define BARK3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B3_OK 0
#define B3_EINVAL (-1)     /* bad argument, shape or layout */
#define B3_ENOMEM (-2)     /* host or device allocation failed */
#define B3_ECUDA (-3)      /* CUDA runtime / driver error */
#define B3_ETIMEOUT (-4)   /* a device-side bounded wait ran out */
#define B3_ESTATE (-5)     /* call out of order (e.g. encode before finalize) */
#define B3_ENOTFOUND (-6)  /* a required tensor was never loaded */

#define B3_DEVICE_PTRS 1u  /* data pointers are device pointers (async) */

/* Tensor element types for b3_load_tensor. */
#define B3_DTYPE_F32 0
#define B3_DTYPE_F16 1
#define B3_DTYPE_BF16 2

typedef struct b3_ctx b3_ctx;

/* Message of the last failed call on this thread ("" if none). */
const char* b3_last_error(void);

/* ABI version, major * 10000 + minor * 100 + patch. */
int b3_version(void);

/* Context on CUDA device `device`: stream, weight store, activation arena.
 * Replaces Gpu::new_with + Encoder::load_with's device setup
 * (src/gpu.rs:448, src/encoder.rs:412).  NULL on failure. */
b3_ctx* b3_create(int device);
void b3_destroy(b3_ctx* ctx);

/* Wait for all work enqueued on the context stream; reports device-side
 * errors (B3_ETIMEOUT) raised by the kernels since the last check. */
int b3_sync(b3_ctx* ctx);

/* The context's cudaStream_t, for callers that order their own work after
 * B3_DEVICE_PTRS calls. */
void* b3_stream(b3_ctx* ctx);

/* Wall-time bound, in nanoseconds, of each grid-barrier wait of the greedy
 * decoder's persistent kernel (default 2 s; grid_barrier_ns <= 0 restores
 * it).  A wait that runs out raises the kernel's abort flag, every CTA leaves
 * at its next barrier with its own copies and MMAs complete, and the call
 * returns B3_ETIMEOUT; the context stays usable.  This is the device-side
 * counterpart of the reference GPU decoder's exit code and step guard
 * (src/tdt_gpu.rs:62-70, src/tdt.rs:422-424); a short bound lets a test make
 * the wait run out without faulting anything. */
int b3_set_wait_limit(b3_ctx* ctx, int64_t grid_barrier_ns);

/* Which greedy-decoder kernel decodes a batch.  B3_DECODER_AUTO (the
 * default): batches of up to 128 utterances run on the weight-stationary
 * kernel (every CTA keeps one 128-row weight tile in shared memory for the
 * whole decode; four grid barriers per lock step), larger ones on the
 * split-K kernel.  B3_DECODER_SPLIT_K: every batch on the split-K kernel
 * (weights streamed from L2 each step, six barriers per step).  Both follow
 * the reference's greedy rule (src/tdt.rs:416-467); the choice changes speed,
 * not the decoding rule. */
#define B3_DECODER_AUTO 0
#define B3_DECODER_SPLIT_K 1
int b3_set_decoder(b3_ctx* ctx, int kind);

/* ───────────────────────── weight loading ─────────────────────────
 * Tensors are pushed by the reference checkpoint's names, the way
 * Encoder::load_with pulls them from a WeightSource (src/weights.rs:22-36,
 * src/encoder.rs:412-640).  A Rust host iterates its WeightSource and calls:
 *   - b3_load_tensor for dense tensors (`WeightSource::read`, any of f32 /
 *     f16 / bf16; matrices are rounded to f16 exactly as src/raw.rs:68-97 and
 *     src/cpu/mod.rs:35-37 do),
 *   - b3_load_lowbit / b3_load_lowbit_levels for 4-bit layers
 *     (`WeightSource::read_lowbit`, src/bark.rs:33-48),
 * then b3_finalize once. */
int b3_load_tensor(b3_ctx* ctx, const char* name, int dtype, const int64_t* shape, int ndim,
                   const void* data);

/* 4-bit layer as codes packed two per byte (low nibble = even column; this is
 * byte-for-byte the reference's u32 words, eight nibbles low-first,
 * src/bark.rs:352-358) plus a per-row 16-entry f16 level table:
 * codes [rows][cols/2], lut16 [rows][16].  cols must be even. */
int b3_load_lowbit(b3_ctx* ctx, const char* name, const uint8_t* codes, const uint16_t* lut16,
                   int rows, int cols);

/* The reference's LowBitTensor as is (src/bark.rs:33-48): code_words
 * [rows][ceil(cols/8)] u32, levels [rows][4] f16 with the first k (1..3) in
 * use.  Converted at load to the 16-entry table with the sign-magnitude rule
 * of `expand` (src/bark.rs:597-611): 0 -> 0, 1..k -> +lev, k+1..2k -> -lev,
 * codes above 2k -> 0. */
int b3_load_lowbit_levels(b3_ctx* ctx, const char* name, const uint32_t* code_words,
                          const uint16_t* levels, int k, int rows, int cols);

/* Build the device-resident encoder from the loaded tensors: fused q|k|v
 * (src/encoder.rs:342-402), BatchNorm fold (src/cpu/mod.rs:103-119),
 * GLU row interleave for pw1, transposed depthwise taps.  `n_layers` is the
 * block count to expect (24 for the released models). */
int b3_finalize(b3_ctx* ctx, int n_layers);

/* ───────────────────────────── encoder ─────────────────────────────
 * One utterance, the CpuEncoder::encode contract (src/cpu/mod.rs:156-188):
 * sub [t][4096] are the conv-subsampled frames; with layers >= n_layers the
 * result is the pooler [t][640] (projector 1024 -> 640 + bias), otherwise the
 * pre-norm_out residual [t][1024] of block `layers - 1` (the reference's
 * h_b{n} dump point). */
int b3_encode(b3_ctx* ctx, const float* sub, int t, int layers, float* out, unsigned flags);

/* Varlen batch: utterance i occupies rows cu_seqlens[i] .. cu_seqlens[i+1]
 * of sub [total][4096] and pooler [total][640].  Attention and the depthwise
 * conv stay inside each utterance; linears run over the concatenation.
 * cu_seqlens is always host memory (n_utt + 1 entries, starting at 0).
 * Both encode calls, at up to 8192 rows, replay a CUDA graph of their launches
 * when the same call (rows, buffers, block count) is repeated: the second such
 * call captures it on the context's stream, later ones replay it. */
int b3_encode_batch(b3_ctx* ctx, const float* sub, const int32_t* cu_seqlens, int n_utt,
                    float* pooler, unsigned flags);

/* ──────────────────────────── TDT decoder ────────────────────────────
 * Greedy TDT decoding (TdtDecoder::decode, src/tdt.rs:319-467) of every
 * utterance of a batch in lock step on the GPU.  The decoder is built by
 * b3_finalize when its tensors were loaded: decoder.embedding.weight
 * (vocab, 640) — the last row is the blank —, decoder.lstm.{weight_ih,
 * weight_hh}_l{0,1} (2560, 640), decoder.lstm.{bias_ih,bias_hh}_l{0,1},
 * decoder.decoder_projector.{weight,bias}, joint.head.weight
 * (vocab + 5, 640) and joint.head.bias; the 5 rows after the vocabulary are
 * the durations 0..4.
 *
 * One emitted token (src/tdt.rs:33-41): id, frame at emission, duration. */
typedef struct b3_token {
    uint32_t id;
    uint32_t frame;
    uint32_t dur;
} b3_token;

/* pooler [total][640] with utterance i at rows cu_seqlens[i] ..
 * cu_seqlens[i+1]; tokens [n_utt][max_tokens]; counts[i] = tokens utterance
 * i emitted (may exceed max_tokens: only the first max_tokens are stored).
 * With B3_DEVICE_PTRS pooler, tokens and counts are device pointers. */
int b3_decode_batch(b3_ctx* ctx, const float* pooler, const int32_t* cu_seqlens, int n_utt,
                    b3_token* tokens, int32_t* counts, int max_tokens, unsigned flags);

/* Encoder + decoder in one call: subsampled frames sub [total][4096] ->
 * tokens (the batched transcription step of BASELINE config 5 from the
 * encoder input on). */
int b3_transcribe_batch(b3_ctx* ctx, const float* sub, const int32_t* cu_seqlens, int n_utt,
                        b3_token* tokens, int32_t* counts, int max_tokens, unsigned flags);

/* ──────────────────────────── front end ────────────────────────────
 * The mel front end (MelFrontend::compute, src/mel.rs:41-138) and the conv
 * subsampling (subsample, src/sub.rs:107-300) on the GPU.  The subsampling
 * is built by b3_finalize when encoder.subsampling.layers.{0,2,3,5,6}.
 * {weight,bias} were loaded.
 *
 * Batched transcription from audio, the AsrInference::transcribe_samples
 * pipeline (src/inference.rs:446, src/transcription.rs:21-260) for many
 * utterances at once: 16 kHz mono samples, utterance i at
 * samples[offsets[i] .. offsets[i+1]] (offsets host, n_utt + 1 entries); the
 * 0.25 s of leading silence the reference prepends is added here.  Tokens as
 * for b3_decode_batch (frames count from the start of the padded audio). */
int b3_transcribe_audio(b3_ctx* ctx, const float* samples, const int64_t* offsets, int n_utt,
                        b3_token* tokens, int32_t* counts, int max_tokens, unsigned flags);

/* The encoder half of b3_transcribe_audio (Encoder::encode_pre's pooler,
 * src/encoder.rs:2005, from audio): pooler [sum T][640] f32 for the same
 * audio, row_offsets (host, n_utt + 1) the per-utterance encoder rows.
 * max_rows is the capacity of pooler in rows (B3_EINVAL if too small).  The
 * pooler is exactly what b3_transcribe_audio decodes. */
int b3_encode_audio(b3_ctx* ctx, const float* samples, const int64_t* offsets, int n_utt, float* pooler,
                    int32_t* row_offsets, int64_t max_rows, unsigned flags);

/* Log-mel features of already padded waves: mel [sum frames][128],
 * frame_offsets (host, n_utt + 1) receives the per-utterance frame offsets
 * (1 + len / 160 frames each; frames past len / 160 are zero). */
int b3_mel(b3_ctx* ctx, const float* wave, const int64_t* offsets, int n_utt, float* mel,
           int32_t* frame_offsets, unsigned flags);

/* Conv subsampling of mel features (frame_offsets and n_valid host):
 * sub [sum T][4096] in the reference's row order (channel * 16 + freq), f32;
 * row_offsets (host, n_utt + 1) receives the per-utterance T offsets,
 * T = conv_len^3(frames), conv_len(l) = (l - 1) / 2 + 1. */
int b3_subsample(b3_ctx* ctx, const float* mel, const int32_t* frame_offsets, const int32_t* n_valid,
                 int n_utt, float* sub, int32_t* row_offsets, unsigned flags);

/* The 128 x 257 slaney mel filterbank the front end uses (host copy). */
int b3_mel_filters(float* out);

/* ─────────────────────────── single kernels ───────────────────────────
 * one 4-bit linear, c[m][n] = a[m][:] . W[n][:] + bias[n]
 * with W from codes [n][k/2] + lut16 [n][16].  Replaces Ctx::gemm_f32 with a
 * low-bit weight + add_bias_f32 (src/encoder.rs:1039-1100, 2078).
 * k must be a multiple of 64 and n of 128; bias may be NULL. */
int b3_linear_lut4(b3_ctx* ctx, const float* a, const uint8_t* codes, const uint16_t* lut16,
                   const float* bias, float* c, int m, int n, int k, unsigned flags);

/* Same with a dense f16 weight w16 [n][k] (the Pro layout after the
 * reference's bf16 -> f16 rounding).  With the weights of b3_linear_lut4
 * expanded through their tables this returns bit-identical results (the
 * reference's lbtest, src/diagnostics/gemm.rs:538-652). */
int b3_linear_f16(b3_ctx* ctx, const float* a, const uint16_t* w16, const float* bias, float* c,
                  int m, int n, int k, unsigned flags);

/* Allocation-free twin of b3_linear_lut4 for callers that must not allocate
 * device memory: latency-critical threads (cudaMalloc / cudaFree can
 * synchronise the device) and hosts that account for all GPU memory in their
 * own pool.  No counterpart in the reference.  All pointers are device
 * pointers; the work is enqueued on `stream` (a cudaStream_t, NULL = legacy
 * default stream) of the current device, and nothing is allocated.  The f16
 * copy of `a` is staged in a fixed 8 MiB scratch array inside the library
 * (held by every GPU that loads it until exit), so m * k <= 4194304; larger
 * calls fail with B3_EINVAL.  The first call on a device looks the scratch
 * address up (cudaGetSymbolAddress); make it before any stream capture.
 * Calls whose work overlaps on one GPU race on the shared scratch. */
int b3_linear_lut4_noalloc(const float* a, const uint8_t* codes, const uint16_t* lut16,
                           const float* bias, float* c, int m, int n, int k, void* stream);

/* BASELINE config 4: the attention and conv sections of block `layer`
 * (src/cpu/layer.rs:198-310) on one sequence, in place:
 *   x += MHSA(LN_att(x));  x += Conv(LN_conv(x)).
 * x is [t][1024]. */
int b3_attn_conv(b3_ctx* ctx, int layer, float* x, int t, unsigned flags);

/* ─────────────────────── .bark container streams ───────────────────────
 * Host-only entropy decoding of the `model.bark` weight container (no GPU
 * work; callable without a device).  The container's JSON index, LZMA fields
 * and level tables are parsed by the caller (bark3-wgpu_b200/bark.py mirrors
 * BarkContainer, src/bark.rs:98-560); these calls replace its constriction
 * 0.5.0 ANS decoding: a stack ANS coder with u32 words and a u64 state over a
 * 24-bit categorical model quantised by from_floating_point_probabilities_fast.
 * Malformed input returns B3_EINVAL with the reference's message. */

/* The model's quantised cumulative table: cdf[0..n_symbols] (cdf[n] = 2^24). */
int b3_bark_ans_cdf(const uint32_t* counts, int n_symbols, uint32_t* cdf);

/* n i.i.d. symbols of one model from one stream (decode_iid_symbols). */
int b3_bark_ans_decode(const uint32_t* counts, int n_symbols, const uint32_t* words, int64_t n_words,
                       int64_t n, uint16_t* symbols);

/* A "levels2" entry (decode_levels2, src/bark.rs:277-366): meta = column
 * classes (4 bits per column, high nibble even) then 16 x (2k+1) u32 counts;
 * words = the ANS stream.  Writes rows x ceil(cols/8) code words, nibble
 * col % 8 of word col / 8 — the layout b3_load_lowbit_levels takes. */
int b3_bark_decode_levels2(const uint8_t* meta, int64_t meta_bytes, const uint32_t* words, int64_t n_words,
                           int rows, int cols, int k, uint32_t* code_words);

/* An "ansint<bits>" entry (src/bark.rs:387-431): out[i] = (symbol_i -
 * (2^(bits-1) - 1)) * f16 row_scales[i / (n / rows)]. */
int b3_bark_decode_ansint(const uint32_t* counts, int n_symbols, const uint32_t* words, int64_t n_words,
                          int64_t n, int bits, const uint16_t* row_scales, int64_t rows, float* out);

/* ──────────────────────────── multi-GPU ────────────────────────────
 * Utterance sharding for one process (or host thread) per GPU.  The reference
 * is single-device; utterances are independent, so a batch is split across
 * GPUs with no collective.  rank_of[i] receives the rank (0..n_ranks-1) that
 * encodes utterance i, chosen longest-processing-time first by the estimated
 * encoder cost c(T) = 52.4e6 T + 6144 T^2 (FLOPs per block; ties go to the
 * lower rank).  Pure host code. */
int b3_shard_lpt(const int32_t* frames, int n_utt, int n_ranks, int32_t* rank_of);

/* ───────────────────────────── profiling ─────────────────────────────
 * Per-kernel-class device timing with CUDA events on the context stream, the
 * counterpart of the reference's BARK3_ENC_PROFILE timestamp queries
 * (src/encoder/prof.rs:1-121).  b3_profile(ctx, 1) resets the counters and
 * starts recording; b3_profile_read waits for the stream and returns, for one
 * kernel class, the summed device milliseconds, algorithmic FLOPs and DRAM
 * bytes of the timed launches and the number of launches issued since the
 * last reset (launches are counted even while recording is off). */
#define B3_K_GEMM_LUT4 0
#define B3_K_GEMM_F16 1
#define B3_K_ATTENTION 2
#define B3_K_LAYERNORM 3
#define B3_K_DWCONV 4
#define B3_K_CONVERT 5
#define B3_K_OTHER 6
#define B3_K_DECODER 7
#define B3_K_FRONTEND 8
#define B3_K_COUNT 9

int b3_profile(b3_ctx* ctx, int enable);
int b3_profile_read(b3_ctx* ctx, int kind, double* ms, double* flops, double* bytes, int64_t* launches);

#ifdef __cplusplus
}
#endif

#endif /* BARK3_B200_H */
