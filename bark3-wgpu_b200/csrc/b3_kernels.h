// b3_kernels.h — host launchers of the non-GEMM kernels.
#pragma once
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
    const int* cu;       // device cu_seqlens [n_utt + 1]
    const int2* work;    // device (utterance, first query) per CTA
    __half* out;         // [M][1024]
    float scale_log2;    // log2(e) / sqrt(128)
};

int launch_attention(const AttnParams& p, int n_work, cudaStream_t st);
int attention_block_rows();

}  // namespace b3
