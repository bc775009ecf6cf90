// Entropy decoding for the `.bark` weight container (host code, no device
// work).  The container stores each 4-bit encoder linear as one rANS stream of
// per-weight codes and each integer matrix as one rANS stream of quantised
// values; these entry points turn a stream into the layouts the encoder loads
// (b3_load_lowbit_levels) or into f32 values.
//
// The stream format is the one the reference decodes with constriction 0.5.0
// (src/bark.rs:277-366 and 387-431): constriction's `DefaultAnsCoder` (a stack
// ANS coder with 32-bit words and a 64-bit state) and its
// `DefaultContiguousCategoricalEntropyModel` (24-bit probabilities) built by
// `from_floating_point_probabilities_fast`.  The published algorithms,
// restated:
//
//   model   p_i = count_i / sum(count) in f64; norm = sum_i p_i (left to
//           right); free = 2^24 - n; scale = free / norm;
//           cdf_i = floor(scale * (p_0 + ... + p_{i-1})) + i, cdf_n = 2^24
//           (every symbol keeps at least one unit of probability mass).
//   start   the compressed words form a stack whose top is the last word.  An
//           empty stack gives state 0; a zero top word is malformed; else the
//           state takes the top word, then further words (state << 32 | w)
//           until it reaches 2^32.
//   decode  q = state mod 2^24; symbol s with cdf_s <= q < cdf_{s+1};
//           state = (state >> 24) * (cdf_{s+1} - cdf_s) + (q - cdf_s);
//           if state < 2^32 and a word is left: state = state << 32 | pop().
//
// An exhausted stack is not an error (the coder keeps decoding from its
// state), exactly as the reference's Vec-backed coder behaves.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "b3_internal.h"

namespace b3 {
namespace {

constexpr int kPrecision = 24;
constexpr uint32_t kOne = 1u << kPrecision;
constexpr int kBucketBits = 12;

// bucket[j] = the symbol whose interval holds quantile j << (24 - 12).
void ans_buckets(const uint32_t* cdf, int n, uint8_t* bucket) {
    int s = 0;
    for (uint32_t j = 0; j < (1u << kBucketBits); ++j) {
        const uint32_t q = j << (kPrecision - kBucketBits);
        while (s + 1 < n && cdf[s + 1] <= q) ++s;
        bucket[j] = static_cast<uint8_t>(s);
    }
}

// Quantised cumulative table (n + 1 entries) for counts[0..n).  Returns false
// when the table cannot form a model.
bool ans_cdf(const uint32_t* counts, int n, uint32_t* cdf) {
    if (n < 2 || static_cast<uint32_t>(n) >= kOne) return false;
    double total = 0.0;
    for (int i = 0; i < n; ++i) total += static_cast<double>(counts[i]);
    if (!(total > 0.0)) return false;
    std::vector<double> p(n);
    double norm = 0.0;
    for (int i = 0; i < n; ++i) {
        p[i] = static_cast<double>(counts[i]) / total;
        norm += p[i];
    }
    if (!std::isnormal(norm) || norm < 0.0) return false;
    const double scale = static_cast<double>(kOne - static_cast<uint32_t>(n)) / norm;
    double cum = 0.0;
    for (int i = 0; i < n; ++i) {
        const double left = cum * scale;
        cdf[i] = static_cast<uint32_t>(left) + static_cast<uint32_t>(i);
        cum += p[i];
    }
    cdf[n] = kOne;
    return true;
}

struct AnsStack {
    const uint32_t* words;
    int64_t top;  // words[0..top) are still on the stack
    uint64_t state;

    // false: the stream's top word is zero, which no coder writes.
    bool open(const uint32_t* w, int64_t n) {
        words = w;
        top = n;
        state = 0;
        if (top == 0) return true;
        const uint32_t first = words[--top];
        if (first == 0) return false;
        state = first;
        while (top > 0 && state < (uint64_t{1} << 32)) state = (state << 32) | words[--top];
        return true;
    }

    // Same as decode(), with the symbol found from a table of the symbol at
    // the start of each 2^-12 quantile bucket, then stepped forward over the
    // (rare) boundaries inside the bucket.
    inline int decode_lut(const uint32_t* cdf, const uint8_t* bucket) {
        const uint32_t q = static_cast<uint32_t>(state) & (kOne - 1);
        int s = bucket[q >> (kPrecision - kBucketBits)];
        while (cdf[s + 1] <= q) ++s;
        state = (state >> kPrecision) * (cdf[s + 1] - cdf[s]) + (q - cdf[s]);
        if (state < (uint64_t{1} << 32) && top > 0) state = (state << 32) | words[--top];
        return s;
    }

    // cdf: n + 1 entries, strictly increasing.
    inline int decode(const uint32_t* cdf, int n) {
        const uint32_t q = static_cast<uint32_t>(state) & (kOne - 1);
        int lo = 0, hi = n;  // cdf[lo] <= q < cdf[hi]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (cdf[mid] <= q)
                lo = mid;
            else
                hi = mid;
        }
        state = (state >> kPrecision) * (cdf[lo + 1] - cdf[lo]) + (q - cdf[lo]);
        if (state < (uint64_t{1} << 32) && top > 0) state = (state << 32) | words[--top];
        return lo;
    }
};

float f16_to_f32(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    } else if (man == 0) {
        bits = sign;
    } else {  // subnormal: renormalise
        int e = -1;
        do {
            ++e;
            man <<= 1;
        } while (!(man & 0x400u));
        bits = sign | ((112u - static_cast<uint32_t>(e)) << 23) | ((man & 0x3FFu) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

}  // namespace
}  // namespace b3

using namespace b3;

extern "C" {

int b3_bark_ans_cdf(const uint32_t* counts, int n_symbols, uint32_t* cdf) {
    if (!counts || !cdf || n_symbols < 1) return set_error(B3_EINVAL, "b3_bark_ans_cdf: bad arguments");
    if (!ans_cdf(counts, n_symbols, cdf)) return set_error(B3_EINVAL, "invalid symbol table");
    return 0;
}

int b3_bark_ans_decode(const uint32_t* counts, int n_symbols, const uint32_t* words, int64_t n_words, int64_t n,
                       uint16_t* symbols) {
    if (!counts || n_symbols < 1 || n_symbols > 65536 || n_words < 0 || (n_words > 0 && !words) || n < 0 ||
        (n > 0 && !symbols))
        return set_error(B3_EINVAL, "b3_bark_ans_decode: bad arguments");
    std::vector<uint32_t> cdf(n_symbols + 1);
    if (!ans_cdf(counts, n_symbols, cdf.data())) return set_error(B3_EINVAL, "invalid symbol table");
    AnsStack ans;
    if (!ans.open(words, n_words)) return set_error(B3_EINVAL, "truncated ANS stream");
    for (int64_t i = 0; i < n; ++i) symbols[i] = static_cast<uint16_t>(ans.decode(cdf.data(), n_symbols));
    return 0;
}

// src/bark.rs:293-359: per column a 4-bit class (high nibble = even column) in
// the first ceil(cols / 2) meta bytes, then 16 tables of 2k + 1 u32 counts;
// classes are decoded in order 0..15 from one stream, each as
// rows x (its columns, ascending) symbols in column-major order.
int b3_bark_decode_levels2(const uint8_t* meta, int64_t meta_bytes, const uint32_t* words, int64_t n_words,
                           int rows, int cols, int k, uint32_t* code_words) {
    if (!meta || meta_bytes < 0 || n_words < 0 || (n_words > 0 && !words) || rows <= 0 || cols <= 0 ||
        !code_words)
        return set_error(B3_EINVAL, "b3_bark_decode_levels2: bad arguments");
    if (k < 1 || k > 3) return set_error(B3_EINVAL, "unsupported level count %d", k);
    const int64_t class_bytes = (static_cast<int64_t>(cols) * 4 + 7) / 8;
    if (meta_bytes < class_bytes) return set_error(B3_EINVAL, "class table is short");
    const int symbols = 2 * k + 1;
    const int64_t have = (meta_bytes - class_bytes) / 4;
    if (have < 16 * symbols)
        return set_error(B3_EINVAL, "symbol tables are short (%lld of %d)", static_cast<long long>(have),
                         16 * symbols);
    std::vector<uint32_t> counts(16 * symbols);
    memcpy(counts.data(), meta + class_bytes, counts.size() * 4);  // little-endian host
    std::vector<std::vector<int>> columns(16);
    for (int col = 0; col < cols; ++col) {
        const uint8_t b = meta[col / 2];
        columns[(col & 1) ? (b & 0xF) : (b >> 4)].push_back(col);
    }
    const int64_t ld = (cols + 7) / 8;
    memset(code_words, 0, static_cast<size_t>(rows) * ld * 4);
    AnsStack ans;
    if (!ans.open(words, n_words)) return set_error(B3_EINVAL, "truncated ANS stream");
    uint32_t cdf[8];
    std::vector<uint8_t> bucket(1u << kBucketBits);
    for (int c = 0; c < 16; ++c) {
        if (columns[c].empty()) continue;
        double total = 0.0;
        for (int s = 0; s < symbols; ++s) total += static_cast<double>(counts[c * symbols + s]);
        if (!(total > 0.0)) return set_error(B3_EINVAL, "empty symbol table for class %d", c);
        if (!ans_cdf(&counts[c * symbols], symbols, cdf)) return set_error(B3_EINVAL, "invalid symbol table");
        ans_buckets(cdf, symbols, bucket.data());
        for (int col : columns[c]) {
            uint32_t* dst = code_words + col / 8;
            const int sh = 4 * (col % 8);
            for (int r = 0; r < rows; ++r)
                dst[static_cast<int64_t>(r) * ld] |= static_cast<uint32_t>(ans.decode_lut(cdf, bucket.data())) << sh;
        }
    }
    return 0;
}

// src/bark.rs:387-431: n symbols from one stream; value i is
// (symbol - (2^(bits-1) - 1)) * scale[i / (n / rows)], scales f16.
int b3_bark_decode_ansint(const uint32_t* counts, int n_symbols, const uint32_t* words, int64_t n_words, int64_t n,
                          int bits, const uint16_t* row_scales, int64_t rows, float* out) {
    if (!counts || n_symbols < 1 || n_words < 0 || (n_words > 0 && !words) || n < 0 || bits < 1 || bits > 16 ||
        rows < 0 || (rows > 0 && !row_scales) || (n > 0 && !out))
        return set_error(B3_EINVAL, "b3_bark_decode_ansint: bad arguments");
    double total = 0.0;
    for (int s = 0; s < n_symbols; ++s) total += static_cast<double>(counts[s]);
    if (!(total > 0.0)) return set_error(B3_EINVAL, "empty symbol table");
    std::vector<uint32_t> cdf(n_symbols + 1);
    if (!ans_cdf(counts, n_symbols, cdf.data())) return set_error(B3_EINVAL, "invalid symbol table");
    AnsStack ans;
    if (!ans.open(words, n_words)) return set_error(B3_EINVAL, "truncated ANS stream");
    const int64_t per_row = rows > 0 ? n / rows : 0;
    const int64_t div = per_row > 0 ? per_row : 1;
    const int64_t bias = (int64_t{1} << (bits - 1)) - 1;
    for (int64_t i = 0; i < n; ++i) {
        const float q = static_cast<float>(static_cast<int64_t>(ans.decode(cdf.data(), n_symbols)) - bias);
        const int64_t r = i / div;
        if (r >= rows) return set_error(B3_EINVAL, "scale table is short (%lld rows)", static_cast<long long>(rows));
        out[i] = q * f16_to_f32(row_scales[r]);
    }
    return 0;
}

}  // extern "C"
