"""`.bark` container writer and ANS restatements (test fixtures).

TEST INFRASTRUCTURE ONLY: builds synthetic `model.bark` containers for the
loader's parity tests and restates the entropy coding the reference decodes
with.  Only tests/ import this module; the product never does.

The layout restated here is the one the reference reader parses
(src/bark.rs, paths relative to the bark3-wgpu crate):
  - header: u64 little-endian JSON length, then JSON
    {"format": "bark-levels-v2" | "bark-levels-v3", "index": [...]}
    (read_header, src/bark.rs:487-507);
  - one index entry per tensor: "n" name, "shape", "k" kind ("levels2",
    "ansint<bits>", "raw"), "K" level count, field byte lengths "lev",
    "meta", "b" (ANS words or raw bytes), "s" (scales), LZMA flags "zl",
    "zs", "zr", and "dtype" for raw integers; payloads follow the header
    back to back in index order (parse_index, src/bark.rs:509-559);
  - levels2: f16 level table rows x K (maybe LZMA), then meta = 4-bit column
    classes (high nibble = even column) + 16 x (2K + 1) u32 symbol counts,
    then the ANS words; classes 0..15 are coded in order, each class's
    columns ascending, rows inner (decode_levels2, src/bark.rs:277-366);
  - ansint<bits>: f16 per-row scales (maybe LZMA), u32 counts, ANS words;
    value = (symbol - (2^(bits-1) - 1)) * scale (src/bark.rs:387-431);
  - raw: little-endian f16 / int64 / int32 bytes, maybe LZMA (xz when the
    bytes start with the xz magic, else the legacy .lzma format;
    BarkContainer::field, src/bark.rs:256-271).

ANS: constriction 0.5.0 (`DefaultAnsCoder`: stack ANS, u32 words, u64
state; `DefaultContiguousCategoricalEntropyModel` with 24-bit precision from
`from_floating_point_probabilities_fast`).  The crate is not vendored in the
reference and no constriction-written stream exists here, so the
restatement is pinned only by round trips (parity unpinned).
"""
from __future__ import annotations

import ctypes
import json
import lzma
import struct

import numpy as np

from . import oracle as _oracle

PRECISION = 24


# ───────────────────── pure-Python restatement (small cases) ─────────────────────
def py_ans_cdf(counts) -> list[int]:
    """from_floating_point_probabilities_fast: p_i = c_i / sum c (f64), every
    symbol keeps one unit, the free 2^24 - n units follow floor(scale * cum)."""
    n = len(counts)
    if n < 2 or n >= 1 << PRECISION:
        raise ValueError("invalid symbol table")
    total = 0.0
    for c in counts:
        total += float(c)
    if not total > 0.0:
        raise ValueError("empty symbol table")
    probs = [float(c) / total for c in counts]
    norm = 0.0
    for p in probs:
        norm += p
    scale = float((1 << PRECISION) - n) / norm
    cdf, run = [], 0.0
    for i, p in enumerate(probs):
        cdf.append(int(run * scale) + i)
        run += p
    cdf.append(1 << PRECISION)
    return cdf


def py_ans_decode(words, counts, n: int) -> list[int]:
    """decode_iid_symbols on a stack of u32 words (top = last)."""
    cdf = py_ans_cdf(counts)
    stack = [int(w) for w in words]
    state = 0
    if stack:
        first = stack.pop()
        if first == 0:
            raise ValueError("truncated ANS stream")
        state = first
        while stack and state < 1 << 32:
            state = (state << 32) | stack.pop()
    out = []
    mask = (1 << PRECISION) - 1
    for _ in range(n):
        q = state & mask
        s = 0
        while cdf[s + 1] <= q:
            s += 1
        state = (state >> PRECISION) * (cdf[s + 1] - cdf[s]) + (q - cdf[s])
        if state < 1 << 32 and stack:
            state = (state << 32) | stack.pop()
        out.append(s)
    return out


def py_ans_encode(symbols, counts) -> list[int]:
    """Stack encoder whose words py_ans_decode pops back in order."""
    cdf = py_ans_cdf(counts)
    words, state = [], 0
    for s in reversed(list(symbols)):
        lo, p = cdf[s], cdf[s + 1] - cdf[s]
        if (state >> (64 - PRECISION)) >= p:
            words.append(state & 0xFFFFFFFF)
            state >>= 32
        state = ((state // p) << PRECISION) | (state % p + lo)
    while state:
        words.append(state & 0xFFFFFFFF)
        state >>= 32
    return words


# ───────────────────────── C restatement (any size) ─────────────────────────
def ans_cdf(counts) -> np.ndarray:
    counts = np.ascontiguousarray(counts, dtype=np.uint32)
    cdf = np.zeros(len(counts) + 1, np.uint32)
    if _oracle.lib().or_ans_cdf(counts.ctypes.data, len(counts), cdf.ctypes.data):
        raise ValueError("invalid symbol table")
    return cdf


class AnsEncoder:
    """Stack encoder (C).  Segments are pushed last-first so that a decoder
    pops them first-first: call push() with the LAST segment first."""

    def __init__(self, capacity_words: int):
        self.words = np.zeros(max(capacity_words, 4), np.uint32)
        self.state = ctypes.c_uint64(0)
        self.n = ctypes.c_int64(0)

    def push(self, symbols, counts) -> None:
        sym = np.ascontiguousarray(symbols, dtype=np.uint16).reshape(-1)
        cdf = ans_cdf(counts)
        rc = _oracle.lib().or_ans_push_reverse(
            ctypes.addressof(self.state), self.words.ctypes.data, ctypes.addressof(self.n), len(self.words),
            sym.ctypes.data, sym.size, cdf.ctypes.data, len(cdf) - 1)
        if rc:
            raise ValueError(f"ANS encode failed ({rc})")

    def finish(self) -> np.ndarray:
        if _oracle.lib().or_ans_flush(ctypes.addressof(self.state), self.words.ctypes.data, ctypes.addressof(self.n),
                                      len(self.words)):
            raise ValueError("ANS encode overflow")
        return self.words[: self.n.value].copy()


def ans_encode(symbols, counts) -> np.ndarray:
    sym = np.asarray(symbols).reshape(-1)
    enc = AnsEncoder(sym.size // 2 + 16)
    enc.push(sym, counts)
    return enc.finish()


def ans_decode(words, counts, n: int) -> np.ndarray:
    words = np.ascontiguousarray(words, dtype=np.uint32)
    cdf = ans_cdf(counts)
    top, state = ctypes.c_int64(len(words)), ctypes.c_uint64(0)
    L = _oracle.lib()
    if L.or_ans_open(words.ctypes.data, ctypes.addressof(top), ctypes.addressof(state)):
        raise ValueError("truncated ANS stream")
    out = np.zeros(n, np.uint16)
    L.or_ans_pop(words.ctypes.data, ctypes.addressof(top), ctypes.addressof(state), cdf.ctypes.data, len(cdf) - 1,
                 out.ctypes.data, n)
    return out


# ─────────────────────────────── container writer ───────────────────────────────
def zip_bytes(raw: bytes, how: str | None) -> bytes:
    if how is None:
        return raw
    if how == "xz":
        return lzma.compress(raw, format=lzma.FORMAT_XZ)
    if how == "alone":
        return lzma.compress(raw, format=lzma.FORMAT_ALONE)
    raise ValueError(how)


def levels2_entry(name: str, codes: np.ndarray, levels: np.ndarray, k: int, classes: np.ndarray | None = None,
                  zip_levels: str | None = None, smoothing: int = 0):
    """codes [rows][cols] in 0..2k; levels [rows][k] f16 bits; classes [cols]
    in 0..15 (default: column % 16).  Counts are the per-class code
    histograms (+ smoothing)."""
    codes = np.asarray(codes, dtype=np.uint8)
    rows, cols = codes.shape
    levels = np.ascontiguousarray(np.asarray(levels, dtype=np.uint16)[:, :k])
    if classes is None:
        classes = np.arange(cols) % 16
    classes = np.asarray(classes, dtype=np.uint8)
    sym = 2 * k + 1
    nib = np.zeros((cols + 1) // 2 * 2, np.uint8)
    nib[:cols] = classes
    class_bytes = ((nib[0::2] << 4) | nib[1::2]).astype(np.uint8).tobytes()
    counts = np.zeros((16, sym), np.uint32)
    for c in range(16):
        cols_c = np.nonzero(classes == c)[0]
        if len(cols_c):
            counts[c] = np.bincount(codes[:, cols_c].reshape(-1), minlength=sym)[:sym] + smoothing
    meta = class_bytes + counts.astype("<u4").tobytes()
    enc = AnsEncoder(rows * cols // 2 + 64)
    for c in reversed(range(16)):
        cols_c = np.nonzero(classes == c)[0]
        if len(cols_c):
            enc.push(codes[:, cols_c].T.reshape(-1), counts[c])
    words = enc.finish().astype("<u4").tobytes()
    lev = zip_bytes(levels.astype("<u2").tobytes(), zip_levels)
    index = {"n": name, "shape": [rows, cols], "k": "levels2", "K": k, "lev": len(lev), "meta": len(meta),
             "b": len(words), "s": 0}
    if zip_levels:
        index["zl"] = True
    return index, lev + meta + words


def ansint_entry(name: str, q: np.ndarray, bits: int, scales: np.ndarray, zip_scales: str | None = None):
    """q: signed integers [rows][...] in [-(2^(bits-1) - 1), 2^(bits-1)];
    scales: f16 bits per row."""
    q = np.asarray(q, dtype=np.int64)
    bias = (1 << (bits - 1)) - 1
    sym = (q + bias).reshape(-1)
    n_sym = 1 << bits
    assert sym.min() >= 0 and sym.max() < n_sym
    counts = np.bincount(sym, minlength=n_sym).astype(np.uint32)
    counts[counts == 0] = 1
    meta = counts.astype("<u4").tobytes()
    words = ans_encode(sym, counts).astype("<u4").tobytes()
    sc = zip_bytes(np.asarray(scales, dtype="<u2").tobytes(), zip_scales)
    index = {"n": name, "shape": list(q.shape), "k": f"ansint{bits}", "s": len(sc), "meta": len(meta),
             "b": len(words)}
    if zip_scales:
        index["zs"] = 1
    return index, sc + meta + words


def raw_entry(name: str, arr: np.ndarray, zip_raw: str | None = None):
    """f16 (as np.float16 or f16 bits in uint16), int64 or int32."""
    arr = np.asarray(arr)
    if arr.dtype == np.int64:
        dt, data = "torch.int64", arr.astype("<i8").tobytes()
    elif arr.dtype == np.int32:
        dt, data = "torch.int32", arr.astype("<i4").tobytes()
    elif arr.dtype == np.uint16:
        dt, data = "torch.float16", arr.astype("<u2").tobytes()
    else:
        dt, data = "torch.float16", arr.astype(np.float16).view("<u2").tobytes()
    data = zip_bytes(data, zip_raw)
    index = {"n": name, "shape": list(arr.shape), "k": "raw", "b": len(data), "dtype": dt}
    if zip_raw:
        index["zr"] = True
    return index, data


def write_container(entries, fmt: str = "bark-levels-v3", extra: dict | None = None) -> bytes:
    head = {"format": fmt, "index": [e[0] for e in entries]}
    if extra:
        head.update(extra)
    js = json.dumps(head).encode()
    return struct.pack("<Q", len(js)) + js + b"".join(e[1] for e in entries)


def quantize_ansint(values: np.ndarray, bits: int):
    """Per-row symmetric quantisation of a float matrix: q in
    [-(2^(bits-1) - 1), 2^(bits-1) - 1], scale = max|row| / (2^(bits-1) - 1)
    rounded to f16.  Returns (q, scale f16 bits, dequantised f32) with the
    dequantised values computed the way the reader computes them."""
    v = np.asarray(values, dtype=np.float32)
    rows = v.shape[0]
    flat = v.reshape(rows, -1)
    qmax = (1 << (bits - 1)) - 1
    amax = np.abs(flat).max(axis=1)
    scale16 = (np.where(amax > 0, amax / qmax, 1.0)).astype(np.float16)
    s32 = scale16.astype(np.float32)
    q = np.clip(np.rint(flat / s32[:, None]), -qmax, qmax).astype(np.int64)
    deq = (q.astype(np.float32) * s32[:, None]).astype(np.float32)
    return q.reshape(v.shape), scale16.view(np.uint16), deq.reshape(v.shape)


def container_from_weights(weights: dict, rng: np.random.Generator, make_levels_k, ansint_bits: int = 6,
                           zip_every: int = 3):
    """A synthetic checkpoint in the container's storage classes, and the same
    values as a direct weight dict (the loader's parity fixture):
      - 4-bit linears ("lut4" / "levels" entries) -> levels2, k in {2, 3},
        fresh codes and levels;
      - other matrices (2-D, >= 16 rows) -> ansint<bits> with f16 row scales;
      - everything else -> raw f16.
    Every `zip_every`-th entry has its optional field LZMA-compressed,
    alternating xz and the legacy format.  Returns (container bytes, direct
    dict for Encoder.load)."""
    entries, direct = [], {}
    for i, (name, v) in enumerate(weights.items()):
        z = (None, "xz", "alone")[i % zip_every] if zip_every else None
        if isinstance(v, tuple) and v[0] in ("lut4", "levels"):
            if v[0] == "lut4":
                rows, cols = v[2].shape[0], v[1].shape[1] * 2
            else:
                rows, cols = v[2].shape[0], v[4]
            k = int(rng.integers(2, 4))
            words, levels, codes = make_levels_k(rng, rows, cols, k)
            entries.append(levels2_entry(name, codes, levels, k, classes=rng.integers(0, 16, cols), zip_levels=z))
            direct[name] = ("levels", words, levels, k, cols)
            continue
        if isinstance(v, tuple):
            vals = _tuple_values(v)
        else:
            vals = np.asarray(v, dtype=np.float32)
        if vals.ndim == 2 and vals.shape[0] >= 16:
            q, sc, deq = quantize_ansint(vals, ansint_bits)
            entries.append(ansint_entry(name, q, ansint_bits, sc, zip_scales=z))
            direct[name] = deq
        else:
            h = vals.astype(np.float16)
            entries.append(raw_entry(name, h, zip_raw=z))
            direct[name] = ("f16", h.view(np.uint16))
    return write_container(entries), direct


def _tuple_values(v) -> np.ndarray:
    if v[0] == "bf16":
        return (v[1].astype(np.uint32) << 16).view(np.float32)
    if v[0] == "f16":
        return v[1].view(np.float16).astype(np.float32)
    raise ValueError(v[0])
