"""Seeded random-init encoder weights and inputs with the reference's tensor
names (src/cpu/mod.rs:47-152, src/encoder.rs:412-640) and the BASELINE
distributions.  There are no checkpoints offline; these stand in for them.

Two layouts:
  "lut4"  every encoder linear as 4-bit codes + a per-row 16-entry f16 table
          (16 levels ~ N(0, 0.02), sorted, then centred: the row's mean level
          is subtracted before rounding to f16; codes uniform in 0..15);
  "bf16"  the Pro layout: bf16 weights ~ N(0, 1/sqrt(fan_in)).
The projector is dense in both (the reference keeps it f16).

`dense_values` turns a weight entry into the f32 values the reference
multiplies (4-bit codes expanded through their table, bf16 widened), which is
what the CPU oracle is given.
"""
from __future__ import annotations

import numpy as np

HIDDEN = 1024
FFN = 4096

LINEARS = [
    ("self_attn.q_proj.weight", HIDDEN, HIDDEN),
    ("self_attn.k_proj.weight", HIDDEN, HIDDEN),
    ("self_attn.v_proj.weight", HIDDEN, HIDDEN),
    ("self_attn.relative_k_proj.weight", HIDDEN, HIDDEN),
    ("self_attn.o_proj.weight", HIDDEN, HIDDEN),
    ("feed_forward1.linear1.weight", FFN, HIDDEN),
    ("feed_forward1.linear2.weight", HIDDEN, FFN),
    ("feed_forward2.linear1.weight", FFN, HIDDEN),
    ("feed_forward2.linear2.weight", HIDDEN, FFN),
    ("conv.pointwise_conv1.weight", 2 * HIDDEN, HIDDEN),
    ("conv.pointwise_conv2.weight", HIDDEN, HIDDEN),
]
NORMS = ["norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out"]


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """src/raw.rs:126-128."""
    return (b.astype(np.uint32) << 16).view(np.float32)


def make_lut4(rng: np.random.Generator, rows: int, cols: int, std: float = 0.02, centre: bool = False):
    """codes uniform 0..15 packed two per byte (low nibble =
    even column), 16 sorted f16 levels ~ N(0, std) per row.

    centre=True subtracts each row's mean level before rounding (the encoder
    model).  Uncentred, every row has a random mean level (~N(0, std/4)), so
    with uniform codes each linear adds a fixed vector (its row means times the
    sum of its input) to every frame; through 24 blocks that common component
    grows until it is the whole residual stream (99.99% of the energy of the
    last block's output at T = 100, per-frame part 0.2% of its rms), and
    every frame of an utterance looks alike.  Centred rows keep the per-frame
    part at ~30% of the rms after 24 blocks."""
    codes = rng.integers(0, 16, size=(rows, cols), dtype=np.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    levels = np.sort(rng.normal(0.0, std, size=(rows, 16)).astype(np.float32), axis=1)
    if centre:
        levels -= levels.mean(axis=1, keepdims=True)
    lut16 = levels.astype(np.float16).view(np.uint16)
    return packed, lut16


def make_levels_k(rng: np.random.Generator, rows: int, cols: int, k: int = 3, scale: float = 0.02):
    """The .bark levels2 form (src/bark.rs:33-48): up to 3 positive f16
    magnitudes per row, codes 0..2k packed eight per u32 (low nibble first)."""
    mags = np.sort(np.abs(rng.normal(0.0, scale, size=(rows, k))).astype(np.float32), axis=1)
    levels = np.zeros((rows, 4), dtype=np.uint16)
    levels[:, :k] = mags.astype(np.float16).view(np.uint16)
    codes = rng.integers(0, 2 * k + 1, size=(rows, cols), dtype=np.uint32)
    ld = (cols + 7) // 8
    words = np.zeros((rows, ld), dtype=np.uint32)
    for j in range(cols):
        words[:, j // 8] |= codes[:, j] << np.uint32(4 * (j % 8))
    return words, levels, codes


def expand_lut4(codes_packed: np.ndarray, lut16: np.ndarray) -> np.ndarray:
    """codes [rows, cols/2] + lut16 [rows, 16] -> f32 [rows, cols]."""
    lo = codes_packed & 0xF
    hi = codes_packed >> 4
    rows, half = codes_packed.shape
    idx = np.empty((rows, 2 * half), dtype=np.int64)
    idx[:, 0::2] = lo
    idx[:, 1::2] = hi
    vals = lut16.view(np.float16).astype(np.float32)
    return np.take_along_axis(vals, idx, axis=1)


def expand_levels(codes: np.ndarray, levels: np.ndarray, k: int) -> np.ndarray:
    """`expand` (src/bark.rs:597-611) on unpacked codes."""
    lev = levels.view(np.float16).astype(np.float32)
    out = np.zeros(codes.shape, dtype=np.float32)
    for c in range(1, 2 * k + 1):
        neg = c > k
        mag = (c - k - 1) if neg else (c - 1)
        v = lev[:, mag : mag + 1]
        out = np.where(codes == c, -v if neg else v, out)
    return out


def dense_values(entry) -> np.ndarray:
    """f32 values of a weight entry as the reference multiplies them."""
    if isinstance(entry, tuple):
        if entry[0] == "lut4":
            return expand_lut4(entry[1], entry[2])
        if entry[0] == "bf16":
            return bf16_bits_to_f32(entry[1])
        if entry[0] == "f16":
            return entry[1].view(np.float16).astype(np.float32)
        raise ValueError(entry[0])
    return np.asarray(entry, dtype=np.float32)


def encoder_weights(seed: int = 0, n_layers: int = 24, layout: str = "lut4") -> dict:
    """Random-init encoder weights keyed by the reference checkpoint names."""
    rng = np.random.default_rng(seed)
    w: dict = {}

    def linear(name, rows, cols):
        if layout == "lut4":
            w[name] = ("lut4",) + make_lut4(rng, rows, cols, centre=True)
        elif layout == "bf16":
            vals = rng.normal(0.0, 1.0 / np.sqrt(cols), size=(rows, cols)).astype(np.float32)
            w[name] = ("bf16", f32_to_bf16_bits(vals))
        else:
            raise ValueError(layout)

    def vec(name, n, mean=0.0, std=0.02):
        w[name] = rng.normal(mean, std, size=n).astype(np.float32)

    linear("encoder.subsampling.linear.weight", HIDDEN, 4096)
    vec("encoder.subsampling.linear.bias", HIDDEN, std=0.01)
    for l in range(n_layers):
        p = f"encoder.layers.{l}."
        for name, rows, cols in LINEARS:
            linear(p + name, rows, cols)
        w[p + "conv.depthwise_conv.weight"] = rng.normal(0.0, 0.1, size=(HIDDEN, 1, 9)).astype(np.float32)
        vec(p + "conv.norm.weight", HIDDEN, 1.0)
        vec(p + "conv.norm.bias", HIDDEN)
        vec(p + "conv.norm.running_mean", HIDDEN)
        w[p + "conv.norm.running_var"] = rng.uniform(0.5, 1.5, size=HIDDEN).astype(np.float32)
        for n in NORMS:
            vec(p + n + ".weight", HIDDEN, 1.0)
            vec(p + n + ".bias", HIDDEN)
        w[p + "self_attn.bias_u"] = rng.normal(0.0, 0.02, size=(8, 128)).astype(np.float32)
        w[p + "self_attn.bias_v"] = rng.normal(0.0, 0.02, size=(8, 128)).astype(np.float32)
    pw = rng.normal(0.0, 1.0 / np.sqrt(HIDDEN), size=(640, HIDDEN)).astype(np.float32)
    w["encoder_projector.weight"] = ("bf16", f32_to_bf16_bits(pw))
    vec("encoder_projector.bias", 640, std=0.01)
    return w


def decoder_weights(seed: int = 0, vocab: int = 1025, blank_bias: float = 2.0) -> dict:
    """Random-init TDT prediction net + joint (2-layer LSTM
    of 640, joint 640, `vocab` rows including the blank as the last one, 5
    duration rows), with the reference's tensor names (src/tdt.rs:142-163).
    LSTM weights follow PyTorch's U(-1/sqrt(640), 1/sqrt(640)) init; the blank
    row gets `blank_bias` so streams are mostly blanks, as real ones are."""
    rng = np.random.default_rng(seed)
    H, G = 640, 2560
    k = 1.0 / np.sqrt(H)
    w = {"decoder.embedding.weight": rng.normal(0.0, 1.0, size=(vocab, H)).astype(np.float32)}
    for l in (0, 1):
        for name, shape in (("weight_ih", (G, H)), ("weight_hh", (G, H)), ("bias_ih", (G,)), ("bias_hh", (G,))):
            w[f"decoder.lstm.{name}_l{l}"] = rng.uniform(-k, k, size=shape).astype(np.float32)
    w["decoder.decoder_projector.weight"] = rng.normal(0.0, k, size=(H, H)).astype(np.float32)
    w["decoder.decoder_projector.bias"] = rng.normal(0.0, 0.01, size=H).astype(np.float32)
    w["joint.head.weight"] = rng.normal(0.0, k, size=(vocab + 5, H)).astype(np.float32)
    hb = rng.normal(0.0, 0.01, size=vocab + 5).astype(np.float32)
    hb[vocab - 1] += blank_bias
    w["joint.head.bias"] = hb
    return w


def frontend_weights(seed: int = 0) -> dict:
    """Random-init conv subsampling (src/sub.rs:56-103 names): conv 1->256
    3x3, two depthwise 3x3 and two pointwise 256->256, PyTorch's default
    U(-1/sqrt(fan_in), 1/sqrt(fan_in)) init."""
    rng = np.random.default_rng(seed)
    w = {}
    p = "encoder.subsampling.layers."
    for l, shape, fan in (("0", (256, 1, 3, 3), 9), ("2", (256, 1, 3, 3), 9), ("3", (256, 256, 1, 1), 256),
                          ("5", (256, 1, 3, 3), 9), ("6", (256, 256, 1, 1), 256)):
        k = 1.0 / np.sqrt(fan)
        w[p + l + ".weight"] = rng.uniform(-k, k, size=shape).astype(np.float32)
        w[p + l + ".bias"] = rng.uniform(-k, k, size=shape[0]).astype(np.float32)
    return w


def synth_audio(rng: np.random.Generator, seconds: float) -> np.ndarray:
    """BASELINE configs 2/5 input: 16 kHz white noise U(-0.1, 0.1) plus three
    sines of amplitude 0.1 at seeded frequencies U(100, 4000) Hz and phases."""
    n = int(round(seconds * 16000))
    t = np.arange(n, dtype=np.float64) / 16000.0
    x = rng.uniform(-0.1, 0.1, size=n)
    for _ in range(3):
        f = rng.uniform(100.0, 4000.0)
        ph = rng.uniform(0.0, 2 * np.pi)
        x += 0.1 * np.sin(2 * np.pi * f * t + ph)
    return x.astype(np.float32)


def sub_features(rng: np.random.Generator, t: int) -> np.ndarray:
    """Stand-in for the conv-subsampling output (T, 4096): the reference's
    last op is a ReLU (src/sub.rs:107-286), so non-negative values."""
    return np.maximum(rng.normal(0.0, 1.0, size=(t, 4096)), 0.0).astype(np.float32)


def batch_lengths(seed: int, n: int = 256, lo: float = 10.0, hi: float = 60.0) -> np.ndarray:
    """utterance lengths uniform in [lo, hi] seconds."""
    return np.random.default_rng(seed).uniform(lo, hi, size=n)
