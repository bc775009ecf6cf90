"""ctypes binding of the CPU oracle (bark3_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs import this module; the product never does.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libbark3_oracle.so"
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float


def build(force: bool = False) -> pathlib.Path:
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "bark3_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE)], check=True, stdout=subprocess.DEVNULL)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        sig = {
            "or_set_threads": (None, [_I]),
            "or_get_threads": (_I, []),
            "or_f32_to_f16_bits": (ctypes.c_uint16, [_F]),
            "or_f16_bits_to_f32": (_F, [ctypes.c_uint16]),
            "or_round_f16": (_F, [_F]),
            "or_bf16_bits_to_f32": (_F, [ctypes.c_uint16]),
            "or_f32_to_f16_array": (None, [_P, _P, ctypes.c_int64]),
            "or_expand_code": (_F, [_I, _I, _P]),
            "or_expand_lut4": (None, [_P, _P, _P, _I, _I]),
            "or_gemm": (None, [_P, _P, _P, _I, _I, _I, _I]),
            "or_packw_new": (_P, [_P, _I, _I, _I]),
            "or_packw_free": (None, [_P]),
            "or_gemm_packed": (None, [_P, _P, _P, _I]),
            "or_layer_norm": (None, [_P, _P, _P, _P, _I, _I]),
            "or_silu": (None, [_P, ctypes.c_int64]),
            "or_glu": (None, [_P, _P, _I, _I]),
            "or_rel_softmax_rows": (None, [_P, _P, _I, _I, _I, _I, _I, _F]),
            "or_dwconv_bn_silu": (None, [_P, _P, _P, _P, _P, _I, _I]),
            "or_pos_embed": (None, [_I, _P]),
            "or_encoder_new": (_P, [_I, _I, _P, _P, _P, _P]),
            "or_encoder_set_layer": (_I, [_P, _I] + [_P] * 20),
            "or_encoder_free": (None, [_P]),
            "or_encode": (_I, [_P, _P, _I, _I, _P]),
            "or_encode_layers": (_I, [_P, _P, _I, _P, _P]),
            "or_attn_conv": (_I, [_P, _I, _P, _I]),
            "or_attention_core": (_I, [_P, _P, _P, _P, _P, _I, _P]),
            "or_tdt_new": (_P, [_I] + [_P] * 9),
            "or_tdt_free": (None, [_P]),
            "or_tdt_decode": (_I, [_P, _P, _I, _P, _I]),
            "or_tdt_decode_margins": (_I, [_P, _P, _I, _P, _I, _P, ctypes.c_long, _P]),
            "or_tdt_decode_batch": (None, [_P, _P, _P, _I, _P, _P, _I]),
            "or_mel": (_I, [_P, ctypes.c_int64, _P, _P, _P]),
            "or_subsample": (_I, [_P, _I, _I] + [_P] * 11),
            "or_ans_cdf": (_I, [_P, _I, _P]),
            "or_ans_push_reverse": (_I, [_P, _P, _P, ctypes.c_int64, _P, ctypes.c_int64, _P, _I]),
            "or_ans_flush": (_I, [_P, _P, _P, ctypes.c_int64]),
            "or_ans_open": (_I, [_P, _P, _P]),
            "or_ans_pop": (None, [_P, _P, _P, _P, _I, _P, ctypes.c_int64]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        L.or_set_threads(os.cpu_count() or 1)
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def threads() -> int:
    return lib().or_get_threads()


def round_f16(x: np.ndarray) -> np.ndarray:
    x = f32(x)
    bits = np.empty(x.shape, dtype=np.uint16)
    lib().or_f32_to_f16_array(_p(x), _p(bits), x.size)
    return bits.view(np.float16).astype(np.float32)


def gemm(a: np.ndarray, w: np.ndarray, half: bool = True) -> np.ndarray:
    """C = A W^T via the restated PackW + 6x16 FMA kernel (src/cpu/gemm.rs)."""
    a, w = f32(a), f32(w)
    m, k = a.shape
    n = w.shape[0]
    c = np.empty((m, n), dtype=np.float32)
    lib().or_gemm(_p(a), _p(w), _p(c), m, n, k, int(half))
    return c


class PackedWeight:
    """A weight packed once (load time), multiplied many times (timing)."""

    def __init__(self, w: np.ndarray, half: bool = True):
        w = f32(w)
        self.n, self.k = w.shape
        self.h = lib().or_packw_new(_p(w), self.n, self.k, int(half))

    def __call__(self, a: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        a = f32(a)
        if out is None:
            out = np.empty((a.shape[0], self.n), dtype=np.float32)
        lib().or_gemm_packed(_p(a), self.h, _p(out), a.shape[0])
        return out

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_packw_free(self.h)
            self.h = None


def layer_norm(x, w, b):
    x, w, b = f32(x), f32(w), f32(b)
    y = np.empty_like(x)
    lib().or_layer_norm(_p(x), _p(y), _p(w), _p(b), x.shape[0], x.shape[1])
    return y


def silu(x):
    x = f32(x).copy()
    lib().or_silu(_p(x), x.size)
    return x


def glu(x):
    x = f32(x)
    rows, c2 = x.shape
    y = np.empty((rows, c2 // 2), dtype=np.float32)
    lib().or_glu(_p(x), _p(y), rows, c2 // 2)
    return y


def dwconv_bn_silu(x, dw, bn_a, bn_b):
    x, dw, bn_a, bn_b = f32(x), f32(dw), f32(bn_a), f32(bn_b)
    y = np.empty_like(x)
    lib().or_dwconv_bn_silu(_p(x), _p(dw), _p(bn_a), _p(bn_b), _p(y), x.shape[0], x.shape[1])
    return y


def pos_embed(t: int) -> np.ndarray:
    out = np.empty((2 * t - 1, 1024), dtype=np.float32)
    lib().or_pos_embed(t, _p(out))
    return out


def mel_filters(n_mels: int = 128, n_fft: int = 512, sr: int = 16000) -> np.ndarray:
    """The (128, 257) slaney mel filterbank the reference bundles as
    data/mel_filters.f32 and hands to `MelFrontend::new` (src/mel.rs:10-40),
    restated from Slaney's Auditory Toolbox construction (as published in
    librosa.filters.mel with htk=False, norm="slaney"): a mel scale linear
    below 1 kHz (200/3 Hz per mel) and logarithmic above it (27 mels per
    factor 6.4), n_mels + 2 equally spaced mel points between 0 Hz and sr/2,
    triangular filters over the linearly spaced FFT bin frequencies, each
    scaled by 2 / (its upper edge - its lower edge) so it has unit area.
    Computed in float64 and rounded once to float32.  Pure numpy: loads no
    shared library."""
    f_sp = 200.0 / 3.0
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0

    def hz_to_mel(f):
        f = np.asarray(f, dtype=np.float64)
        m = f / f_sp
        return np.where(f >= min_log_hz, min_log_mel + np.log(np.maximum(f, 1e-300) / min_log_hz) / logstep, m)

    def mel_to_hz(m):
        m = np.asarray(m, dtype=np.float64)
        return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), f_sp * m)

    bins = np.linspace(0.0, sr / 2.0, 1 + n_fft // 2)
    edges = mel_to_hz(np.linspace(hz_to_mel(0.0), hz_to_mel(sr / 2.0), n_mels + 2))
    width = np.diff(edges)
    dist = edges[:, None] - bins[None, :]
    fb = np.zeros((n_mels, len(bins)), dtype=np.float64)
    for i in range(n_mels):
        rise = -dist[i] / width[i]
        fall = dist[i + 2] / width[i + 1]
        fb[i] = np.maximum(0.0, np.minimum(rise, fall))
    fb *= (2.0 / (edges[2 : n_mels + 2] - edges[:n_mels]))[:, None]
    return fb.astype(np.float32)


def mel(wave: np.ndarray, filters: np.ndarray):
    """MelFrontend::compute restated: padded wave -> ((frames, 128), n_valid)."""
    wave = f32(wave)
    filters = f32(filters)
    n_frames = 1 + len(wave) // 160
    out = np.zeros((n_frames, 128), dtype=np.float32)
    nv = ctypes.c_int()
    lib().or_mel(_p(wave), len(wave), _p(filters), _p(out), ctypes.byref(nv))
    return out, nv.value


def subsample(mel_rows: np.ndarray, n_valid: int, w: dict) -> np.ndarray:
    """subsample (src/sub.rs:107-300) restated: (frames, 128) -> (T, 4096)."""
    mel_rows = f32(mel_rows)
    f = mel_rows.shape[0]

    def clen(v):
        return (v - 1) // 2 + 1

    t = clen(clen(clen(f)))
    out = np.zeros((t, 4096), dtype=np.float32)
    p = "encoder.subsampling.layers."
    keep = [f32(w[p + n].reshape(-1)) for n in ("0.weight", "0.bias", "2.weight", "2.bias", "3.weight", "3.bias",
                                                 "5.weight", "5.bias", "6.weight", "6.bias")]
    got = lib().or_subsample(_p(mel_rows), f, n_valid, *[_p(a) for a in keep], _p(out))
    assert got == t
    return out


def expand_code(code: int, k: int, levels: np.ndarray) -> float:
    levels = np.ascontiguousarray(levels, dtype=np.uint16)
    return lib().or_expand_code(code, k, _p(levels))


class OracleEncoder:
    """Restated CpuEncoder (src/cpu/mod.rs) over dense f32 weight values."""

    def __init__(self, weights: dict, n_layers: int, half: bool = True):
        import importlib

        syn = importlib.import_module("bark3_b200.synthetic")
        dv = syn.dense_values
        L = lib()
        self.n_layers = n_layers
        keep = []

        def arr(x):
            a = f32(x)
            keep.append(a)
            return _p(a)

        self.h = L.or_encoder_new(
            n_layers, int(half),
            arr(dv(weights["encoder.subsampling.linear.weight"])),
            arr(weights["encoder.subsampling.linear.bias"]),
            arr(dv(weights["encoder_projector.weight"])),
            arr(weights["encoder_projector.bias"]),
        )
        for l in range(n_layers):
            p = f"encoder.layers.{l}."
            g = lambda n: dv(weights[p + n])  # noqa: E731
            ln_w = np.stack([weights[p + n + ".weight"] for n in syn.NORMS])
            ln_b = np.stack([weights[p + n + ".bias"] for n in syn.NORMS])
            rc = L.or_encoder_set_layer(
                self.h, l,
                arr(g("self_attn.q_proj.weight")), arr(g("self_attn.k_proj.weight")),
                arr(g("self_attn.v_proj.weight")), arr(g("self_attn.relative_k_proj.weight")),
                arr(g("self_attn.o_proj.weight")),
                arr(g("feed_forward1.linear1.weight")), arr(g("feed_forward1.linear2.weight")),
                arr(g("feed_forward2.linear1.weight")), arr(g("feed_forward2.linear2.weight")),
                arr(g("conv.pointwise_conv1.weight")), arr(g("conv.pointwise_conv2.weight")),
                arr(weights[p + "conv.depthwise_conv.weight"].reshape(1024, 9)),
                arr(weights[p + "conv.norm.weight"]), arr(weights[p + "conv.norm.bias"]),
                arr(weights[p + "conv.norm.running_mean"]), arr(weights[p + "conv.norm.running_var"]),
                arr(ln_w), arr(ln_b),
                arr(weights[p + "self_attn.bias_u"].reshape(-1)), arr(weights[p + "self_attn.bias_v"].reshape(-1)),
            )
            assert rc == 0
            keep.clear()

    def encode(self, sub: np.ndarray, layers: int | None = None) -> np.ndarray:
        layers = self.n_layers if layers is None else layers
        sub = f32(sub)
        t = sub.shape[0]
        out = np.empty((t, 640 if layers >= self.n_layers else 1024), dtype=np.float32)
        assert lib().or_encode(self.h, _p(sub), t, layers, _p(out)) == 0
        return out

    def encode_layers(self, sub: np.ndarray):
        """One pass over every block: (per-block pre-norm_out residuals
        [n_layers, t, 1024], pooler [t, 640]); entry l equals
        encode(sub, layers=l + 1)."""
        sub = f32(sub)
        t = sub.shape[0]
        dump = np.empty((self.n_layers, t, 1024), dtype=np.float32)
        out = np.empty((t, 640), dtype=np.float32)
        assert lib().or_encode_layers(self.h, _p(sub), t, _p(dump), _p(out)) == 0
        return dump, out

    def attn_conv(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = f32(x).copy()
        assert lib().or_attn_conv(self.h, layer, _p(x), x.shape[0]) == 0
        return x

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_encoder_free(self.h)
            self.h = None


class OracleTdt:
    """Restated TdtDecoder (src/tdt.rs): greedy TDT over a pooler (t, 640)."""

    def __init__(self, w: dict):
        emb = f32(w["decoder.embedding.weight"])
        self.vocab = emb.shape[0]
        keep = [emb]

        def cat(a, b):
            x = f32(np.concatenate([f32(w[a]).reshape(-1), f32(w[b]).reshape(-1)]))
            keep.append(x)
            return _p(x)

        def one(n):
            x = f32(w[n])
            keep.append(x)
            return _p(x)

        self.h = lib().or_tdt_new(
            self.vocab, _p(emb),
            cat("decoder.lstm.weight_ih_l0", "decoder.lstm.weight_ih_l1"),
            cat("decoder.lstm.weight_hh_l0", "decoder.lstm.weight_hh_l1"),
            cat("decoder.lstm.bias_ih_l0", "decoder.lstm.bias_ih_l1"),
            cat("decoder.lstm.bias_hh_l0", "decoder.lstm.bias_hh_l1"),
            one("decoder.decoder_projector.weight"), one("decoder.decoder_projector.bias"),
            one("joint.head.weight"), one("joint.head.bias"),
        )

    def decode(self, pooler: np.ndarray, max_tokens: int = 1 << 16) -> np.ndarray:
        pooler = f32(pooler)
        out = np.zeros((max_tokens, 3), dtype=np.uint32)
        n = lib().or_tdt_decode(self.h, _p(pooler), pooler.shape[0], _p(out), max_tokens)
        return out[: min(n, max_tokens)]

    def decode_margins(self, pooler: np.ndarray, max_tokens: int = 1 << 16):
        """decode() plus every step's decision margins: (tokens, gaps [steps, 2])
        with gaps[:, 0] = best - runner-up token score and gaps[:, 1] the same
        over the five durations."""
        pooler = f32(pooler)
        t = pooler.shape[0]
        cap = t * 14 + 64
        out = np.zeros((max_tokens, 3), dtype=np.uint32)
        gaps = np.zeros((cap, 2), dtype=np.float32)
        steps = ctypes.c_long()
        n = lib().or_tdt_decode_margins(self.h, _p(pooler), t, _p(out), max_tokens, _p(gaps), cap,
                                        ctypes.byref(steps))
        return out[: min(n, max_tokens)], gaps[: min(steps.value, cap)]

    def decode_batch(self, pooler: np.ndarray, cu, max_tokens: int = 4096) -> list:
        pooler = f32(pooler)
        cu = np.ascontiguousarray(cu, dtype=np.int32)
        n = len(cu) - 1
        toks = np.zeros((n, max_tokens, 3), dtype=np.uint32)
        counts = np.zeros(n, dtype=np.int32)
        lib().or_tdt_decode_batch(self.h, _p(pooler), _p(cu), n, _p(toks), _p(counts), max_tokens)
        return [toks[i, : min(int(counts[i]), max_tokens)] for i in range(n)]

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_tdt_free(self.h)
            self.h = None
