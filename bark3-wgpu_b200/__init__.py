"""bark3_b200 — Python view of the B200 encoder library (libbark3_b200.so).

The library's C ABI (include/bark3_b200.h) is the product boundary; this
module is a thin ctypes binding used by the tests, the benchmark and the smoke
check, mirroring the reference crate's encoder seam:

    Encoder(device)            ~ Encoder::load_with(Gpu, &dyn WeightSource)
                                 (src/encoder.rs:412)
    .load(weights) / .finalize ~ WeightSource::read / read_lowbit
                                 (src/weights.rs:22-36)
    .encode(sub, layers)       ~ CpuEncoder::encode (src/cpu/mod.rs:156)
    .encode_batch(sub, cu)     varlen batch (one utterance per segment)
    .linear_lut4(...)          Ctx::gemm_f32 with a low-bit weight + add_bias
                               (src/encoder.rs:1039-1100)

There is no CPU fallback: if the shared library is missing or cannot load,
every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

PKG_DIR = pathlib.Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libbark3_b200.so"
HEADER = PKG_DIR.parent / "include" / "bark3_b200.h"

B3_OK = 0
B3_EINVAL = -1
B3_ENOMEM = -2
B3_ECUDA = -3
B3_ETIMEOUT = -4
B3_ESTATE = -5
B3_ENOTFOUND = -6
B3_DEVICE_PTRS = 1
B3_DECODER_AUTO, B3_DECODER_SPLIT_K = 0, 1
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2

N_LAYERS = 24
HIDDEN = 1024


class B3Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"bark3_b200 error {code}: {msg}")
        self.code = code


_lib = None


def build(force: bool = False) -> pathlib.Path:
    """Compile libbark3_b200.so in place with nvcc (sm_100a)."""
    if force or not LIB_PATH.exists():
        subprocess.run(["make", "-C", str(PKG_DIR), "-j8"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    """The loaded CUDA library.  Raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise B3Error(B3_ESTATE, f"{LIB_PATH} is not built (run make -C {PKG_DIR})")
    L = ctypes.CDLL(str(LIB_PATH))
    c_p, c_i, c_u = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint
    sig = {
        "b3_last_error": (ctypes.c_char_p, []),
        "b3_version": (c_i, []),
        "b3_create": (c_p, [c_i]),
        "b3_destroy": (None, [c_p]),
        "b3_sync": (c_i, [c_p]),
        "b3_stream": (c_p, [c_p]),
        "b3_set_wait_limit": (c_i, [c_p, ctypes.c_int64]),
        "b3_set_decoder": (c_i, [c_p, c_i]),
        "b3_load_tensor": (c_i, [c_p, ctypes.c_char_p, c_i, c_p, c_i, c_p]),
        "b3_load_lowbit": (c_i, [c_p, ctypes.c_char_p, c_p, c_p, c_i, c_i]),
        "b3_load_lowbit_levels": (c_i, [c_p, ctypes.c_char_p, c_p, c_p, c_i, c_i, c_i]),
        "b3_finalize": (c_i, [c_p, c_i]),
        "b3_encode": (c_i, [c_p, c_p, c_i, c_i, c_p, c_u]),
        "b3_encode_batch": (c_i, [c_p, c_p, c_p, c_i, c_p, c_u]),
        "b3_linear_lut4": (c_i, [c_p, c_p, c_p, c_p, c_p, c_p, c_i, c_i, c_i, c_u]),
        "b3_linear_f16": (c_i, [c_p, c_p, c_p, c_p, c_p, c_i, c_i, c_i, c_u]),
        "b3_attn_conv": (c_i, [c_p, c_i, c_p, c_i, c_u]),
        "b3_linear_lut4_noalloc": (c_i, [c_p, c_p, c_p, c_p, c_p, c_i, c_i, c_i, c_p]),
        "b3_profile": (c_i, [c_p, c_i]),
        "b3_profile_read": (c_i, [c_p, c_i, c_p, c_p, c_p, c_p]),
        "b3_shard_lpt": (c_i, [c_p, c_i, c_i, c_p]),
        "b3_decode_batch": (c_i, [c_p, c_p, c_p, c_i, c_p, c_p, c_i, c_u]),
        "b3_transcribe_batch": (c_i, [c_p, c_p, c_p, c_i, c_p, c_p, c_i, c_u]),
        "b3_transcribe_audio": (c_i, [c_p, c_p, c_p, c_i, c_p, c_p, c_i, c_u]),
        "b3_encode_audio": (c_i, [c_p, c_p, c_p, c_i, c_p, c_p, ctypes.c_int64, c_u]),
        "b3_mel": (c_i, [c_p, c_p, c_p, c_i, c_p, c_p, c_u]),
        "b3_subsample": (c_i, [c_p, c_p, c_p, c_p, c_i, c_p, c_p, c_u]),
        "b3_mel_filters": (c_i, [c_p]),
        "b3_bark_ans_cdf": (c_i, [c_p, c_i, c_p]),
        "b3_bark_ans_decode": (c_i, [c_p, c_i, c_p, ctypes.c_int64, ctypes.c_int64, c_p]),
        "b3_bark_decode_levels2": (c_i, [c_p, ctypes.c_int64, c_p, ctypes.c_int64, c_i, c_i, c_i, c_p]),
        "b3_bark_decode_ansint": (c_i, [c_p, c_i, c_p, ctypes.c_int64, ctypes.c_int64, c_i, c_p, ctypes.c_int64,
                                        c_p]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def header_symbols() -> list[str]:
    """Function names declared in include/bark3_b200.h."""
    import re

    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(b3_\w+)\s*\(", text, re.M)))


def last_error() -> str:
    msg = lib().b3_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> None:
    if rc != B3_OK:
        raise B3Error(rc, last_error())


def check_bark(name: str, fn: str, *args) -> None:
    """Calls a .bark stream decoder of the library; a failure raises
    BarkError("<tensor>: <reason>")."""
    from .bark import BarkError

    rc = getattr(lib(), fn)(*args)
    if rc != 0:
        raise BarkError(f"{name}: {last_error()}")


def _ptr(a) -> int | None:
    """Address of a contiguous numpy array or torch tensor (None passes NULL)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"], "arrays must be C-contiguous"
        return a.ctypes.data
    return a.data_ptr()  # torch tensor


def _is_device(a) -> bool:
    return a is not None and not isinstance(a, np.ndarray) and getattr(a, "is_cuda", False)


class Encoder:
    """One b3_ctx: a device-resident encoder on one GPU."""

    def __init__(self, device: int = 0):
        self._L = lib()
        self.ctx = self._L.b3_create(device)
        if not self.ctx:
            raise B3Error(B3_ECUDA, last_error())
        self.device = device
        self.n_layers = 0

    def close(self) -> None:
        if self.ctx:
            self._L.b3_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ── weights ──
    def load(self, weights: dict) -> None:
        """weights: name -> np.ndarray (f32 / f16-bits uint16 with dtype tag) or
        ("lut4", codes u8 [rows, cols/2], lut16 u16 [rows, 16]) or
        ("levels", code_words u32, levels u16 [rows, 4], k) or
        ("bf16", bits u16 array)."""
        for name, v in weights.items():
            self.load_one(name, v)

    def load_one(self, name: str, v) -> None:
        nm = name.encode()
        L = self._L
        if isinstance(v, tuple) and v[0] == "lut4":
            _, codes, lut16 = v
            codes = np.ascontiguousarray(codes, dtype=np.uint8)
            lut16 = np.ascontiguousarray(lut16, dtype=np.uint16)
            check(L.b3_load_lowbit(self.ctx, nm, _ptr(codes), _ptr(lut16), lut16.shape[0], codes.shape[1] * 2))
        elif isinstance(v, tuple) and v[0] == "levels":
            _, words, levels, k, cols = v
            words = np.ascontiguousarray(words, dtype=np.uint32)
            levels = np.ascontiguousarray(levels, dtype=np.uint16)
            check(L.b3_load_lowbit_levels(self.ctx, nm, _ptr(words), _ptr(levels), k, levels.shape[0], cols))
        elif isinstance(v, tuple) and v[0] in ("bf16", "f16"):
            _, bits = v
            bits = np.ascontiguousarray(bits, dtype=np.uint16)
            shape = (ctypes.c_int64 * bits.ndim)(*bits.shape)
            dt = DTYPE_BF16 if v[0] == "bf16" else DTYPE_F16
            check(L.b3_load_tensor(self.ctx, nm, dt, shape, bits.ndim, _ptr(bits)))
        else:
            arr = np.ascontiguousarray(v, dtype=np.float32)
            shape = (ctypes.c_int64 * arr.ndim)(*arr.shape)
            check(L.b3_load_tensor(self.ctx, nm, DTYPE_F32, shape, arr.ndim, _ptr(arr)))

    def load_source(self, src, threads: int | None = None) -> int:
        """Loads every float tensor of a checkpoint source (bark.BarkContainer
        or bark.SafetensorsSource, see bark.open_weights) the way the
        reference's Encoder::load_with reads a WeightSource
        (src/encoder.rs:412-560): 4-bit tensors in their code-word + level
        form, everything else at its stored precision (f16 / bf16 bits, or
        f32 for dequantised integer matrices); integer tensors are skipped.
        Returns the encoder layer count the source describes."""
        from . import bark

        src.prefetch(threads)
        for name in src.tensor_names():
            lb = src.read_lowbit(name)
            if lb is not None:
                self.load_one(name, ("levels", lb.codes, lb.levels, lb.k, lb.cols))
                continue
            if isinstance(src, bark.SafetensorsSource) and src.read_dtype(name) == "BF16":
                self.load_one(name, ("bf16", src.read(name)))
                continue
            v = src.read(name)
            if v.dtype == np.float16:
                self.load_one(name, ("f16", v.view(np.uint16)))
            elif v.dtype == np.float32:
                self.load_one(name, v)
        if isinstance(src, bark.BarkContainer):
            return src.layers()
        return len({n.split(".")[2] for n in src.tensor_names() if n.startswith("encoder.layers.")})

    def finalize(self, n_layers: int = N_LAYERS) -> None:
        check(self._L.b3_finalize(self.ctx, n_layers))
        self.n_layers = n_layers

    # ── compute ──
    def encode(self, sub, layers: int | None = None, out=None):
        """sub: (t, 4096) f32.  Returns the pooler (t, 640) when layers covers
        every block, else the residual (t, 1024) after block layers-1."""
        layers = self.n_layers if layers is None else layers
        t = sub.shape[0]
        cols = 640 if layers >= self.n_layers else HIDDEN
        dev = _is_device(sub)
        if out is None:
            out = _empty_like_kind(sub, (t, cols))
        flags = B3_DEVICE_PTRS if dev else 0
        check(self._L.b3_encode(self.ctx, _ptr(sub), t, layers, _ptr(out), flags))
        return out

    def encode_batch(self, sub, cu_seqlens, out=None):
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        total = int(cu[-1])
        dev = _is_device(sub)
        if out is None:
            out = _empty_like_kind(sub, (total, 640))
        flags = B3_DEVICE_PTRS if dev else 0
        check(self._L.b3_encode_batch(self.ctx, _ptr(sub), _ptr(cu), len(cu) - 1, _ptr(out), flags))
        return out

    def decode_batch(self, pooler, cu_seqlens, max_tokens: int = 4096):
        """Greedy TDT decode of a varlen pooler; returns a list of (n, 3)
        uint32 arrays (id, frame, duration) per utterance."""
        return self._tokens_call("b3_decode_batch", pooler, cu_seqlens, max_tokens)

    def transcribe_batch(self, sub, cu_seqlens, max_tokens: int = 4096):
        """Encoder + decoder: subsampled frames -> token streams per utterance."""
        return self._tokens_call("b3_transcribe_batch", sub, cu_seqlens, max_tokens)

    def transcribe_audio(self, waves, max_tokens: int = 4096):
        """16 kHz mono utterances (list of f32 arrays) -> token streams; the
        0.25 s lead-in of the reference pipeline is added by the library."""
        off = np.concatenate([[0], np.cumsum([len(w) for w in waves])]).astype(np.int64)
        samples = np.ascontiguousarray(np.concatenate(waves), dtype=np.float32)
        n = len(waves)
        tokens = np.zeros((n, max_tokens, 3), dtype=np.uint32)
        counts = np.zeros(n, dtype=np.int32)
        check(self._L.b3_transcribe_audio(self.ctx, _ptr(samples), _ptr(off), n, _ptr(tokens), _ptr(counts),
                                          max_tokens, 0))
        return [tokens[i, : min(int(counts[i]), max_tokens)] for i in range(n)]

    def encode_audio(self, waves):
        """16 kHz utterances -> (pooler [sum T][640] f32, row offsets): the
        encoder half of transcribe_audio on the same audio."""
        off = np.concatenate([[0], np.cumsum([len(w) for w in waves])]).astype(np.int64)
        samples = np.ascontiguousarray(np.concatenate(waves), dtype=np.float32)
        n = len(waves)
        rows = sum(frames_for_seconds(len(w) / 16000.0) for w in waves)
        pooler = np.zeros((rows, 640), dtype=np.float32)
        roff = np.zeros(n + 1, dtype=np.int32)
        check(self._L.b3_encode_audio(self.ctx, _ptr(samples), _ptr(off), n, _ptr(pooler), _ptr(roff), rows, 0))
        return pooler[: roff[n]], roff

    def mel(self, waves):
        """Padded waves -> list of (frames, 128) normalised log-mel arrays."""
        off = np.concatenate([[0], np.cumsum([len(w) for w in waves])]).astype(np.int64)
        samples = np.ascontiguousarray(np.concatenate(waves), dtype=np.float32)
        n = len(waves)
        frames = int(sum(1 + len(w) // 160 for w in waves))
        out = np.zeros((frames, 128), dtype=np.float32)
        foff = np.zeros(n + 1, dtype=np.int32)
        check(self._L.b3_mel(self.ctx, _ptr(samples), _ptr(off), n, _ptr(out), _ptr(foff), 0))
        return [out[foff[i]:foff[i + 1]] for i in range(n)]

    def subsample(self, mels, n_valid):
        """List of (frames, 128) mel arrays -> list of (T, 4096) rows."""
        foff = np.concatenate([[0], np.cumsum([m.shape[0] for m in mels])]).astype(np.int32)
        mel = np.ascontiguousarray(np.concatenate(mels), dtype=np.float32)
        nv = np.ascontiguousarray(n_valid, dtype=np.int32)
        n = len(mels)

        def clen(v):
            return (v - 1) // 2 + 1

        total = int(sum(clen(clen(clen(m.shape[0]))) for m in mels))
        out = np.zeros((total, 4096), dtype=np.float32)
        roff = np.zeros(n + 1, dtype=np.int32)
        check(self._L.b3_subsample(self.ctx, _ptr(mel), _ptr(foff), _ptr(nv), n, _ptr(out), _ptr(roff), 0))
        return [out[roff[i]:roff[i + 1]] for i in range(n)]

    def _tokens_call(self, fn, src, cu_seqlens, max_tokens):
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        n = len(cu) - 1
        tokens = np.zeros((n, max_tokens, 3), dtype=np.uint32)
        counts = np.zeros(n, dtype=np.int32)
        if _is_device(src):
            import torch

            tt = torch.zeros((n, max_tokens, 3), dtype=torch.int32, device=src.device)
            tc = torch.zeros(n, dtype=torch.int32, device=src.device)
            check(getattr(self._L, fn)(self.ctx, _ptr(src), _ptr(cu), n, _ptr(tt), _ptr(tc), max_tokens,
                                       B3_DEVICE_PTRS))
            self.sync()
            tokens = tt.cpu().numpy().view(np.uint32)
            counts = tc.cpu().numpy()
        else:
            src = np.ascontiguousarray(src, dtype=np.float32)
            check(getattr(self._L, fn)(self.ctx, _ptr(src), _ptr(cu), n, _ptr(tokens), _ptr(counts), max_tokens, 0))
        return [tokens[i, : min(int(counts[i]), max_tokens)] for i in range(n)]

    def attn_conv(self, layer: int, x) -> None:
        flags = B3_DEVICE_PTRS if _is_device(x) else 0
        check(self._L.b3_attn_conv(self.ctx, layer, _ptr(x), x.shape[0], flags))

    def linear_lut4(self, a, codes, lut16, bias=None, out=None):
        m, k = a.shape
        n = lut16.shape[0]
        dev = _is_device(a)
        if out is None:
            out = _empty_like_kind(a, (m, n))
        flags = B3_DEVICE_PTRS if dev else 0
        check(self._L.b3_linear_lut4(self.ctx, _ptr(a), _ptr(codes), _ptr(lut16), _ptr(bias), _ptr(out), m, n, k, flags))
        return out

    def linear_f16(self, a, w16, bias=None, out=None):
        m, k = a.shape
        n = w16.shape[0]
        dev = _is_device(a)
        if out is None:
            out = _empty_like_kind(a, (m, n))
        flags = B3_DEVICE_PTRS if dev else 0
        check(self._L.b3_linear_f16(self.ctx, _ptr(a), _ptr(w16), _ptr(bias), _ptr(out), m, n, k, flags))
        return out

    def sync(self) -> None:
        check(self._L.b3_sync(self.ctx))

    @property
    def stream(self) -> int:
        return self._L.b3_stream(self.ctx)


def _empty_like_kind(ref, shape):
    if isinstance(ref, np.ndarray):
        return np.empty(shape, dtype=np.float32)
    import torch

    return torch.empty(shape, dtype=torch.float32, device=ref.device)


def mel_filters() -> np.ndarray:
    """The (128, 257) slaney filterbank the library's front end uses."""
    out = np.zeros((128, 257), dtype=np.float32)
    check(lib().b3_mel_filters(_ptr(out)))
    return out


def shard_lpt(frames, n_ranks: int) -> np.ndarray:
    """rank_of[i] for each utterance (b3_shard_lpt: longest processing time
    first by the estimated encoder cost)."""
    fr = np.ascontiguousarray(frames, dtype=np.int32)
    out = np.empty(len(fr), dtype=np.int32)
    check(lib().b3_shard_lpt(_ptr(fr), len(fr), n_ranks, _ptr(out)))
    return out


def frames_for_seconds(seconds: float) -> int:
    """Encoder frames T for an utterance of `seconds` at 16 kHz: the pipeline
    prepends 0.25 s (src/transcription.rs:48-52), the mel front end produces
    1 + len/160 frames (src/mel.rs:50) and three stride-2 convs give
    l -> (l - 1)//2 + 1 each (src/sub.rs:11-13, 283)."""
    n = int(round(seconds * 16000)) + 4000
    v = 1 + n // 160
    for _ in range(3):
        v = (v - 1) // 2 + 1
    return v
