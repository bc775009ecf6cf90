"""Reader for the `model.bark` weight container and the checkpoint sources.

Mirrors the reference's `BarkContainer` (src/bark.rs:98-560) and
`weights::open` / `open_bytes` / `looks_like_container`
(src/weights.rs:84-136):

    BarkContainer.open(dir)          BarkContainer::open (src/bark.rs:98-117)
    BarkContainer.from_bytes(data)   BarkContainer::from_bytes (:119-133)
    .info() / .tensor_names() / .tensor_count() / .layers()
    .read_lowbit(name)               4-bit form or None (:273-291)
    .read(name)                      values as an array (:362-452)
    .prefetch(threads)               decode every 4-bit tensor in parallel (:454-476)
    open_weights(dir)                model.bark, else model.safetensors
    looks_like_container(data)

The JSON index and the LZMA-compressed fields are parsed here (json and the
standard library's lzma: xz when the bytes carry the xz magic, the legacy
.lzma format otherwise, as src/bark.rs:256-271 chooses); the ANS entropy
decoding of the code streams runs in the native library
(b3_bark_decode_levels2 / b3_bark_decode_ansint), one tensor per call with
the GIL released, so prefetch() decodes tensors on several cores at once.

Errors raise BarkError with the reference's messages.
"""
from __future__ import annotations

import json
import lzma
import math
import os
import pathlib
import re
import struct
import threading
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

FORMATS = ("bark-levels-v2", "bark-levels-v3")
_XZ_MAGIC = b"\xfd7zXZ\x00"


class BarkError(ValueError):
    """A malformed or unsupported container."""


@dataclass
class LowBitTensor:
    """One 4-bit tensor in the layout the encoder loads (src/bark.rs:33-48):
    codes [rows][ceil(cols/8)] u32 (nibble col % 8 of word col / 8) and
    levels [rows][4] f16 bits (the first k in use, zero padded)."""

    codes: np.ndarray
    levels: np.ndarray
    k: int
    rows: int
    cols: int

    def code_words(self) -> int:
        return self.rows * ((self.cols + 7) // 8)

    def expand(self) -> np.ndarray:
        """f32 values by the sign-magnitude rule of `expand`
        (src/bark.rs:597-611): 0 -> 0, 1..k -> +lev[c-1], k+1.. -> -lev[c-k-1]
        (a magnitude index past the k levels reads 0)."""
        col = np.arange(self.cols)
        codes = (self.codes[:, col // 8] >> (4 * (col % 8)).astype(np.uint32)) & 0xF
        lev = self.levels.view(np.float16).astype(np.float32)
        table = np.zeros((self.rows, 16), np.float32)
        for c in range(1, 16):
            neg = c > self.k
            mag = c - self.k - 1 if neg else c - 1
            v = lev[:, mag] if mag < self.k else np.zeros(self.rows, np.float32)
            table[:, c] = -v if neg else v
        return np.take_along_axis(table, codes.astype(np.int64), axis=1)


@dataclass
class ModelInfo:
    """What a checkpoint holds (crate::weights_io::ModelInfo)."""

    release: str | None
    layout: str
    tensors: int
    weights: int
    layers: int
    hidden: int
    ffn: int
    vocab: int


@dataclass
class _Entry:
    kind: str          # "levels2" | "ansint" | "raw"
    bits: int
    shape: list
    level_count: int
    offset: int
    lev: int
    meta: int
    words: int
    scale: int
    zipped_levels: bool
    zipped_scale: bool
    zipped_raw: bool
    raw_dtype: str     # "f16" | "i64" | "i32"

    def n(self) -> int:
        return int(math.prod(self.shape))

    def rows_cols(self) -> tuple[int, int]:
        rows = self.shape[0]
        return rows, self.n() // max(rows, 1)


def _u64(v) -> int:
    """serde_json's as_u64().unwrap_or(0)."""
    return v if isinstance(v, int) and not isinstance(v, bool) and 0 <= v < 1 << 64 else 0


def _flag(e: dict, key: str) -> bool:
    if key not in e:
        return False
    v = e[key]
    return v if isinstance(v, bool) else _u64(v) != 0


def _read_header(data_at) -> bytes:
    """src/bark.rs:487-507: u64 length (0 < len < 64 MiB), JSON with a
    bark-levels-v2/v3 `format`."""
    raw = data_at(0, 8)
    if len(raw) < 8:
        raise BarkError("header: file is shorter than its length prefix")
    (n,) = struct.unpack("<Q", raw)
    if not (0 < n < 64 << 20):
        raise BarkError(f"header claims {n} bytes")
    header = data_at(8, n)
    if len(header) != n:
        raise BarkError("header: file ends inside the header")
    try:
        head = json.loads(header)
    except ValueError as ex:
        raise BarkError("header is not JSON") from ex
    fmt = head.get("format") if isinstance(head, dict) else None
    fmt = fmt if isinstance(fmt, str) else ""
    if fmt not in FORMATS:
        raise BarkError(f"unsupported container format {fmt!r}")
    return header


def _parse_index(header: bytes, base: int) -> dict[str, _Entry]:
    """src/bark.rs:509-559: entries in index order, payloads back to back."""
    head = json.loads(header)
    index = head.get("index")
    if not isinstance(index, list):
        raise BarkError("container index")
    entries: dict[str, _Entry] = {}
    offset = base
    for e in index:
        if not isinstance(e, dict):
            raise BarkError("container index")
        name = e.get("n")
        if not isinstance(name, str):
            raise BarkError("tensor name")
        shape = e.get("shape")
        if not isinstance(shape, list):
            raise BarkError(f"{name}: tensor shape")
        shape = [_u64(v) for v in shape]
        kind = e.get("k") if isinstance(e.get("k"), str) else ""
        bits = 0
        if kind == "levels2" or kind == "raw":
            pass
        elif kind.startswith("ansint"):
            digits = kind[6:]
            if not re.fullmatch(r"\+?[0-9]+", digits) or int(digits) >= 1 << 32:
                raise BarkError(f"{name}: {kind}")
            bits = int(digits)
            kind = "ansint"
        else:
            raise BarkError(f"{name}: unsupported entry kind {kind!r}")
        dt = e.get("dtype")
        raw_dtype = {"torch.int64": "i64", "torch.int32": "i32"}.get(dt if isinstance(dt, str) else "", "f16")
        ent = _Entry(kind=kind, bits=bits, shape=shape, level_count=_u64(e.get("K")), offset=offset,
                     lev=_u64(e.get("lev")), meta=_u64(e.get("meta")), words=_u64(e.get("b")),
                     scale=_u64(e.get("s")), zipped_levels=_flag(e, "zl"), zipped_scale=_flag(e, "zs"),
                     zipped_raw=_flag(e, "zr"), raw_dtype=raw_dtype)
        offset += ent.lev + ent.meta + ent.words + ent.scale
        entries[name] = ent
    return entries


def looks_like_container(data: bytes) -> bool:
    """src/weights.rs:102-124: length-prefixed JSON whose `format` starts with
    "bark-levels-" (a safetensors file is length-prefixed JSON too)."""
    if len(data) <= 8:
        return False
    (n,) = struct.unpack("<Q", bytes(data[:8]))
    if not (0 < n < 64 << 20 and len(data) > 8 + n):
        return False
    try:
        head = json.loads(bytes(data[8:8 + n]))
    except ValueError:
        return False
    fmt = head.get("format") if isinstance(head, dict) else None
    return isinstance(fmt, str) and fmt.startswith("bark-levels-")


def _words(b: bytes) -> np.ndarray:
    """chunks_exact(4) as little-endian u32 (a ragged tail is dropped)."""
    return np.frombuffer(b, dtype="<u4", count=len(b) // 4).astype(np.uint32)


class BarkContainer:
    def __init__(self, data_at, entries: dict[str, _Entry], release: str | None, closer=None):
        self._data_at = data_at
        self._entries = entries
        self._cache: dict[str, LowBitTensor] = {}
        self._lock = threading.Lock()
        self._closer = closer
        self._info = self._describe(release)

    # ── construction ──
    @classmethod
    def open(cls, dir) -> "BarkContainer":
        """<dir>/model.bark, read with positional reads (prefetch reads from
        several threads)."""
        path = pathlib.Path(dir) / "model.bark"
        try:
            fd = os.open(path, os.O_RDONLY)
        except OSError as ex:
            raise BarkError(f"open {path}: {ex.strerror}") from ex
        size = os.fstat(fd).st_size

        def data_at(off: int, n: int) -> bytes:
            if n == 0:
                return b""
            if off + n > size:
                raise BarkError("read container blob: unexpected end of file")
            return os.pread(fd, n, off)

        try:
            header = _read_header(data_at)
            entries = _parse_index(header, 8 + len(header))
        except BarkError as ex:
            os.close(fd)
            raise BarkError(f"{path}: {ex}") from ex
        return cls(data_at, entries, pathlib.Path(dir).name or None, closer=lambda: os.close(fd))

    @classmethod
    def from_bytes(cls, data: bytes, release: str | None = None) -> "BarkContainer":
        buf = memoryview(bytes(data))

        def data_at(off: int, n: int) -> bytes:
            if n == 0:
                return b""
            if off + n > len(buf):
                raise BarkError("blob outside the buffer")
            return buf[off:off + n].tobytes()

        try:
            header = _read_header(lambda o, n: buf[o:o + n].tobytes())
        except BarkError as ex:
            raise BarkError(f"container header: {ex}") from ex
        return cls(data_at, _parse_index(header, 8 + len(header)), release)

    def close(self) -> None:
        if self._closer:
            self._closer()
            self._closer = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ── description ──
    def _describe(self, release) -> ModelInfo:
        weights = sum(e.n() for e in self._entries.values() if e.raw_dtype == "f16")
        arch = self._architecture()
        return ModelInfo(release=release, layout="lowbit", tensors=len(self._entries), weights=weights, layers=arch[0],
                         hidden=arch[1], ffn=arch[2], vocab=arch[3])

    def _architecture(self) -> tuple[int, int, int, int]:
        ffn = self._entries.get("encoder.layers.0.feed_forward1.linear1.weight")
        emb = self._entries.get("decoder.embedding.weight")
        if ffn is None or emb is None or not ffn.shape or not emb.shape:
            return (0, 0, 0, 0)
        rows, hidden = ffn.rows_cols()
        return (self.layers(), hidden, rows, emb.shape[0])

    def info(self) -> ModelInfo:
        return self._info

    def tensor_names(self) -> list[str]:
        return sorted(self._entries)

    def tensor_count(self) -> int:
        return len(self._entries)

    def layers(self) -> int:
        seen = set()
        for name in self._entries:
            if name.startswith("encoder.layers."):
                n, dot, _ = name[len("encoder.layers."):].partition(".")
                if dot and n.isdigit():
                    seen.add(int(n))
        return len(seen)

    def kind(self, name: str) -> str:
        return self._entry(name).kind

    def shape(self, name: str) -> list[int]:
        return list(self._entry(name).shape)

    # ── payloads ──
    def _entry(self, name: str) -> _Entry:
        e = self._entries.get(name)
        if e is None:
            raise BarkError(f"{name}: not in the container")
        return e

    def _field(self, e: _Entry, off: int, n: int, zipped: bool) -> bytes:
        raw = self._data_at(e.offset + off, n)
        if not zipped:
            return raw
        try:
            if raw.startswith(_XZ_MAGIC):
                return lzma.decompress(raw, format=lzma.FORMAT_XZ)
            return lzma.decompress(raw, format=lzma.FORMAT_ALONE)
        except lzma.LZMAError as ex:
            raise BarkError("xz" if raw.startswith(_XZ_MAGIC) else "lzma") from ex

    def read_lowbit(self, name: str) -> LowBitTensor | None:
        """The 4-bit form, or None when the tensor is stored another way; the
        first call decodes, later calls return the cached tensor."""
        with self._lock:
            hit = self._cache.get(name)
        if hit is not None:
            return hit
        e = self._entry(name)
        if e.kind != "levels2":
            return None
        try:
            t = self._decode_levels2(name, e)
        except BarkError as ex:
            raise BarkError(f"{name}: decoding levels2 entry at offset {e.offset}: {ex}") from ex
        with self._lock:
            return self._cache.setdefault(name, t)

    def _decode_levels2(self, name: str, e: _Entry) -> LowBitTensor:
        from . import check_bark

        rows, cols = e.rows_cols()
        k = e.level_count
        if not 1 <= k <= 3:
            raise BarkError(f"{name}: unsupported level count {k}")
        lev = self._field(e, 0, e.lev, e.zipped_levels)
        if len(lev) != rows * k * 2:
            raise BarkError(f"{name}: level table is {len(lev)} bytes, expected {rows * k * 2}")
        meta = self._field(e, e.lev, e.meta, False)
        words = _words(self._field(e, e.lev + e.meta, e.words, False))
        levels = np.zeros((rows, 4), np.uint16)
        levels[:, :k] = np.frombuffer(lev, dtype="<u2").reshape(rows, k)
        if rows == 0 or cols == 0:
            return LowBitTensor(np.zeros((rows, (cols + 7) // 8), np.uint32), levels, k, rows, cols)
        codes = np.zeros((rows, (cols + 7) // 8), np.uint32)
        meta_a = np.frombuffer(meta, dtype=np.uint8) if meta else np.zeros(1, np.uint8)
        check_bark(name, "b3_bark_decode_levels2", meta_a.ctypes.data, len(meta), words.ctypes.data, len(words), rows,
                   cols, k, codes.ctypes.data)
        return LowBitTensor(codes, levels, k, rows, cols)

    def read(self, name: str) -> np.ndarray:
        """The tensor's values: 4-bit layers expanded to their f32 levels,
        integer layers to q * row_scale (f32), raw entries as float16 / int64
        / int32 arrays of the recorded shape."""
        try:
            return self._read(name)
        except BarkError as ex:
            raise BarkError(f"{name}: reading container entry: {ex}") from ex

    def _read(self, name: str) -> np.ndarray:
        from . import check_bark

        e = self._entry(name)
        if e.kind == "levels2":
            return self.read_lowbit(name).expand().reshape(e.shape)
        if e.kind == "ansint":
            if not 1 <= e.bits <= 16:
                raise BarkError(f"{name}: ansint{e.bits}")
            sb = self._field(e, 0, e.scale, e.zipped_scale)
            scales = np.frombuffer(sb, dtype="<u2", count=len(sb) // 2).astype(np.uint16)
            meta = self._field(e, e.scale, e.meta, False)
            counts = _words(meta)
            if not counts.size or float(counts.astype(np.float64).sum()) <= 0.0:
                raise BarkError(f"{name}: empty symbol table")
            words = _words(self._field(e, e.scale + e.meta, e.words, False))
            n = e.n()
            out = np.zeros(n, np.float32)
            sc = scales if scales.size else np.zeros(1, np.uint16)
            check_bark(name, "b3_bark_decode_ansint", counts.ctypes.data, len(counts), words.ctypes.data, len(words),
                       n, e.bits, sc.ctypes.data, scales.size, out.ctypes.data)
            return out.reshape(e.shape)
        data = self._field(e, 0, e.words, e.zipped_raw)
        dt = {"i64": "<i8", "i32": "<i4", "f16": "<f2"}[e.raw_dtype]
        width = np.dtype(dt).itemsize
        if len(data) != e.n() * width:
            raise BarkError(f"{name}: {len(data)} bytes for {e.n()} values of {width} bytes")
        return np.frombuffer(data, dtype=dt).reshape(e.shape).astype(dt[1:])

    def prefetch(self, threads: int | None = None) -> None:
        """Decode every 4-bit tensor, one tensor per worker."""
        names = [n for n, e in self._entries.items() if e.kind == "levels2"]
        workers = threads or os.cpu_count() or 1
        if workers <= 1 or len(names) <= 1:
            for n in names:
                self.read_lowbit(n)
            return
        with ThreadPoolExecutor(max_workers=min(workers, len(names))) as ex:
            for _ in ex.map(self.read_lowbit, names):
                pass


# ───────────────────────────── safetensors ─────────────────────────────
class SafetensorsSource:
    """`model.safetensors` (the bf16 Pro release; src/weights.rs:40-66): a
    length-prefixed JSON table of {dtype, shape, data_offsets} and the raw
    little-endian tensor bytes.  read() returns float16 / int arrays as
    stored, and bf16 as its uint16 bit patterns (read_dtype() says which)."""

    _DT = {"F16": "<f2", "BF16": "<u2", "F32": "<f4", "I64": "<i8", "I32": "<i4"}

    def __init__(self, data: bytes, release: str | None = None):
        self._buf = memoryview(bytes(data))
        if len(self._buf) < 8:
            raise BarkError("safetensors: file is shorter than its length prefix")
        (n,) = struct.unpack("<Q", self._buf[:8].tobytes())
        if not 0 < n <= len(self._buf) - 8:
            raise BarkError(f"safetensors: header claims {n} bytes")
        try:
            head = json.loads(self._buf[8:8 + n].tobytes())
        except ValueError as ex:
            raise BarkError("safetensors: header is not JSON") from ex
        self._base = 8 + n
        self._meta = {k: v for k, v in head.items() if k != "__metadata__"}
        self.release = release

    @classmethod
    def open(cls, dir) -> "SafetensorsSource":
        path = pathlib.Path(dir) / "model.safetensors"
        return cls(path.read_bytes(), pathlib.Path(dir).name or None)

    def tensor_names(self) -> list[str]:
        return sorted(self._meta)

    def read_dtype(self, name: str) -> str:
        return self._spec(name)["dtype"]

    def _spec(self, name: str) -> dict:
        s = self._meta.get(name)
        if s is None:
            raise BarkError(f"{name}: not in the checkpoint")
        return s

    def read(self, name: str) -> np.ndarray:
        s = self._spec(name)
        dt = self._DT.get(s["dtype"])
        if dt is None:
            raise BarkError(f"{name}: unsupported dtype {s['dtype']}")
        a, b = s["data_offsets"]
        if not 0 <= a <= b <= len(self._buf) - self._base:
            raise BarkError(f"{name}: data outside the file")
        arr = np.frombuffer(self._buf[self._base + a:self._base + b].tobytes(), dtype=dt)
        return arr.reshape(s["shape"]).astype(dt[1:])

    def read_lowbit(self, name: str):
        self._spec(name)
        return None

    def prefetch(self, threads: int | None = None) -> None:
        return None


def open_weights(dir):
    """src/weights.rs:86-100: model.bark when present, else model.safetensors."""
    d = pathlib.Path(dir)
    if (d / "model.bark").is_file():
        return BarkContainer.open(d)
    if (d / "model.safetensors").is_file():
        return SafetensorsSource.open(d)
    raise BarkError(f"{d} has neither model.bark nor model.safetensors")


def open_bytes(data: bytes, release: str | None = None):
    """src/weights.rs:126-136: the layout is sniffed from the bytes."""
    if looks_like_container(data):
        return BarkContainer.from_bytes(data, release)
    return SafetensorsSource(data, release)
