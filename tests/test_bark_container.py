"""The `model.bark` loader (bark3_b200.bark + the library's ANS decoders)
against the container layout and entropy coding the reference reads
(src/bark.rs:98-611, src/weights.rs:84-136).  CPU only: the stream decoders
are host code.

No `.bark` release file or constriction-written stream is available here, so
the ANS restatement is pinned by round trips through the oracle's encoder and
by agreement of three independent decoders (product C++, oracle C, oracle
pure Python): parity of the entropy coding itself is unpinned.  The layout
(class order, column-major symbol order, nibble packing, level table, raw
widths, LZMA flags, offsets) is checked exactly."""
import ctypes
import json
import lzma
import struct

import numpy as np
import pytest

from oracle import bark_container as bc


@pytest.fixture(scope="module")
def bark(pkg):
    import importlib

    return importlib.import_module("bark3_b200.bark")


def unpack_codes(lb):
    col = np.arange(lb.cols)
    return (lb.codes[:, col // 8] >> (4 * (col % 8)).astype(np.uint32)) & 0xF


# ───────────────────────────── entropy coding ─────────────────────────────
@pytest.mark.parametrize("n", [2, 3, 5, 7, 13, 64])
def test_cdf_three_ways(pkg, n):
    rng = np.random.default_rng(n)
    for trial in range(20):
        counts = rng.integers(0, [10, 1000, 1 << 31][trial % 3], n).astype(np.uint32)
        if trial % 4 == 0:
            counts[rng.integers(0, n)] = 0
        if counts.sum() == 0:
            counts[0] = 1
        want = bc.py_ans_cdf(counts)
        assert list(bc.ans_cdf(counts)) == want
        got = np.zeros(n + 1, np.uint32)
        assert pkg.lib().b3_bark_ans_cdf(counts.ctypes.data, n, got.ctypes.data) == 0
        assert list(got) == want
        assert got[-1] == 1 << 24 and np.all(np.diff(got.astype(np.int64)) >= 1)


def test_cdf_rejects_bad_tables(pkg):
    L = pkg.lib()
    out = np.zeros(8, np.uint32)
    for counts in (np.zeros(3, np.uint32), np.array([5], np.uint32)):
        assert L.b3_bark_ans_cdf(counts.ctypes.data, len(counts), out.ctypes.data) == pkg.B3_EINVAL
        assert "invalid symbol table" in pkg.last_error()


@pytest.mark.parametrize("dist", ["skewed", "uniform", "one_hot", "with_zero"])
def test_ans_round_trip(pkg, dist):
    rng = np.random.default_rng(1)
    n_sym = 7
    counts = {"skewed": [1, 50, 400, 3000, 400, 50, 1], "uniform": [1] * 7, "one_hot": [0, 0, 0, 1, 0, 0, 0],
              "with_zero": [10, 0, 30, 0, 5, 5, 5]}[dist]
    counts = np.array(counts, np.uint32)
    p = counts / counts.sum()
    n = 200_000
    sym = rng.choice(n_sym, size=n, p=p).astype(np.uint16)
    words = bc.ans_encode(sym, counts)
    got = np.zeros(n, np.uint16)
    assert pkg.lib().b3_bark_ans_decode(counts.ctypes.data, n_sym, words.ctypes.data, len(words), n,
                                        got.ctypes.data) == 0
    assert np.array_equal(got, sym)
    assert np.array_equal(bc.ans_decode(words, counts, n), sym)
    # the pure-Python restatement agrees on a prefix, from the same stream
    small = sym[:3000]
    w_small = bc.ans_encode(small, counts)
    assert list(w_small) == bc.py_ans_encode(small, counts)
    assert bc.py_ans_decode(w_small, counts, 3000) == list(small)


def test_ans_stream_edges(pkg):
    L = pkg.lib()
    counts = np.array([3, 1, 1], np.uint32)
    out = np.zeros(16, np.uint16)
    # an empty stream decodes from state 0 (symbol 0 forever), as the Vec-backed coder does
    empty = np.zeros(1, np.uint32)
    assert L.b3_bark_ans_decode(counts.ctypes.data, 3, empty.ctypes.data, 0, 16, out.ctypes.data) == 0
    assert np.all(out == 0) and bc.py_ans_decode([], counts, 16) == [0] * 16
    # a zero top word is malformed
    bad = np.array([7, 0], np.uint32)
    assert L.b3_bark_ans_decode(counts.ctypes.data, 3, bad.ctypes.data, 2, 4, out.ctypes.data) == pkg.B3_EINVAL
    assert "truncated ANS stream" in pkg.last_error()
    # reading past the end of the data keeps decoding (no error), like the reference
    words = bc.ans_encode(np.array([1, 2, 1], np.uint16), counts)
    assert L.b3_bark_ans_decode(counts.ctypes.data, 3, words.ctypes.data, len(words), 16, out.ctypes.data) == 0
    assert list(out[:3]) == [1, 2, 1]
    assert list(out) == bc.py_ans_decode(list(words), counts, 16)


# ─────────────────────────────── container ───────────────────────────────
def _levels2_case(rng, rows, cols, k, n_classes=16):
    codes = rng.integers(0, 2 * k + 1, size=(rows, cols)).astype(np.uint8)
    mags = np.sort(np.abs(rng.normal(0, 0.02, size=(rows, k))), axis=1).astype(np.float16).view(np.uint16)
    classes = rng.integers(0, n_classes, cols)
    return codes, mags, classes


@pytest.mark.parametrize("rows,cols,k,zl,n_classes", [
    (96, 100, 3, "xz", 16), (10, 13, 1, "alone", 16), (7, 64, 2, None, 3), (33, 8, 3, None, 1), (5, 1, 2, "xz", 16)])
def test_levels2_layout(bark, rows, cols, k, zl, n_classes):
    rng = np.random.default_rng(rows * cols + k)
    codes, mags, classes = _levels2_case(rng, rows, cols, k, n_classes)
    blob = bc.write_container([bc.levels2_entry("w", codes, mags, k, classes, zl)])
    c = bark.BarkContainer.from_bytes(blob)
    lb = c.read_lowbit("w")
    assert (lb.rows, lb.cols, lb.k) == (rows, cols, k)
    assert lb.codes.shape == (rows, (cols + 7) // 8) and lb.codes.dtype == np.uint32
    assert np.array_equal(unpack_codes(lb), codes)
    assert np.array_equal(lb.levels[:, :k], mags) and np.all(lb.levels[:, k:] == 0)
    # read(): the expand rule (0 -> 0, 1..k -> +lev, k+1..2k -> -lev)
    lev = mags.view(np.float16).astype(np.float32)
    want = np.zeros((rows, cols), np.float32)
    for c_ in range(1, 2 * k + 1):
        m = c_ - 1 if c_ <= k else c_ - k - 1
        sign = 1.0 if c_ <= k else -1.0
        want = np.where(codes == c_, sign * lev[:, m:m + 1], want)
    assert np.array_equal(c.read("w"), want)
    assert c.read_lowbit("w") is lb  # cached


def test_levels2_symbol_order_is_class_then_column_then_row(bark, pkg):
    """Decode the stream directly with one model per class and check that
    symbols land at (row, column) in the reference's scatter order
    (src/bark.rs:327-343)."""
    rng = np.random.default_rng(3)
    rows, cols, k = 4, 6, 1
    codes = rng.integers(0, 3, size=(rows, cols)).astype(np.uint8)
    classes = np.array([2, 0, 2, 1, 0, 2])
    idx, blob = bc.levels2_entry("w", codes, np.full((rows, 1), 0x2000, np.uint16), k, classes)
    meta = blob[idx["lev"]:idx["lev"] + idx["meta"]]
    words = np.frombuffer(blob[idx["lev"] + idx["meta"]:], "<u4")
    counts = np.frombuffer(meta[3:], "<u4").reshape(16, 3)
    order = []
    for c_ in range(16):
        for col in np.nonzero(classes == c_)[0]:
            order += [(r, col) for r in range(rows)]
    # a single decoder walking the classes' models in order
    top, state = ctypes.c_int64(len(words)), ctypes.c_uint64(0)
    from oracle import oracle as orc
    L = orc.lib()
    w = np.ascontiguousarray(words, np.uint32)
    assert L.or_ans_open(w.ctypes.data, ctypes.addressof(top), ctypes.addressof(state)) == 0
    got = {}
    for c_ in range(16):
        cols_c = np.nonzero(classes == c_)[0]
        if not len(cols_c):
            continue
        cdf = bc.ans_cdf(counts[c_])
        out = np.zeros(rows * len(cols_c), np.uint16)
        L.or_ans_pop(w.ctypes.data, ctypes.addressof(top), ctypes.addressof(state), cdf.ctypes.data, 3,
                     out.ctypes.data, out.size)
        for j, col in enumerate(cols_c):
            for r in range(rows):
                got[(r, col)] = out[j * rows + r]
    assert [got[p] for p in order] == [codes[r, col] for r, col in order]
    assert meta[0] == (2 << 4) | 0 and meta[1] == (2 << 4) | 1 and meta[2] == (0 << 4) | 2


@pytest.mark.parametrize("bits,zs", [(5, None), (6, "xz"), (4, "alone")])
def test_ansint(bark, bits, zs):
    rng = np.random.default_rng(bits)
    vals = rng.normal(0, 0.1, size=(40, 24)).astype(np.float32)
    q, sc, deq = bc.quantize_ansint(vals, bits)
    c = bark.BarkContainer.from_bytes(bc.write_container([bc.ansint_entry("m", q, bits, sc, zs)]))
    got = c.read("m")
    assert got.dtype == np.float32 and got.shape == vals.shape
    assert np.array_equal(got, deq)
    assert c.read_lowbit("m") is None
    # value = (symbol - (2^(bits-1) - 1)) * scale, computed in f32
    bias = (1 << (bits - 1)) - 1
    assert np.array_equal(got, ((q + bias - bias).astype(np.float32) * sc.view(np.float16).astype(np.float32)[:, None]))


def test_raw_entries(bark):
    rng = np.random.default_rng(2)
    h = rng.normal(size=(3, 5)).astype(np.float16)
    i64 = np.array([1, -2, 1 << 40], np.int64)
    i32 = np.arange(6, dtype=np.int32).reshape(2, 3)
    blob = bc.write_container([bc.raw_entry("h", h, "xz"), bc.raw_entry("a", i64), bc.raw_entry("b", i32, "alone")])
    c = bark.BarkContainer.from_bytes(blob)
    assert c.read("h").dtype == np.float16 and np.array_equal(c.read("h"), h)
    assert np.array_equal(c.read("a"), i64) and c.read("a").dtype == np.int64
    assert np.array_equal(c.read("b"), i32) and c.read("b").dtype == np.int32
    assert c.info().weights == h.size  # integer tensors are not weights


def test_offsets_follow_index_order(bark):
    """Payloads sit back to back after the header in index order
    (offset += lev + meta + b + s)."""
    rng = np.random.default_rng(5)
    arrays = [rng.normal(size=i + 1).astype(np.float16) for i in range(6)]
    ents = [bc.raw_entry(f"t{i}", a) for i, a in enumerate(arrays)]
    codes, mags, classes = _levels2_case(rng, 8, 16, 2)
    ents.insert(3, bc.levels2_entry("lv", codes, mags, 2, classes, "xz"))
    c = bark.BarkContainer.from_bytes(bc.write_container(ents))
    for i, a in enumerate(arrays):
        assert np.array_equal(c.read(f"t{i}"), a)
    assert np.array_equal(unpack_codes(c.read_lowbit("lv")), codes)


def test_info_names_layers(bark):
    rng = np.random.default_rng(6)
    ents = []
    for layer in (0, 1, 5):
        codes, mags, classes = _levels2_case(rng, 12, 10, 2)
        ents.append(bc.levels2_entry(f"encoder.layers.{layer}.feed_forward1.linear1.weight", codes, mags, 2, classes))
    ents.append(bc.raw_entry("encoder.layers.x.bias", np.zeros(3, np.float16)))
    ents.append(bc.raw_entry("decoder.embedding.weight", np.zeros((17, 4), np.float16)))
    c = bark.BarkContainer.from_bytes(bc.write_container(ents), "rel")
    info = c.info()
    assert (info.layers, info.hidden, info.ffn, info.vocab) == (3, 10, 12, 17)
    assert info.tensors == 5 == c.tensor_count() and info.release == "rel" and info.layout == "lowbit"
    assert info.weights == 3 * 120 + 3 + 68
    assert c.tensor_names() == sorted(e[0]["n"] for e in ents)
    assert c.layers() == 3


def test_prefetch_parallel_matches_serial(bark):
    rng = np.random.default_rng(7)
    ents, want = [], {}
    for i in range(12):
        codes, mags, classes = _levels2_case(rng, 64, 96, 1 + i % 3)
        ents.append(bc.levels2_entry(f"w{i}", codes, mags, 1 + i % 3, classes))
        want[f"w{i}"] = codes
    blob = bc.write_container(ents)
    par = bark.BarkContainer.from_bytes(blob)
    par.prefetch(threads=6)
    ser = bark.BarkContainer.from_bytes(blob)
    ser.prefetch(threads=1)
    for name, codes in want.items():
        assert np.array_equal(unpack_codes(par.read_lowbit(name)), codes)
        assert np.array_equal(par.read_lowbit(name).codes, ser.read_lowbit(name).codes)


def test_open_dir_and_sniffing(bark, tmp_path):
    rng = np.random.default_rng(8)
    codes, mags, classes = _levels2_case(rng, 4, 8, 2)
    blob = bc.write_container([bc.levels2_entry("w", codes, mags, 2, classes)])
    (tmp_path / "model.bark").write_bytes(blob)
    src = bark.open_weights(tmp_path)
    assert isinstance(src, bark.BarkContainer)
    assert np.array_equal(unpack_codes(src.read_lowbit("w")), codes)
    assert src.info().release == tmp_path.name
    src.close()
    assert bark.looks_like_container(blob)
    # a safetensors file is length-prefixed JSON too
    st_head = json.dumps({"__metadata__": {"format": "pt"},
                          "x": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}}).encode()
    st = struct.pack("<Q", len(st_head)) + st_head + np.array([0x3F80, 0xC000], "<u2").tobytes()
    assert not bark.looks_like_container(st)
    s = bark.open_bytes(st)
    assert isinstance(s, bark.SafetensorsSource) and s.read_dtype("x") == "BF16"
    assert list(s.read("x")) == [0x3F80, 0xC000] and s.read_lowbit("x") is None
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(bark.BarkError, match="neither model.bark nor model.safetensors"):
        bark.open_weights(empty)
    (empty / "model.safetensors").write_bytes(st)
    assert isinstance(bark.open_weights(empty), bark.SafetensorsSource)


# ─────────────────────────────── errors ───────────────────────────────
def _container_with(index_entry, payload, fmt="bark-levels-v2"):
    js = json.dumps({"format": fmt, "index": [index_entry]}).encode()
    return struct.pack("<Q", len(js)) + js + payload


def test_header_errors(bark):
    with pytest.raises(bark.BarkError, match="unsupported container format"):
        bark.BarkContainer.from_bytes(bc.write_container([], fmt="bark-levels-v9"))
    with pytest.raises(bark.BarkError, match="header claims 0 bytes"):
        bark.BarkContainer.from_bytes(struct.pack("<Q", 0) + b"{}")
    with pytest.raises(bark.BarkError, match="header claims"):
        bark.BarkContainer.from_bytes(struct.pack("<Q", 64 << 20) + b"{}")
    with pytest.raises(bark.BarkError, match="header is not JSON"):
        bark.BarkContainer.from_bytes(struct.pack("<Q", 3) + b"{x}")
    with pytest.raises(bark.BarkError, match="unsupported entry kind"):
        bark.BarkContainer.from_bytes(_container_with({"n": "a", "shape": [1], "k": "zstd"}, b""))
    with pytest.raises(bark.BarkError, match="a: ansintx"):
        bark.BarkContainer.from_bytes(_container_with({"n": "a", "shape": [1], "k": "ansintx"}, b""))
    assert not bark.looks_like_container(b"short")


def test_entry_errors(bark):
    rng = np.random.default_rng(9)
    codes, mags, classes = _levels2_case(rng, 4, 8, 2)
    idx, blob = bc.levels2_entry("w", codes, mags, 2, classes)
    ok = bark.BarkContainer.from_bytes(_container_with(idx, blob))
    with pytest.raises(bark.BarkError, match="nope: not in the container"):
        ok.read("nope")

    def bad(change, payload=blob, match=""):
        e = dict(idx)
        e.update(change)
        c = bark.BarkContainer.from_bytes(_container_with(e, payload))
        with pytest.raises(bark.BarkError, match=match):
            c.read_lowbit("w")

    bad({"K": 4}, match="unsupported level count 4")
    bad({"K": 0}, match="unsupported level count 0")
    bad({"lev": idx["lev"] - 2, "meta": idx["meta"] + 2}, match="level table is 14 bytes, expected 16")
    bad({"meta": 2, "b": idx["b"] + idx["meta"] - 2}, match="class table is short")
    bad({"meta": 4 + 16 * 5 * 4 - 4, "b": idx["b"] + 4}, match=r"symbol tables are short \(79 of 80\)")
    # a zero top word
    zero_top = blob + b"\x00\x00\x00\x00"
    bad({"b": idx["b"] + 4}, payload=zero_top, match="truncated ANS stream")
    # an empty table for a class that has columns
    meta_off = idx["lev"]
    m = bytearray(blob)
    c0 = int(classes[0])
    m[meta_off + 4 + c0 * 5 * 4: meta_off + 4 + (c0 + 1) * 5 * 4] = bytes(20)
    bad({}, payload=bytes(m), match=f"empty symbol table for class {c0}")
    # an LZMA field that does not decompress
    bad({"zl": True}, match="lzma")
    # a blob past the end of the buffer
    bad({"b": idx["b"] + 1000}, match="blob outside the buffer")
    # raw size mismatch
    r = bark.BarkContainer.from_bytes(_container_with({"n": "r", "shape": [3], "k": "raw", "b": 4}, b"\x00" * 4))
    with pytest.raises(bark.BarkError, match="4 bytes for 3 values of 2 bytes"):
        r.read("r")
    # ansint with an empty symbol table
    z = bark.BarkContainer.from_bytes(_container_with(
        {"n": "q", "shape": [1, 2], "k": "ansint5", "s": 2, "meta": 8, "b": 0}, b"\x00\x3c" + bytes(8)))
    with pytest.raises(bark.BarkError, match="empty symbol table"):
        z.read("q")


def test_legacy_lzma_with_unknown_size(bark):
    """A .lzma stream with the 'size unknown' header and an end marker
    (lzma_rs::lzma_decompress accepts both header forms)."""
    raw = np.arange(20, dtype=np.float16).tobytes()
    z = lzma.compress(raw, format=lzma.FORMAT_ALONE)
    assert z[5:13] == b"\xff" * 8  # Python writes 'unknown size' + end marker
    c = bark.BarkContainer.from_bytes(_container_with(
        {"n": "r", "shape": [20], "k": "raw", "b": len(z), "zr": 1}, z))
    assert np.array_equal(c.read("r"), np.arange(20, dtype=np.float16))


def test_load_source_host_side(bark, pkg, syn):
    """container_from_weights + load_source bookkeeping without a GPU: every
    float entry is offered with the storage form the reader returned."""
    rng = np.random.default_rng(10)
    w = syn.decoder_weights(seed=1, vocab=33)
    blob, direct = bc.container_from_weights(w, rng, syn.make_levels_k)
    c = bark.BarkContainer.from_bytes(blob)
    assert sorted(direct) == c.tensor_names()
    for name, v in direct.items():
        got = c.read(name)
        if isinstance(v, tuple):
            assert got.dtype == np.float16 and np.array_equal(got.view(np.uint16), v[1])
        else:
            assert got.dtype == np.float32 and np.array_equal(got, v)
