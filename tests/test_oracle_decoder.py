"""The restated TDT decoder (oracle) against an independent float64
restatement of TdtDecoder::decode (src/tdt.rs:416-467).  CPU only."""
import numpy as np
import pytest


def decode_f64(w, pooler):
    """Greedy TDT in float64 with the reference's f16-rounded matrices."""
    r16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float64)  # noqa: E731
    emb = np.asarray(w["decoder.embedding.weight"], np.float64)
    V = emb.shape[0]
    blank = V - 1
    Wih = [r16(w[f"decoder.lstm.weight_ih_l{l}"]) for l in (0, 1)]
    Whh = [r16(w[f"decoder.lstm.weight_hh_l{l}"]) for l in (0, 1)]
    b = [np.asarray(w[f"decoder.lstm.bias_ih_l{l}"], np.float64) + w[f"decoder.lstm.bias_hh_l{l}"] for l in (0, 1)]
    Wp, bp = r16(w["decoder.decoder_projector.weight"]), np.asarray(w["decoder.decoder_projector.bias"], np.float64)
    Wh, bh = r16(w["joint.head.weight"]), np.asarray(w["joint.head.bias"], np.float64)
    sig = lambda z: 1 / (1 + np.exp(-z))  # noqa: E731
    h = [np.zeros(640), np.zeros(640)]
    c = [np.zeros(640), np.zeros(640)]

    def lstm(x):
        for l in (0, 1):
            xin = x if l == 0 else h[0]
            g = b[l] + Wih[l] @ xin + Whh[l] @ h[l]
            i_, f_, g_, o_ = sig(g[:640]), sig(g[640:1280]), np.tanh(g[1280:1920]), sig(g[1920:])
            c[l] = f_ * c[l] + i_ * g_
            h[l] = o_ * np.tanh(c[l])

    lstm(emb[blank])
    dec = bp + Wp @ h[1]
    T = pooler.shape[0]
    frame, guard, out = 0, 0, []
    while frame < T:
        guard += 1
        if guard > T * 14 + 64:
            break
        s = np.maximum(pooler[frame] + dec, 0)
        sc = bh + Wh @ s
        tok = int(np.argmax(sc[:V]))
        dur = int(np.argmax(sc[V:]))
        if tok == blank:
            frame += max(dur, 1)
        else:
            out.append((tok, frame, dur))
            lstm(emb[tok])
            dec = bp + Wp @ h[1]
            frame += dur
    return np.array(out, dtype=np.uint32).reshape(-1, 3)


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_decoder_matches_float64(oracle, syn, seed):
    w = syn.decoder_weights(seed=seed, vocab=65)
    dec = oracle.OracleTdt(w)
    rng = np.random.default_rng(seed)
    pooler = rng.normal(0, 1, size=(40, 640)).astype(np.float32)
    got = dec.decode(pooler)
    want = decode_f64(w, pooler.astype(np.float64))
    assert got.shape[0] > 0
    assert np.array_equal(got, want)


def test_decoder_stream_invariants(oracle, syn):
    w = syn.decoder_weights(seed=3, vocab=1025)
    dec = oracle.OracleTdt(w)
    pooler = np.random.default_rng(3).normal(0, 1, size=(120, 640)).astype(np.float32)
    toks = dec.decode(pooler)
    assert len(toks) > 0
    assert np.all(toks[:, 0] < 1024)          # blank is never emitted
    assert np.all(np.diff(toks[:, 1].astype(np.int64)) >= 0)
    assert np.all(toks[:, 1] < 120)
    assert np.all(toks[:, 2] <= 4)
    batch = dec.decode_batch(np.concatenate([pooler, pooler[:50]]), [0, 120, 170])
    assert np.array_equal(batch[0], toks)
    assert np.array_equal(batch[1], dec.decode(pooler[:50]))
