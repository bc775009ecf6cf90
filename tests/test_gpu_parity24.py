"""Full-depth parity: all 24 encoder blocks against the CPU oracle (the
reference's CpuEncoder restated, src/cpu/mod.rs:156-189), block by block, on
BASELINE configs 2 and 3, and the whole audio -> tokens pipeline against the
oracle pipeline (mel, subsampling, encoder, greedy TDT; src/mel.rs,
src/sub.rs, src/cpu/*, src/tdt.rs:416-467) on a config-5-like batch.

Two errors per block, both required <= 2e-2 (the north star's per-layer
tolerance):
  max-normalised   max|gpu - oracle| / max|oracle|;
  frame-centred    the same after subtracting each side's mean frame (the
                   per-channel mean over the utterance's frames).  A random-
                   init encoder carries a large component common to every
                   frame; this error measures the part that differs between
                   frames on its own scale, so a wrong per-frame component
                   cannot hide behind the common one.
Token match: 1 - token edit distance / oracle tokens over the batch, >= 0.99
(the north star), with (id, frame, duration) triples compared as units.
"""
import numpy as np
import pytest

from conftest import centred_err, rel_err
from test_gpu_decoder import token_match

pytestmark = pytest.mark.gpu

LAYER_TOL = 2e-2
MATCH = 0.99
LEAD_IN = np.zeros(4000, np.float32)   # the 0.25 s the pipeline prepends (src/transcription.rs:48-52)


def oracle_sub(oracle, w, wave):
    """Oracle front end: padded wave -> mel (the oracle's own slaney table) ->
    conv subsampling -> (T, 4096)."""
    mel, nv = oracle.mel(np.concatenate([LEAD_IN, wave]), oracle.mel_filters())
    return oracle.subsample(mel, nv, w)


def models(syn, oracle, gpu_encoder_factory, seed, layout, n=24):
    """(GPU encoder of n blocks, GPU encoder of n + 1 blocks, oracle of n
    blocks) over the same first n blocks and projector.  b3_encode returns
    the pre-norm_out residual of block `layers - 1` for layers < the context's
    block count and the pooler otherwise, so block n-1's residual is read
    from the context that holds one block more."""
    w1 = syn.encoder_weights(seed=seed, n_layers=n + 1, layout=layout)
    w = {k: v for k, v in w1.items() if not k.startswith(f"encoder.layers.{n}.")}
    return w, gpu_encoder_factory(w, n), gpu_encoder_factory(w1, n + 1), oracle.OracleEncoder(w, n)


def per_block(enc, enc_deep, ref_enc, sub, n_layers):
    """(max-normalised, frame-centred) error of every block's pre-norm_out
    residual and of the pooler; the oracle runs all blocks in one pass."""
    dump, ref_pool = ref_enc.encode_layers(sub)
    rows = []
    for l in range(n_layers):
        got = enc_deep.encode(sub, layers=l + 1)
        assert got.shape == dump[l].shape and np.isfinite(got).all()
        rows.append((rel_err(got, dump[l]), centred_err(got, dump[l])))
    pool = enc.encode(sub)
    assert pool.shape == ref_pool.shape and np.isfinite(pool).all()
    return rows, (rel_err(pool, ref_pool), centred_err(pool, ref_pool))


def report(tag, rows, pool):
    for l, (e, c) in enumerate(rows):
        print(f"{tag} block {l:2d}: max-normalised {e:.2e}  frame-centred {c:.2e}")
    print(f"{tag} pooler:   max-normalised {pool[0]:.2e}  frame-centred {pool[1]:.2e}")


def test_config2_lut4_24_blocks_from_audio(syn, oracle, gpu_encoder_factory):
    """the 24-block 4-bit encoder on 30 s of seeded audio
    (T = 379), every block's residual and the pooler against the oracle."""
    n = 24
    w, enc, deep, ref = models(syn, oracle, gpu_encoder_factory, 31, "lut4", n)
    sub = oracle_sub(oracle, syn.frontend_weights(seed=31), syn.synth_audio(np.random.default_rng(31), 30.0))
    assert sub.shape[0] == 379
    rows, pool = per_block(enc, deep, ref, sub, n)
    report("config 2 (4-bit, T=379)", rows, pool)
    assert len(rows) == n
    assert max(max(r) for r in rows) <= LAYER_TOL
    assert max(pool) <= LAYER_TOL


def test_config3_bf16_24_blocks_150s(syn, oracle, gpu_encoder_factory):
    """the 24-block encoder in the bf16 Pro layout on 150 s
    of seeded audio (T = 1879), every block's residual and the pooler."""
    n = 24
    w, enc, deep, ref = models(syn, oracle, gpu_encoder_factory, 32, "bf16", n)
    sub = oracle_sub(oracle, syn.frontend_weights(seed=32), syn.synth_audio(np.random.default_rng(32), 150.0))
    assert sub.shape[0] == 1879
    rows, pool = per_block(enc, deep, ref, sub, n)
    report("config 3 (bf16, T=1879)", rows, pool)
    assert max(max(r) for r in rows) <= LAYER_TOL
    assert max(pool) <= LAYER_TOL


def test_pipeline_tokens_match_oracle_pipeline(syn, oracle, pkg):
    """Whole pipeline, both sides from the same 16 kHz audio: GPU
    transcribe_audio (mel, subsampling, 24-block 4-bit encoder, greedy TDT in
    one call) against the oracle's mel -> subsample -> encode -> decode, on 16
    utterances with config 5's length distribution (U(10, 60) s).  Asserts
    >= 99% token match over the batch and prints the oracle's decision
    margins (best - runner-up score per greedy step)."""
    n = 24
    w = syn.encoder_weights(seed=5, n_layers=n, layout="lut4")
    w.update(syn.decoder_weights(seed=5, vocab=1025))
    w.update(syn.frontend_weights(seed=5))
    enc = pkg.Encoder(0)
    try:
        enc.load(w)
        enc.finalize(n)
        rng = np.random.default_rng(55)
        secs = syn.batch_lengths(55, 16)
        waves = [syn.synth_audio(rng, s) for s in secs]
        got = enc.transcribe_audio(waves)
        pooler, roff = enc.encode_audio(waves)
    finally:
        enc.close()
    oenc = oracle.OracleEncoder(w, n)
    odec = oracle.OracleTdt(w)
    want, gaps, perr = [], [], []
    for i, wv in enumerate(waves):
        ref_pool = oenc.encode(oracle_sub(oracle, w, wv))
        g = pooler[roff[i]:roff[i + 1]]
        assert g.shape == ref_pool.shape
        perr.append((rel_err(g, ref_pool), centred_err(g, ref_pool)))
        toks, gp = odec.decode_margins(ref_pool)
        want.append(toks)
        gaps.append(gp)
    gp = np.concatenate(gaps)
    m, exact = token_match(got, want)
    n_tok = sum(len(x) for x in want)
    print(f"16 utterances, {sum(secs):.0f} audio-s, {n_tok} oracle tokens, {len(gp)} greedy steps: "
          f"token match {m:.4f}, identical streams {exact:.2f}")
    print("pooler error per utterance (max-normalised, frame-centred): "
          + " ".join(f"{a:.1e}/{b:.1e}" for a, b in perr))
    q = [0.0, 0.001, 0.01, 0.1, 0.5]
    print("token margin quantiles", dict(zip(q, np.round(np.quantile(gp[:, 0], q), 5))))
    print("duration margin quantiles", dict(zip(q, np.round(np.quantile(gp[:, 1], q), 5))))
    assert max(max(p) for p in perr) <= LAYER_TOL
    assert m >= MATCH
