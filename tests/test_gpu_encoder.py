"""Encoder parity on the GPU against the CPU oracle (the reference's CpuEncoder
restated), through the C ABI.

Tolerance (north star): max relative error <= 2e-2 per layer, measured as
max|gpu - oracle| / max|oracle| on the pre-norm residual after each block and
on the pooler.  The GPU rounds activations to f16 at GEMM inputs and
accumulates in f32 on tensor cores; the reference keeps f32 activations with
the same f16 weights.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

LAYER_TOL = 2e-2


@pytest.fixture(scope="module")
def lut_model(syn, oracle, gpu_encoder_factory):
    n_layers = 3
    w = syn.encoder_weights(seed=1, n_layers=n_layers, layout="lut4")
    return w, gpu_encoder_factory(w, n_layers), oracle.OracleEncoder(w, n_layers), n_layers


@pytest.mark.parametrize("t", [1, 7, 64, 130, 379])
def test_per_layer_parity_lut4(lut_model, syn, t):
    w, enc, ref, n_layers = lut_model
    sub = syn.sub_features(np.random.default_rng(t), t)
    errs = []
    for layers in range(1, n_layers + 1):
        got = enc.encode(sub, layers=layers)
        want = ref.encode(sub, layers=layers)
        assert got.shape == want.shape
        assert np.isfinite(got).all()
        errs.append(rel_err(got, want))
    print(f"T={t} per-layer errors {['%.2e' % e for e in errs]}")
    assert max(errs) <= LAYER_TOL


def test_bf16_layout_parity(syn, oracle, gpu_encoder_factory):
    n_layers = 2
    w = syn.encoder_weights(seed=2, n_layers=n_layers, layout="bf16")
    enc = gpu_encoder_factory(w, n_layers)
    ref = oracle.OracleEncoder(w, n_layers)
    sub = syn.sub_features(np.random.default_rng(3), 257)
    for layers in (1, 2):
        e = rel_err(enc.encode(sub, layers=layers), ref.encode(sub, layers=layers))
        print(f"bf16 layers={layers} err {e:.2e}")
        assert e <= LAYER_TOL


def test_bf16_layout_long_utterance(syn, oracle, gpu_encoder_factory):
    """BASELINE config 2's length: 150 s of audio (T = 1875 encoder frames) in
    the bf16 Pro layout, 15 query blocks per head and the f16-weight K1 path at
    M = 1875."""
    n_layers = 2
    w = syn.encoder_weights(seed=2, n_layers=n_layers, layout="bf16")
    enc = gpu_encoder_factory(w, n_layers)
    ref = oracle.OracleEncoder(w, n_layers)
    sub = syn.sub_features(np.random.default_rng(5), 1875)
    for layers in (1, 2):
        e = rel_err(enc.encode(sub, layers=layers), ref.encode(sub, layers=layers))
        print(f"bf16 T=1875 layers={layers} err {e:.2e}")
        assert e <= LAYER_TOL


def test_long_and_short_utterances_batch_exactly(lut_model, syn):
    """A varlen batch mixing a ten-minute utterance with tiny ones equals the
    utterances encoded one by one, bit for bit (the persistent attention walks
    items of every utterance in one launch)."""
    w, enc, ref, n_layers = lut_model
    rng = np.random.default_rng(19)
    lens = [3, 7500, 1, 640, 129]
    subs = [syn.sub_features(rng, t) for t in lens]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    got = enc.encode_batch(np.concatenate(subs), cu)
    assert np.isfinite(got).all()
    for i, s in enumerate(subs):
        assert np.array_equal(got[cu[i]:cu[i + 1]], enc.encode(s)), f"utterance {i} (T={lens[i]})"


def test_repeated_encode_replays_identically(lut_model, syn):
    """A small batch encoded again with the same buffers is replayed from a
    CUDA graph (the first call runs eagerly, the second captures, later calls
    replay): every call gives the eager result bit for bit, on the device-
    pointer and the host-pointer paths."""
    import torch

    w, enc, ref, n_layers = lut_model
    rng = np.random.default_rng(29)
    lens = [120, 57]
    host = np.concatenate([syn.sub_features(rng, t) for t in lens])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    dev = torch.from_numpy(host).cuda()
    out = torch.empty(int(cu[-1]), 640, device="cuda")
    runs = []
    for _ in range(4):
        enc.encode_batch(dev, cu, out=out)
        enc.sync()
        runs.append(out.cpu().numpy().copy())
    host_runs = [enc.encode_batch(host, cu) for _ in range(4)]
    for r in runs[1:] + host_runs:
        assert np.array_equal(r, runs[0])
    # another shape in between (a new plan) invalidates the replay; coming
    # back to the first shape rebuilds it and still gives the same rows
    other = syn.sub_features(rng, 33)
    one = [enc.encode(other) for _ in range(3)]
    assert all(np.array_equal(x, one[0]) for x in one)
    for _ in range(3):
        assert np.array_equal(enc.encode_batch(host, cu), runs[0])


def test_batch_equals_single(lut_model, syn):
    """Varlen batching is exact: every kernel is row- or segment-local."""
    w, enc, ref, n_layers = lut_model
    rng = np.random.default_rng(9)
    lens = [37, 130, 1, 64, 200]
    subs = [syn.sub_features(rng, t) for t in lens]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    got = enc.encode_batch(np.concatenate(subs), cu)
    for i, s in enumerate(subs):
        one = enc.encode(s)
        assert np.array_equal(got[cu[i]:cu[i + 1]], one), f"utterance {i}"


def test_levels_format(syn, oracle, pkg, gpu_encoder_factory):
    """The .bark levels2 form (k <= 3 sign-magnitude levels, u32 code words)
    converts to the same values as `expand` (src/bark.rs:597-611)."""
    n_layers = 1
    rng = np.random.default_rng(4)
    w = syn.encoder_weights(seed=4, n_layers=n_layers, layout="lut4")
    dense = dict(w)
    for name in list(w):
        if isinstance(w[name], tuple) and w[name][0] == "lut4":
            rows, cols = w[name][2].shape[0], w[name][1].shape[1] * 2
            k = int(rng.integers(1, 4))
            words, levels, codes = syn.make_levels_k(rng, rows, cols, k)
            w[name] = ("levels", words, levels, k, cols)
            dense[name] = syn.expand_levels(codes, levels, k)
    enc = gpu_encoder_factory(w, n_layers)
    ref = oracle.OracleEncoder(dense, n_layers)
    sub = syn.sub_features(rng, 90)
    e = rel_err(enc.encode(sub), ref.encode(sub))
    print(f"levels-format err {e:.2e}")
    assert e <= LAYER_TOL


def test_attn_conv_section(lut_model, syn):
    """BASELINE config 4 shape family: attention + conv sections alone."""
    w, enc, ref, n_layers = lut_model
    x = np.random.default_rng(12).normal(0, 1, size=(300, 1024)).astype(np.float32)
    got = x.copy()
    enc.attn_conv(1, got)
    want = ref.attn_conv(1, x)
    e = rel_err(got - x, want - x)
    print(f"attn+conv delta err {e:.2e}")
    assert e <= LAYER_TOL


@pytest.mark.parametrize("t", [2001, 7500])
def test_attn_conv_long_sequence(lut_model, t):
    """BASELINE config 3's sequence length (T = 7500, ten minutes of audio):
    59 query blocks x 118 key blocks per head, the 256-row R ring wrapping many
    times, a ragged last block; the same section through the CPU oracle."""
    w, enc, ref, n_layers = lut_model
    x = np.random.default_rng(t).normal(0, 1, size=(t, 1024)).astype(np.float32)
    got = x.copy()
    enc.attn_conv(1, got)
    want = ref.attn_conv(1, x)
    assert np.isfinite(got).all()
    e = rel_err(got - x, want - x)
    mean = float(np.mean(np.abs((got - x) - (want - x))) / np.mean(np.abs(want - x)))
    print(f"T={t} attn+conv delta err max {e:.2e} mean {mean:.2e}")
    assert e <= LAYER_TOL


def test_errors(pkg, syn):
    enc = pkg.Encoder(0)
    sub = np.zeros((4, 4096), dtype=np.float32)
    with pytest.raises(pkg.B3Error) as ei:
        enc.encode(sub, layers=1)
    assert ei.value.code == pkg.B3_ESTATE
    w = syn.encoder_weights(seed=0, n_layers=1, layout="lut4")
    del w["encoder.layers.0.norm_conv.bias"]
    enc.load(w)
    with pytest.raises(pkg.B3Error) as ei:
        enc.finalize(1)
    assert ei.value.code == pkg.B3_ENOTFOUND
    assert "norm_conv.bias" in str(ei.value)
    enc.close()
