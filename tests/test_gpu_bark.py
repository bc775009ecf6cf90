"""A checkpoint loaded from a `model.bark` container runs the same encoder and
decoder as the same values loaded tensor by tensor: the container path
(open_weights -> prefetch -> Encoder.load_source, the reference's
weights::open + Encoder::load_with, src/weights.rs:86-100,
src/encoder.rs:412) must give bit-identical poolers and identical tokens."""
import time

import numpy as np
import pytest

from oracle import bark_container as bc

pytestmark = pytest.mark.gpu


def test_container_model_equals_direct_load(pkg, syn, tmp_path):
    import importlib

    bark = importlib.import_module("bark3_b200.bark")
    n_layers = 2
    rng = np.random.default_rng(21)
    w = syn.encoder_weights(seed=21, n_layers=n_layers, layout="lut4")
    w.update(syn.decoder_weights(seed=21, vocab=1025))
    t0 = time.perf_counter()
    blob, direct = bc.container_from_weights(w, rng, syn.make_levels_k)
    (tmp_path / "model.bark").write_bytes(blob)
    t1 = time.perf_counter()

    src = bark.open_weights(tmp_path)
    assert isinstance(src, bark.BarkContainer) and src.layers() == n_layers
    a = pkg.Encoder(0)
    layers = a.load_source(src)
    t2 = time.perf_counter()
    a.finalize(layers)
    b = pkg.Encoder(0)
    b.load(direct)
    b.finalize(n_layers)
    print(f"container {len(blob) / 1e6:.1f} MB written in {t1 - t0:.2f} s; opened, decoded and staged in "
          f"{t2 - t1:.2f} s")

    lens = [40, 117, 9]
    subs = [syn.sub_features(rng, t) for t in lens]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    sub = np.concatenate(subs)
    pa, pb = a.encode_batch(sub, cu), b.encode_batch(sub, cu)
    assert np.isfinite(pa).all()
    assert np.array_equal(pa, pb)
    ta, tb = a.transcribe_batch(sub, cu), b.transcribe_batch(sub, cu)
    assert all(np.array_equal(x, y) for x, y in zip(ta, tb))
    a.close()
    b.close()
    src.close()
