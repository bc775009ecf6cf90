"""Generates tests/golden/oracle_golden.npz: small seeded outputs of the CPU
oracle (GEMM, LayerNorm, rel-softmax rows, depthwise conv, position table and
a one-block encoder), used by tests/test_oracle.py as a regression guard.

    python tests/golden/make_golden.py
"""
import pathlib
import sys

import numpy as np


def compute(oracle, syn):
    rng = np.random.default_rng(1234)
    out = {}
    a = rng.normal(size=(13, 40)).astype(np.float32)
    w = oracle.round_f16(rng.normal(0, 0.1, size=(33, 40)).astype(np.float32))
    out["gemm_13x33x40"] = oracle.gemm(a, w)
    x = rng.normal(0, 2, size=(5, 1024)).astype(np.float32)
    out["layer_norm"] = oracle.layer_norm(x, rng.normal(1, 0.1, 1024).astype(np.float32),
                                          rng.normal(0, 0.1, 1024).astype(np.float32))
    g = rng.normal(size=(21, 1024)).astype(np.float32)
    out["dwconv"] = oracle.dwconv_bn_silu(g, rng.normal(0, 0.2, size=(1024, 9)).astype(np.float32),
                                          np.ones(1024, np.float32), np.zeros(1024, np.float32))
    out["pos_embed_t9"] = oracle.pos_embed(9)
    weights = syn.encoder_weights(seed=21, n_layers=1, layout="lut4")
    enc = oracle.OracleEncoder(weights, 1)
    sub = syn.sub_features(np.random.default_rng(22), 20)
    out["encoder_1block_t20"] = enc.encode(sub)
    return out


def main():
    root = pathlib.Path(__file__).resolve().parents[2]
    sys.path.insert(0, str(root))
    from __graft_entry__ import load_oracle, load_package

    load_package()
    import bark3_b200.synthetic as syn

    oracle = load_oracle()
    oracle.set_threads(4)
    np.savez_compressed(pathlib.Path(__file__).with_name("oracle_golden.npz"), **compute(oracle, syn))


if __name__ == "__main__":
    main()
