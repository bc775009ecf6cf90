"""K1 (4-bit LUT / f16 tcgen05 GEMM) against the CPU oracle, through the C ABI.

The oracle is the reference's own CPU GEMM restated (f16 weights, f32
activations, one FMA chain per output).  The GPU computes with f16 activations
and f32 accumulation on tensor cores, so results agree to f16 input rounding;
the bound below is max|gpu - oracle| / max|oracle|.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

GEMM_TOL = 2e-3  # normwise; f16 rounding of A is ~5e-4 relative per element


@pytest.fixture(scope="module")
def enc(pkg):
    e = pkg.Encoder(0)
    yield e
    e.close()


@pytest.mark.parametrize("m", [1, 63, 128, 191, 1875])
def test_lut4_linear_matches_oracle(enc, oracle, syn, m):
    """BASELINE config 1 (M=1875, K=1024, N=4096) plus ragged M."""
    rng = np.random.default_rng(100 + m)
    k, n = 1024, 4096
    a = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    codes, lut16 = syn.make_lut4(rng, n, k)
    bias = rng.normal(0, 0.01, size=n).astype(np.float32)
    got = enc.linear_lut4(a, codes, lut16, bias)
    w = syn.expand_lut4(codes, lut16)
    ref = oracle.gemm(a, w) + bias
    assert got.shape == (m, n)
    assert np.isfinite(got).all()
    assert rel_err(got, ref) < GEMM_TOL


@pytest.mark.parametrize("n,k", [(128, 64), (640, 1024), (1024, 4096), (3072, 1024)])
def test_lut4_linear_shapes(enc, oracle, syn, n, k):
    rng = np.random.default_rng(n + k)
    m = 77
    a = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    codes, lut16 = syn.make_lut4(rng, n, k)
    got = enc.linear_lut4(a, codes, lut16)
    ref = oracle.gemm(a, syn.expand_lut4(codes, lut16))
    assert rel_err(got, ref) < GEMM_TOL


def test_lowbit_equals_f16_bit_exact(enc, syn):
    """The reference's lbtest (src/diagnostics/gemm.rs:538-652): m=64, n=128,
    k=1024, two levels per row [0.02 (row%7+1), 0.05 (row%5+1)], codes
    (i*13 + i/k) % 5, A ((i%89) - 44) * 0.002.  The low-bit kernel must equal
    the f16 kernel on the expanded weights bit for bit."""
    m, n, k = 64, 128, 1024
    i = np.arange(m * k)
    a = (((i % 89).astype(np.float32) - 44.0) * np.float32(0.002)).reshape(m, k).astype(np.float32)
    j = np.arange(n * k)
    codes = ((j * 13 + j // k) % 5).astype(np.uint8).reshape(n, k)
    rows = np.arange(n)
    l0 = (np.float32(0.02) * (rows % 7 + 1).astype(np.float32)).astype(np.float16)
    l1 = (np.float32(0.05) * (rows % 5 + 1).astype(np.float32)).astype(np.float16)
    lut = np.zeros((n, 16), dtype=np.float16)
    lut[:, 1], lut[:, 2], lut[:, 3], lut[:, 4] = l0, l1, -l0, -l1
    lut16 = lut.view(np.uint16)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    w16 = syn.expand_lut4(packed, lut16).astype(np.float16).view(np.uint16)
    c_lb = enc.linear_lut4(a, packed, lut16)
    c_16 = enc.linear_f16(a, w16)
    assert np.array_equal(c_lb.view(np.uint32), c_16.view(np.uint32))
    # and against the f32 naive product the diagnostic prints
    wf = syn.expand_lut4(packed, lut16).astype(np.float64)
    ref = a.astype(np.float64) @ wf.T
    assert np.max(np.abs(c_lb - ref)) < 1e-3


def test_all_sixteen_codes(enc, oracle, syn):
    """Every code 0..15 reaches its own table entry (guards the PRMT lookup)."""
    rng = np.random.default_rng(5)
    m, n, k = 128, 128, 64
    codes = np.tile(np.arange(16, dtype=np.uint8), (n, k // 16))
    for r in range(n):
        codes[r] = np.roll(codes[r], r)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    lut16 = (rng.normal(0, 1, size=(n, 16)).astype(np.float16)).view(np.uint16)
    a = np.eye(m, k, dtype=np.float32)  # picks single columns
    got = enc.linear_lut4(a, packed, lut16)
    want = syn.expand_lut4(packed, lut16)[:, :m].T  # (m, n) with m <= k
    assert np.array_equal(got[:k], want[:k])


def test_device_pointer_path(enc, oracle, syn):
    import torch

    rng = np.random.default_rng(11)
    m, n, k = 300, 1024, 1024
    a = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    codes, lut16 = syn.make_lut4(rng, n, k)
    ta = torch.from_numpy(a).cuda()
    tc = torch.from_numpy(codes).cuda()
    tl = torch.from_numpy(lut16.view(np.int16)).cuda()
    torch.cuda.synchronize()
    out = enc.linear_lut4(ta, tc, tl)
    enc.sync()
    ref = oracle.gemm(a, syn.expand_lut4(codes, lut16))
    assert rel_err(out.cpu().numpy(), ref) < GEMM_TOL


def test_bad_shapes_rejected(enc, pkg, syn):
    rng = np.random.default_rng(1)
    a = np.zeros((4, 100), dtype=np.float32)
    codes, lut16 = syn.make_lut4(rng, 128, 100)
    with pytest.raises(pkg.B3Error) as ei:
        enc.linear_lut4(a, codes, lut16)
    assert ei.value.code == pkg.B3_EINVAL


@pytest.mark.parametrize("lut", [True, False])
def test_pair_tiles_equal_single_cta_tiles(enc, syn, lut):
    """Problems that fill every SM pair run on 256 x 256 CTA-pair tiles
    (tcgen05 cta_group::2); small ones on single-CTA tiles.  Both issue the
    same K-ordered MMAs per output element, so a row slice computed alone
    (single-CTA tiles) must equal the same rows of the large problem."""
    rng = np.random.default_rng(7 if lut else 8)
    m, n, k = 2304, 4096, 1024
    a = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    codes, lut16 = syn.make_lut4(rng, n, k)
    bias = rng.normal(0, 0.01, size=n).astype(np.float32)
    if lut:
        run = lambda x: enc.linear_lut4(x, codes, lut16, bias)
    else:
        w16 = syn.expand_lut4(codes, lut16).astype(np.float16).view(np.uint16)
        run = lambda x: enc.linear_f16(x, w16, bias)
    big = run(a)
    for r0, r1 in [(0, 100), (1000, 1077), (2200, 2304)]:
        part = run(np.ascontiguousarray(a[r0:r1]))
        assert np.array_equal(part.view(np.uint32), big[r0:r1].view(np.uint32)), (r0, r1)


def test_pair_tiles_lowbit_equals_f16(enc, syn):
    """lbtest's bit-exact criterion at a size that runs on CTA-pair tiles."""
    rng = np.random.default_rng(11)
    m, n, k = 2048, 4096, 1024
    a = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    codes, lut16 = syn.make_lut4(rng, n, k)
    w16 = syn.expand_lut4(codes, lut16).astype(np.float16).view(np.uint16)
    assert np.array_equal(enc.linear_lut4(a, codes, lut16).view(np.uint32), enc.linear_f16(a, w16).view(np.uint32))
