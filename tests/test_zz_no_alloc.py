"""b3_linear_lut4_noalloc: the 4-bit linear for callers that cannot allocate
device memory (latency-critical threads that must not block in cudaMalloc /
cudaFree, hosts that keep every GPU byte in their own pool).  It stages its f16
activations in a fixed scratch array inside the library instead of a
context-owned buffer.

Checked through the C ABI against the allocating entry point b3_linear_lut4 on
the same device buffers, for two calls in a row with different shapes (the
second call must not see anything left over from the first).  This file runs
last so that a failure here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

GEMM_TOL = 2e-3  # same bound as the other K1 tests (max|d| / max|ref|)


def test_noalloc_matches_allocating_entry_point(pkg, syn):
    import torch

    L = pkg.lib()
    enc = pkg.Encoder(0)
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(2024)
    for m, n, k in [(300, 1024, 1024), (1875, 4096, 1024)]:
        a = torch.from_numpy(rng.normal(0, 1, size=(m, k)).astype(np.float32)).cuda()
        codes, lut16 = syn.make_lut4(rng, n, k)
        tc = torch.from_numpy(codes).cuda()
        tl = torch.from_numpy(lut16.view(np.int16)).cuda()
        bias = torch.from_numpy(rng.normal(0, 0.01, size=n).astype(np.float32)).cuda()
        want = torch.empty(m, n, device="cuda")
        got = torch.full((m, n), float("nan"), device="cuda")
        torch.cuda.synchronize()
        enc.linear_lut4(a, tc, tl, bias, out=want)
        enc.sync()
        rc = L.b3_linear_lut4_noalloc(a.data_ptr(), tc.data_ptr(), tl.data_ptr(), bias.data_ptr(),
                                      got.data_ptr(), m, n, k, ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, pkg.last_error()
        stream.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        assert rel_err(g, w) <= GEMM_TOL
    enc.close()


def test_noalloc_rejects_oversize(pkg):
    import torch

    L = pkg.lib()
    m, n, k = 8192, 128, 1024  # m * k above the 4 Mi-value scratch
    a = torch.zeros(1, device="cuda")
    rc = L.b3_linear_lut4_noalloc(a.data_ptr(), a.data_ptr(), a.data_ptr(), None, a.data_ptr(), m, n, k, None)
    assert rc == pkg.B3_EINVAL
    assert "scratch" in pkg.last_error()
