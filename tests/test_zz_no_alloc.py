"""b3_linear_lut4_noalloc: the 4-bit linear for callers that cannot allocate
device memory (latency-critical threads that must not block in cudaMalloc /
cudaFree, hosts that keep every GPU byte in their own pool).  It stages its f16
activations in a fixed scratch array inside the library instead of a
context-owned buffer.

Checked through the C ABI against the allocating entry point b3_linear_lut4 on
the same device buffers, for two calls in a row: first the largest shape the
scratch holds, then a small one, so the second call runs over scratch that
still holds the first call's larger contents and must not read any of it.
Both entry points run the same conversion and GEMM kernels on the same
inputs, so their outputs must be identical bit for bit.  A further call at the
largest shape must leave the device's free memory unchanged.  This file runs
last so that a failure here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_M, MAX_K = 4096, 1024   # m * k = 4 Mi values: the scratch's whole capacity


def _call(L, a, tc, tl, bias, out, m, n, k, stream):
    return L.b3_linear_lut4_noalloc(a.data_ptr(), tc.data_ptr(), tl.data_ptr(), bias.data_ptr(), out.data_ptr(),
                                    m, n, k, ctypes.c_void_p(stream.cuda_stream))


def test_noalloc_matches_allocating_entry_point(pkg, syn):
    import torch

    L = pkg.lib()
    enc = pkg.Encoder(0)
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(2024)
    try:
        for m, n, k in [(MAX_M, 4096, MAX_K), (300, 1024, 1024)]:
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
            rc = _call(L, a, tc, tl, bias, got, m, n, k, stream)
            assert rc == 0, pkg.last_error()
            stream.synchronize()
            g, w = got.cpu().numpy(), want.cpu().numpy()
            assert np.isfinite(g).all()
            assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), f"m={m} n={n} k={k}: outputs differ"
    finally:
        enc.close()


def test_noalloc_allocates_nothing(pkg, syn):
    """After a first call (which looks up the scratch's device address and
    loads the kernels), a call at the largest shape leaves cudaMemGetInfo's
    free-memory figure exactly where it was."""
    import torch

    L = pkg.lib()
    stream = torch.cuda.current_stream()
    rng = np.random.default_rng(7)
    m, n, k = MAX_M, 4096, MAX_K
    a = torch.from_numpy(rng.normal(0, 1, size=(m, k)).astype(np.float32)).cuda()
    codes, lut16 = syn.make_lut4(rng, n, k)
    tc = torch.from_numpy(codes).cuda()
    tl = torch.from_numpy(lut16.view(np.int16)).cuda()
    bias = torch.zeros(n, device="cuda")
    out = torch.empty(m, n, device="cuda")
    assert _call(L, a, tc, tl, bias, out, m, n, k, stream) == 0, pkg.last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    assert _call(L, a, tc, tl, bias, out, m, n, k, stream) == 0, pkg.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_rejects_oversize(pkg):
    import torch

    L = pkg.lib()
    m, n, k = MAX_M + 1, 128, MAX_K  # m * k one row above the 4 Mi-value scratch
    a = torch.zeros(1, device="cuda")
    rc = L.b3_linear_lut4_noalloc(a.data_ptr(), a.data_ptr(), a.data_ptr(), None, a.data_ptr(), m, n, k, None)
    assert rc == pkg.B3_EINVAL
    assert "scratch" in pkg.last_error()
