"""The C ABI without a GPU: the library loads, exports every function the
header declares, and reports argument / state errors as codes + messages
instead of aborting.  CPU only (no kernel is launched)."""
import ctypes
import pathlib
import re

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_library_exports_every_declared_symbol(pkg):
    L = pkg.lib()
    declared = pkg.header_symbols()
    assert len(declared) >= 15
    for name in declared:
        assert hasattr(L, name), f"{name} is declared in include/bark3_b200.h but not exported"


def test_header_symbols_all_bound(pkg):
    """Every declared function has a ctypes signature in the Python view."""
    src = (pathlib.Path(pkg.__file__)).read_text()
    for name in pkg.header_symbols():
        assert f'"{name}"' in src, name


def test_version_and_last_error(pkg):
    L = pkg.lib()
    assert L.b3_version() >= 100
    assert isinstance(pkg.last_error(), str)


def test_null_context_is_an_error(pkg):
    L = pkg.lib()
    assert L.b3_sync(None) == pkg.B3_EINVAL
    assert L.b3_finalize(None, 24) == pkg.B3_EINVAL
    assert L.b3_profile(None, 1) == pkg.B3_EINVAL
    one = (ctypes.c_int64 * 1)(4)
    data = np.zeros(4, np.float32)
    assert L.b3_load_tensor(None, b"x", 0, one, 1, data.ctypes.data) == pkg.B3_EINVAL
    assert "bad arguments" in pkg.last_error()
    assert L.b3_encode(None, data.ctypes.data, 1, 1, data.ctypes.data, 0) == pkg.B3_EINVAL
    assert L.b3_stream(None) is None


def test_noalloc_argument_checks_run_before_any_device_call(pkg):
    L = pkg.lib()
    buf = np.zeros(16, np.float32)
    p = buf.ctypes.data
    assert L.b3_linear_lut4_noalloc(None, p, p, None, p, 4, 128, 64, None) == pkg.B3_EINVAL
    assert L.b3_linear_lut4_noalloc(p, p, p, None, p, 4, 100, 64, None) == pkg.B3_EINVAL
    assert L.b3_linear_lut4_noalloc(p, p, p, None, p, 4096 + 1, 128, 1024, None) == pkg.B3_EINVAL
    assert "scratch" in pkg.last_error()


def test_create_without_gpu_fails_cleanly(pkg):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(pkg.B3Error) as ei:
        pkg.Encoder(0)
    assert ei.value.code == pkg.B3_ECUDA


def test_product_never_imports_the_oracle():
    """The product package must not route through the CPU oracle."""
    pkg_dir = ROOT / "bark3-wgpu_b200"
    pat = re.compile(r"(import\s+oracle|from\s+oracle|load_oracle|bark3_oracle|\bor_[a-z0-9_]+\()")
    for f in list(pkg_dir.rglob("*.py")) + list(pkg_dir.rglob("*.cu")) + list(pkg_dir.rglob("*.h")):
        assert not pat.search(f.read_text()), f


def test_shard_lpt_balances_and_covers(pkg, syn):
    secs = syn.batch_lengths(5, 256)
    frames = [pkg.frames_for_seconds(s) for s in secs]
    for n in (1, 2, 4, 8):
        rank_of = pkg.shard_lpt(frames, n)
        assert rank_of.min() >= 0 and rank_of.max() < n
        cost = np.array([52.4e6 * t + 6144.0 * t * t for t in frames])
        loads = np.bincount(rank_of, weights=cost, minlength=n)
        assert loads.max() / loads.mean() < 1.02
    with pytest.raises(pkg.B3Error):
        pkg.shard_lpt([10, 0, 5], 2)


def test_frames_for_seconds_matches_reference_arithmetic(pkg):
    # 30 s -> 484000 samples with the 0.25 s pad -> 3025 valid mel frames ->
    # 1513 -> 757 -> 379 (the T quoted for BASELINE config 2)
    assert pkg.frames_for_seconds(30.0) == 379
    assert pkg.frames_for_seconds(150.0) == 1879
    assert pkg.frames_for_seconds(600.0) == 7504
