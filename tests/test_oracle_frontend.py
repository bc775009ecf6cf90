"""Front-end oracle (mel, conv subsampling) and the library's filterbank
against the reference's own filterbank file and independent implementations.
CPU only."""
import pathlib

import numpy as np
import pytest

# The filterbank the reference bundles and hands to MelFrontend::new
# (src/mel.rs:10-40): raw little-endian f32, 128 x 257.  Present where the
# reference tree is (this container); absent on GPU boxes.
REF_FILTERS = pathlib.Path("/root/reference/data/mel_filters.f32")


def reference_filters():
    if not REF_FILTERS.exists():
        pytest.skip("the reference tree (data/mel_filters.f32) is not present on this machine")
    fb = np.fromfile(REF_FILTERS, dtype="<f4")
    assert fb.size == 128 * 257
    return fb.reshape(128, 257)


def test_oracle_filterbank_equals_reference_file(oracle):
    """The oracle's numpy slaney restatement against the reference's own
    data/mel_filters.f32 (measured: max difference 3.7e-9, 99.5% of the
    32,896 entries bit-identical)."""
    ours = oracle.mel_filters()
    ref = reference_filters()
    assert ours.shape == ref.shape
    assert np.max(np.abs(ours.astype(np.float64) - ref)) <= 1e-8


def test_library_filterbank_equals_reference_file(pkg):
    """b3_mel_filters (the table the GPU front end uses) against the
    reference's data/mel_filters.f32."""
    ours = pkg.mel_filters()
    ref = reference_filters()
    assert np.max(np.abs(ours.astype(np.float64) - ref)) <= 1e-8


def test_library_filterbank_equals_oracle(pkg, oracle):
    """Runs everywhere (the reference file is not needed): the library's
    table and the oracle's restatement agree to 1e-8."""
    assert np.max(np.abs(pkg.mel_filters().astype(np.float64) - oracle.mel_filters())) <= 1e-8


def test_oracle_mel_same_with_either_table(oracle, syn):
    """The oracle's mel features with its own table equal those computed with
    the reference file's table to 1e-6 (normalised units), so tests and the
    CPU baseline that use the oracle's table see the reference's front end."""
    ref = reference_filters()
    rng = np.random.default_rng(4)
    wave = np.concatenate([np.zeros(4000, np.float32), syn.synth_audio(rng, 5.0)])
    a, na = oracle.mel(wave, oracle.mel_filters())
    b, nb = oracle.mel(wave, ref)
    assert na == nb
    assert np.max(np.abs(a - b)) <= 1e-6


def transformers_filters():
    from transformers.audio_utils import mel_filter_bank

    fb = mel_filter_bank(num_frequency_bins=257, num_mel_filters=128, min_frequency=0.0, max_frequency=8000.0,
                         sampling_rate=16000, norm="slaney", mel_scale="slaney")
    return fb.T.astype(np.float32)


def test_library_filterbank_is_slaney(pkg):
    """b3_mel_filters against transformers' slaney mel_filter_bank (which the
    reference's data/mel_filters.f32 equals to within 4e-9)."""
    ours = pkg.mel_filters()
    ref = transformers_filters()
    assert np.max(np.abs(ours - ref)) < 1e-7


def mel_numpy(wave, fb):
    """Independent float64 restatement of src/mel.rs:41-138 with numpy's rfft."""
    w = wave.astype(np.float64)
    pre = np.concatenate([w[:1], w[1:] - 0.97 * w[:-1]])
    n_frames = 1 + len(pre) // 160
    n_valid = len(pre) // 160
    win = np.zeros(512)
    i = np.arange(400)
    win[56:456] = 0.5 * (1 - np.cos(2 * np.pi * i / 399))
    padded = np.concatenate([np.zeros(256), pre, np.zeros(512)])
    frames = np.stack([padded[t * 160 : t * 160 + 512] * win for t in range(n_frames)])
    power = np.abs(np.fft.rfft(frames, axis=1)) ** 2
    mel = np.log(power @ fb.astype(np.float64).T + 2.0**-24)
    v = mel[:n_valid]
    mean = v.mean(0)
    std = v.std(0, ddof=1)
    out = (mel - mean) / (std + 1e-5)
    out[n_valid:] = 0
    return out


def test_oracle_mel_matches_numpy(oracle, syn):
    rng = np.random.default_rng(0)
    wave = np.concatenate([np.zeros(4000, np.float32), syn.synth_audio(rng, 3.3)])
    fb = transformers_filters()
    got, nv = oracle.mel(wave, fb)
    want = mel_numpy(wave, fb)
    assert nv == len(wave) // 160
    assert got.shape == want.shape
    assert np.max(np.abs(got - want)) < 2e-3


def subsample_torch(mel, n_valid, w):
    import torch
    import torch.nn.functional as F

    t = lambda n: torch.from_numpy(np.asarray(w["encoder.subsampling.layers." + n], np.float64))  # noqa: E731
    clen = lambda v: (v - 1) // 2 + 1  # noqa: E731
    x = torch.from_numpy(mel.astype(np.float64))[None, None]
    x = F.relu(F.conv2d(x, t("0.weight"), t("0.bias"), stride=2, padding=1))
    v = clen(max(n_valid, 1))
    x[:, :, v:] = 0
    x = F.conv2d(x, t("2.weight"), t("2.bias"), stride=2, padding=1, groups=256)
    v = clen(v)
    x[:, :, v:] = 0
    x = F.relu(F.conv2d(x, t("3.weight"), t("3.bias")))
    x = F.conv2d(x, t("5.weight"), t("5.bias"), stride=2, padding=1, groups=256)
    v = clen(v)
    x[:, :, v:] = 0
    x = F.relu(F.conv2d(x, t("6.weight"), t("6.bias")))
    return x[0].permute(1, 0, 2).reshape(x.shape[2], -1).numpy()


@pytest.mark.parametrize("frames,n_valid", [(1, 0), (9, 8), (120, 119), (301, 250)])
def test_oracle_subsample_matches_torch(oracle, syn, frames, n_valid):
    w = syn.frontend_weights(seed=frames)
    mel = np.random.default_rng(frames).normal(size=(frames, 128)).astype(np.float32)
    mel[n_valid:] = 0
    got = oracle.subsample(mel, n_valid, w)
    want = subsample_torch(mel, n_valid, w)
    assert got.shape == want.shape
    assert np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-6) < 1e-5
