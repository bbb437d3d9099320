"""The GPU log-mel frontend (Frontend, crates/voxrt/src/frontend.rs:36-200) against the numpy restatement in
oracle/. The filterbank and window are host-side and checked on CPU; the FFT is this library's own radix-2
transform, so the spectra are compared with a tolerance: mel powers within 1e-5 of the frame's largest mel power,
log-mel within 1e-3 absolute on bands holding at least 1e-3 of that power, normalised features within 1e-3 there."""
import numpy as np
import pytest


def test_filterbank_matches_restatement(oracle_lib):
    from voxrt_b200.frontend import filterbank

    fb = filterbank()
    want = oracle_lib.mel_filterbank()
    assert fb.shape == (128, 257)
    np.testing.assert_allclose(fb, want, rtol=1e-6, atol=1e-9)
    assert np.array_equal(fb > 0, want > 0)


@pytest.mark.gpu
def test_frontend_gpu_matches_restatement(oracle_lib):
    import torch

    from voxrt_b200 import synth
    from voxrt_b200._lib import check_device
    from voxrt_b200.frontend import Frontend

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    rng = np.random.default_rng(31)
    t = np.arange(16000 * 3) / 16000.0
    waves = [
        synth.bandlimited_noise(rng, 2.5),                                  # config 3's audio
        (0.1 * rng.standard_normal(16000 * 3)).astype(np.float32),           # white noise
        (0.3 * np.sin(2 * np.pi * 440.0 * t) + 0.05 * rng.standard_normal(t.size)).astype(np.float32),
        (0.1 * rng.standard_normal(159)).astype(np.float32),                 # shorter than a hop: no frames
        (0.1 * rng.standard_normal(200)).astype(np.float32),                 # one frame: not normalised
        synth.bandlimited_noise(rng, 30.0),
    ]
    fe = Frontend()
    raw = fe.compute(waves, normalize=False)
    norm = fe.compute(waves, normalize=True)
    check_device()
    for w, r, nrm in zip(waves, raw, norm):
        n = len(w) // 160
        assert r.shape == (n, 128) and nrm.shape == (n, 128)
        if n == 0:
            continue
        p = oracle_lib.mel_power(w)
        want = oracle_lib.log_mel(w)
        got_p = np.exp(r.astype(np.float64)) - 5.9604645e-8
        scale = p.max(axis=1, keepdims=True)
        assert np.max(np.abs(got_p - p) / scale) < 1e-5
        strong = p >= 1e-3 * scale
        assert np.max(np.abs(r - want)[strong]) < 1e-3
        if n == 1:
            np.testing.assert_array_equal(nrm, r)
            continue
        wn = oracle_lib.normalize_feats(want)
        assert np.max(np.abs(nrm - wn)[strong]) < 1e-3
