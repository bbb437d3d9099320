"""TDT decoder (decoder.rs, int8 mode): the product's host decoder (libvxg, C ABI) against the oracle restatement,
bit for bit: joint logits, one prediction-network step, greedy emissions (token, frame, duration) on utterances of
ragged lengths including the zero-duration / max-symbols and all-blank paths, and the threaded batch entry. The GPU
encoder projection (project_encoder) is checked against the oracle's linear in tests/test_decoder_gpu.py."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def dec():
    import oracle
    from voxrt_b200 import synth
    from voxrt_b200.decoder import TdtDecoder

    m = synth.decoder(seed=7)
    return m, TdtDecoder(m), oracle.TdtDecoder(m)


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_joint_bit_exact(dec):
    m, P, O = dec
    rng = np.random.default_rng(1)
    for scale in (0.1, 1.0, 30.0):
        enc_t = (scale * rng.standard_normal(m["hidden"])).astype(np.float32)
        g = (scale * rng.standard_normal(m["hidden"])).astype(np.float32)
        assert np.array_equal(_bits(P.joint(enc_t, g)), _bits(O.joint(enc_t, g)))
    z = np.zeros(m["hidden"], np.float32)  # all-zero joint input: every group scale is 1
    assert np.array_equal(_bits(P.joint(z, z)), _bits(O.joint(z, z)))


def test_pred_step_bit_exact(dec):
    m, P, O = dec
    rng = np.random.default_rng(2)
    h = m["hidden"]
    for token in (0, m["blank"], 4095):
        hs = (0.5 * rng.standard_normal((2, h))).astype(np.float32)
        cs = rng.standard_normal((2, h)).astype(np.float32)
        for a, b in zip(P.pred_step(token, hs, cs), O.pred_step(token, hs, cs)):
            assert np.array_equal(_bits(a), _bits(b))
    zero = np.zeros((2, h), np.float32)  # the greedy loop's first step: blank from the zero state
    for a, b in zip(P.pred_step(m["blank"], zero, zero), O.pred_step(m["blank"], zero, zero)):
        assert np.array_equal(_bits(a), _bits(b))


@pytest.mark.parametrize("t", [0, 1, 2, 7, 40])
def test_greedy_matches_oracle(dec, t):
    m, P, O = dec
    proj = np.random.default_rng(100 + t).standard_normal((t, m["hidden"])).astype(np.float32)
    got, want = P.greedy(proj), O.greedy(proj)
    np.testing.assert_array_equal(got, want)
    if t:
        assert got.shape[0] > 0


def _biased(m, dur0=0.0, blank=0.0):
    m = dict(m)
    hb = np.array(m["head_b"], np.float32).copy()
    hb[m["vocab"]] += dur0          # duration 0 preferred: the inner loop runs to max_symbols
    hb[m["blank"]] += blank         # blank preferred: the prediction output is reused across frames
    m["head_b"] = hb
    return m


@pytest.mark.parametrize("dur0,blank", [(50.0, 0.0), (50.0, 50.0), (0.0, 50.0)])
def test_greedy_edge_paths(dec, dur0, blank):
    import oracle
    from voxrt_b200.decoder import TdtDecoder

    m = _biased(dec[0], dur0, blank)
    P, O = TdtDecoder(m), oracle.TdtDecoder(m)
    proj = np.random.default_rng(5).standard_normal((6, m["hidden"])).astype(np.float32)
    got, want = P.greedy(proj), O.greedy(proj)
    np.testing.assert_array_equal(got, want)
    if dur0 and not blank:  # every frame emits max_symbols tokens at duration 0
        assert got.shape[0] == 6 * m["max_symbols"] and (got[:, 2] == 0).all()
    if blank:
        assert got.shape[0] == 0


def test_greedy_batch_equals_single(dec):
    m, P, _ = dec
    rng = np.random.default_rng(9)
    projs = [rng.standard_normal((t, m["hidden"])).astype(np.float32) for t in (3, 0, 17, 1, 25, 9)]
    batch = P.greedy_batch(projs, threads=3)
    for p, b in zip(projs, batch):
        np.testing.assert_array_equal(P.greedy(p), b)


def test_bad_arguments(dec):
    from voxrt_b200._lib import VxgError

    m, P, _ = dec
    with pytest.raises(VxgError):
        P.pred_step(m["vocab"], np.zeros((2, m["hidden"]), np.float32), np.zeros((2, m["hidden"]), np.float32))
    bad = dict(m)
    bad["hidden"] = 100  # not a multiple of 128
    from voxrt_b200.decoder import TdtDecoder

    with pytest.raises(VxgError):
        TdtDecoder(bad)
