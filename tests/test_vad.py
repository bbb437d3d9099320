"""VAD segmentation and the long-form state machine on the host: the library's segment() (vad.rs:140-240) against
the oracle's restatement on many probability tracks and configurations, and LongForm (longform.rs) in collect-only
mode over an external VAD against the oracle's LongFormOracle fed by the same VAD function: identical closed
ranges, call by call, for streams pushed in ragged chunks."""
import numpy as np
import pytest


def _tracks(rng):
    yield np.zeros(0, np.float32)
    yield np.full(40, 0.1, np.float32)                      # no speech: one segment over everything
    yield np.full(2000, 0.9, np.float32)                    # one run far above max_frames: split at minima
    yield rng.random(3000).astype(np.float32)               # noise around the threshold
    for _ in range(20):                                     # speech runs and pauses of random lengths
        parts = []
        for _ in range(rng.integers(1, 30)):
            n = int(rng.integers(1, 300))
            hi = rng.random() < 0.5
            parts.append((0.5 + 0.5 * rng.random(n) if hi else 0.5 * rng.random(n)).astype(np.float32))
        yield np.concatenate(parts)
    yield np.array([0.5, 0.49999997, 0.5], np.float32)      # the threshold itself counts as speech


@pytest.mark.parametrize("cfg", [{}, {"min_pause_frames": 0}, {"max_frames": 2, "min_frames": 0, "pad_frames": 0},
                                 {"max_frames": 100, "min_frames": 30, "pad_frames": 5, "threshold": 0.3},
                                 {"min_pause_frames": 3, "max_frames": 751, "min_frames": 1000}])
def test_segment_matches_oracle(cfg):
    import oracle
    from voxrt_b200.vad import SegmentConfig, segment

    rng = np.random.default_rng(3)
    for p in _tracks(rng):
        assert segment(p, SegmentConfig(**cfg)) == oracle.segment(p, cfg), (len(p), cfg)


def _audio(rng, seconds, sr=16000):
    """Alternating loud / quiet stretches (0.3-25 s) of noise: the VAD below calls a frame speech by its level."""
    out, n = [], int(seconds * sr)
    while sum(len(a) for a in out) < n:
        m = int(rng.uniform(0.3, 25.0) * sr)
        out.append((rng.standard_normal(m) * (1.0 if rng.random() < 0.6 else 0.05)).astype(np.float32))
    return np.concatenate(out)[:n]


def _level_vad(block, skip, want, spf=1280):
    """Probability of frame f of a block: a squashed RMS level of its 1280 samples (context-independent)."""
    n = len(block) // spf
    fr = np.asarray(block[:n * spf], np.float32).reshape(n, spf)
    p = (np.sqrt((fr.astype(np.float64) ** 2).mean(axis=1)) / 1.2).clip(0, 1).astype(np.float32)
    return p[skip:skip + want]


@pytest.mark.parametrize("seconds,seed", [(5.0, 1), (95.0, 2), (301.5, 3)])
def test_longform_collect_only_matches_oracle(seconds, seed):
    from oracle.longform import LongFormOracle
    from voxrt_b200.longform import LongForm

    rng = np.random.default_rng(seed)
    x = _audio(rng, seconds)
    lf = LongForm(vad_fn=_level_vad)
    ref = LongFormOracle(_level_vad)
    a = 0
    while a < len(x):
        n = int(rng.integers(1, 7 * 16000))
        got, want = lf.push(x[a:a + n]), ref.push(x[a:a + n])
        assert got == want, (a, n)
        a += n
    assert lf.flush() == ref.flush()
    assert lf.ranges() == ref.ranges
    assert lf.stats()["max_pending"] == ref.max_pending
    if seconds > 60:
        assert len(ref.ranges) > 1
    # segments are ordered, disjoint and inside the stream
    r = lf.ranges()
    assert all(0 <= s < e <= len(x) for s, e in r) and all(r[i][1] <= r[i + 1][0] for i in range(len(r) - 1))


def test_longform_bad_callback_reports_error():
    from voxrt_b200._lib import VxgError
    from voxrt_b200.longform import LongForm

    def bad(block, skip, want):
        raise RuntimeError("no VAD")

    lf = LongForm(vad_fn=bad)
    with pytest.raises(VxgError):
        lf.push(np.zeros(200000, np.float32))


def test_segment_known_answers_from_the_reference_tests():
    """The reference's own segmentation_rules test (crates/voxrt/tests/golden_vad.rs:44-79): under max 375 / min 63,
    10 s of speech, a 1 s pause and 5 s of speech give exactly [(0, 127), (136, 201)]; 60 s of speech is split under
    the cap from 0 to 750; under the defaults the 5 s run merges into one segment and 90 s is split in >= 2 pieces
    of at most 750 + 2 frames."""
    from voxrt_b200.vad import SegmentConfig, segment

    cfg = SegmentConfig(max_frames=375, min_frames=63)
    p = np.array([0.9] * 125 + [0.1] * 13 + [0.9] * 63, np.float32)
    assert segment(p, cfg) == [(0, 127), (136, 201)]
    long = np.full(750, 0.95, np.float32)
    s = segment(long, cfg)
    assert all(e - b <= 375 + 2 for b, e in s) and s[0][0] == 0 and s[-1][1] == 750
    d = SegmentConfig()
    assert (d.max_frames, d.min_frames, d.min_pause_frames, d.pad_frames) == (750, 125, 8, 2)
    assert abs(d.threshold - 0.5) == 0
    assert len(segment(p, d)) == 1
    s = segment(np.full(1125, 0.95, np.float32), d)
    assert len(s) >= 2 and all(e - b <= 750 + 2 for b, e in s)


@pytest.mark.parametrize("seed", [4, 5])
def test_longform_ranges_do_not_depend_on_chunking(seed):
    """Streaming equals offline (crates/voxrt/tests/streaming.rs:9-40): the closed ranges are the same whatever
    the push sizes (1 s, 3.7 s, 10 s, one piece)."""
    from voxrt_b200.longform import LongForm

    rng = np.random.default_rng(seed)
    x = _audio(rng, 140.0)
    got = []
    for chunk in (16000, 59200, 160000, len(x)):
        lf = LongForm(vad_fn=_level_vad)
        for a in range(0, len(x), chunk):
            lf.push(x[a:a + chunk])
        lf.flush()
        got.append(lf.ranges())
    assert all(g == got[0] for g in got[1:]) and len(got[0]) >= 2
