"""GPU: the VAD head (VadHead::probs, vad.rs:39-82) against the oracle, bit for bit, on stacked utterances; the
long-form path (LongForm over the GPU frontend, subsampling and VAD head) against the oracle's LongForm fed with the
oracle's subsampling and VAD on the same log-mel features; and transcribe_long end to end (segments encoded and
decoded on the GPU) against the oracle encoder + decoder on every segment."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    _torch()
    from voxrt_b200 import synth

    enc_w, dec_w = synth.encoder(2), synth.decoder(seed=7)
    tensors, _ = synth.model_dir_tensors(enc_w, dec_w)
    path = synth.write_model_dir(str(tmp_path_factory.mktemp("m") / "m"), enc_w, dec_w)
    return path, enc_w, synth.decoder_f16_rounded(dec_w), synth.vad_weights(tensors)


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_vad_probs_bit_exact(model):
    torch = _torch()
    import oracle
    from voxrt_b200.vad import VadHead

    _, _, _, vw = model
    v = VadHead(vw, device=torch.cuda.current_device())
    rng = np.random.default_rng(4)
    lens = [1, 2, 3, 5, 37, 300]
    subs = [(rng.standard_normal((t, 1024)) * rng.choice([0.3, 1.0, 3.0])).astype(np.float32) for t in lens]
    got = v.probs_device(torch.from_numpy(np.concatenate(subs)).cuda(), lens).cpu().numpy()
    o = 0
    for s, t in zip(subs, lens):
        want = oracle.vad_probs(s, vw)
        assert np.array_equal(_bits(got[o:o + t]), _bits(want)), t
        o += t
    assert 0.0 < got.min() and got.max() < 1.0


def test_vad_from_model_dir(model):
    torch = _torch()
    from voxrt_b200.vad import VadHead

    path, _, _, vw = model
    a, b = VadHead(vw, device=torch.cuda.current_device()), VadHead.from_model(path, torch.cuda.current_device())
    x = torch.from_numpy(np.random.default_rng(5).standard_normal((50, 1024)).astype(np.float32)).cuda()
    assert np.array_equal(_bits(a.probs_device(x).cpu().numpy()), _bits(b.probs_device(x).cpu().numpy()))


def _components(path):
    torch = _torch()
    from voxrt_b200.decoder import TdtDecoder
    from voxrt_b200.encoder import CudaEncoder
    from voxrt_b200.frontend import Frontend
    from voxrt_b200.vad import VadHead

    dev = torch.cuda.current_device()
    return (Frontend(device=dev), CudaEncoder.from_model(path, device=dev), VadHead.from_model(path, dev),
            TdtDecoder.from_model(path, device=dev))


def _speechlike(rng, seconds, sr=16000):
    from voxrt_b200 import synth

    parts = []
    while sum(len(p) for p in parts) < seconds * sr:
        s = synth.bandlimited_noise(rng, float(rng.uniform(0.5, 12.0)), dbfs=-20.0 if rng.random() < 0.6 else -60.0)
        parts.append(s.astype(np.float32))
    return np.concatenate(parts)[:int(seconds * sr)]


def _oracle_block_vad(fe, sub_o, vw):
    import oracle

    def fn(block, skip, want):
        feats = fe.compute([np.asarray(block, np.float32)])[0]
        return oracle.vad_probs(sub_o.forward(feats), vw)[skip:skip + want]
    return fn


def test_longform_gpu_matches_oracle_state_machine(model):
    """Collect-only LongForm on the GPU components over 75 s of audio pushed in ragged chunks, against the oracle
    LongForm whose block probabilities come from the same GPU log-mel features through the oracle's subsampling and
    VAD head: the same closed ranges call by call, hence the same probabilities."""
    import oracle
    from oracle.longform import LongFormOracle
    from voxrt_b200.longform import LongForm, LongFormConfig

    path, enc_w, _, vw = model
    fe, enc, vad, dec = _components(path)
    rng = np.random.default_rng(6)
    x = _speechlike(rng, 75.0)
    cfg = LongFormConfig(collect_only=1, min_frames=20, max_frames=300)
    lf = LongForm(fe, enc, vad, None, cfg)
    ref = LongFormOracle(_oracle_block_vad(fe, oracle.OracleSubsampling(enc_w["sub"]), vw),
                         {"min_frames": 20, "max_frames": 300})
    a = 0
    while a < len(x):
        n = int(rng.integers(4000, 9 * 16000))
        assert lf.push(x[a:a + n]) == ref.push(x[a:a + n]), a
        a += n
    assert lf.flush() == ref.flush()
    assert lf.ranges() == ref.ranges and len(ref.ranges) >= 2


def _oracle_transcribe(fe, sub_o, layers, dec_o, x, ranges, spf=1280):
    import oracle

    out = []
    for s, e in ranges:
        feats = fe.compute([x[s:e]])[0]
        enc = oracle.encoder_forward(sub_o, layers, feats)
        em = dec_o.greedy(dec_o.project(enc))
        em = np.asarray(em, np.int32).reshape(-1, 3).copy()
        em[:, 1] += s // spf
        out.append(em)
    return np.concatenate(out) if out else np.zeros((0, 3), np.int32)


@pytest.mark.parametrize("seconds", [12.0, 47.0])
def test_transcribe_long_matches_oracle(model, seconds):
    """transcribe_long: 12 s (whole clip) and 47 s (VAD-segmented, segments batched through the encoder and one
    lockstep GPU decode) against the oracle encoder (2 layers) + decoder on every range: identical emissions."""
    import oracle
    from voxrt_b200.longform import LongFormConfig, transcribe_long

    path, enc_w, dec_w, vw = model
    fe, enc, vad, dec = _components(path)
    x = _speechlike(np.random.default_rng(int(seconds)), seconds)
    cfg = LongFormConfig(min_frames=20, max_frames=300)
    em, ranges = transcribe_long(fe, enc, vad, dec, x, cfg)
    if seconds <= 30:
        assert ranges == [(0, len(x))]
    else:
        assert len(ranges) >= 2
    sub_o = oracle.OracleSubsampling(enc_w["sub"])
    layers = [oracle.OracleLayer(lw) for lw in enc_w["layers"]]
    want = _oracle_transcribe(fe, sub_o, layers, oracle.TdtDecoder(dec_w), x, ranges)
    np.testing.assert_array_equal(em, want)
    assert em.shape[0] > 0


def test_longform_streaming_emissions_match_transcribe_per_segment(model):
    """Streaming LongForm (transcribing each closed segment as it closes) gives the emissions of its ranges
    transcribed independently."""
    import oracle
    from voxrt_b200.longform import LongForm, LongFormConfig

    path, enc_w, dec_w, vw = model
    fe, enc, vad, dec = _components(path)
    x = _speechlike(np.random.default_rng(9), 40.0)
    lf = LongForm(fe, enc, vad, dec, LongFormConfig(min_frames=20, max_frames=300))
    for a in range(0, len(x), 48000):
        lf.push(x[a:a + 48000])
    lf.flush()
    r = lf.ranges()
    assert len(r) >= 1
    sub_o = oracle.OracleSubsampling(enc_w["sub"])
    layers = [oracle.OracleLayer(lw) for lw in enc_w["layers"]]
    np.testing.assert_array_equal(lf.emissions(), _oracle_transcribe(fe, sub_o, layers, oracle.TdtDecoder(dec_w), x,
                                                                     r))


def test_encoder_subsample_device_matches_oracle(model):
    """vxg_encoder_subsample_device (the VAD head's input) on stacked utterances against the oracle's
    subsampling, bit for bit."""
    torch = _torch()
    import oracle
    from voxrt_b200 import synth
    from voxrt_b200.encoder import CudaEncoder

    path, enc_w, _, _ = model
    enc = CudaEncoder.from_model(path, device=torch.cuda.current_device())
    rng = np.random.default_rng(12)
    t_in = [16, 161, 400, 97]
    feats = [synth.feats(rng, t) for t in t_in]
    got = enc.subsample_device(torch.from_numpy(np.concatenate(feats)).cuda(), t_in).cpu().numpy()
    sub = oracle.OracleSubsampling(enc_w["sub"])
    o = 0
    for f in feats:
        want = sub.forward(f)
        assert np.array_equal(_bits(got[o:o + want.shape[0]]), _bits(want))
        o += want.shape[0]
    assert o == got.shape[0]
    enc.close()
