"""GPU: the TDT decoder's encoder projection (Decoder::project_encoder, decoder.rs:123-134) on the device against
the oracle's linear, bit for bit, for one frame (the reference's gemv order) and several (tile_rows order)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t", [1, 2, 5, 37, 300])
def test_project_device_bit_exact(t):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import oracle
    from voxrt_b200 import synth
    from voxrt_b200._lib import check_device
    from voxrt_b200.decoder import TdtDecoder

    m = synth.decoder(seed=11)
    P = TdtDecoder(m, device=torch.cuda.current_device())
    O = oracle.TdtDecoder(m)
    enc = np.random.default_rng(t).standard_normal((t, m["d_model"])).astype(np.float32)
    got = P.project_device(torch.from_numpy(enc).cuda())
    torch.cuda.synchronize()
    check_device()
    want = O.project(enc)
    g = got.cpu().numpy()
    bad = np.flatnonzero(g.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{bad.size} mismatches, first {np.unravel_index(bad[0], g.shape)}"


# ------------------------------------------------------------------------------ batched greedy decode on the GPU
def _gpu_or_skip():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def gdec():
    torch = _gpu_or_skip()
    import oracle
    from voxrt_b200 import synth
    from voxrt_b200.decoder import TdtDecoder

    m = synth.decoder(seed=7)
    return m, TdtDecoder(m, device=torch.cuda.current_device()), oracle.TdtDecoder(m)


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_pred_step_device_bit_exact(gdec):
    """vxg_tdt_pred_step_device on 70 inputs (two lane tiles) against the host step, which the CPU tests pin to
    the oracle: g, h', c' as bit patterns."""
    import torch

    from voxrt_b200._lib import check_device

    m, P, _ = gdec
    rng = np.random.default_rng(21)
    n, h, nl = 70, m["hidden"], len(m["lstm"])
    tokens = rng.integers(0, m["vocab"], n).astype(np.int32)
    tokens[:3] = (0, m["blank"], m["vocab"] - 1)
    hs = (0.5 * rng.standard_normal((n, nl, h))).astype(np.float32)
    cs = (rng.standard_normal((n, nl, h)) * rng.choice([0.1, 1.0, 30.0], (n, 1, 1))).astype(np.float32)
    hs[3], cs[3] = 0.0, 0.0  # the loop's first step: zero state
    dev = lambda a: torch.from_numpy(a).cuda()
    g, hn, cn = P.pred_step_device(dev(tokens), dev(hs), dev(cs))
    torch.cuda.synchronize()
    check_device()
    g, hn, cn = g.cpu().numpy(), hn.cpu().numpy(), cn.cpu().numpy()
    for j in range(n):
        wg, wh, wc = P.pred_step(int(tokens[j]), hs[j], cs[j])
        assert np.array_equal(_bits(g[j]), _bits(wg)), f"g of input {j}"
        assert np.array_equal(_bits(hn[j]), _bits(wh)), f"h of input {j}"
        assert np.array_equal(_bits(cn[j]), _bits(wc)), f"c of input {j}"


def test_joint_device_bit_exact(gdec):
    """vxg_tdt_joint_device on 130 inputs (three lane tiles, all 129 head row blocks) against the host joint."""
    import torch

    m, P, _ = gdec
    rng = np.random.default_rng(22)
    n, h = 130, m["hidden"]
    sc = rng.choice([0.1, 1.0, 30.0], (n, 1))
    enc = (sc * rng.standard_normal((n, h))).astype(np.float32)
    g = (sc * rng.standard_normal((n, h))).astype(np.float32)
    enc[5], g[5] = 0.0, 0.0  # all-zero joint input: every group scale is 1
    got = P.joint_device(torch.from_numpy(enc).cuda(), torch.from_numpy(g).cuda())
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    for j in range(n):
        assert np.array_equal(_bits(got[j]), _bits(P.joint(enc[j], g[j]))), f"input {j}"


def _stack(projs):
    import torch

    return torch.from_numpy(np.concatenate(projs) if projs else np.zeros((0, 1), np.float32)).cuda().contiguous()


def test_greedy_device_matches_oracle(gdec):
    """Ragged utterances (0 frames included) decoded together on the GPU, against the oracle's greedy each."""
    m, P, O = gdec
    lens = [0, 1, 2, 7, 40, 3, 17, 25, 9, 0, 64, 33]
    projs = [np.random.default_rng(100 + i).standard_normal((t, m["hidden"])).astype(np.float32)
             for i, t in enumerate(lens)]
    got = P.greedy_device(_stack(projs), lens)
    for i, (p, g) in enumerate(zip(projs, got)):
        np.testing.assert_array_equal(g, O.greedy(p), err_msg=f"utterance {i} ({lens[i]} frames)")


@pytest.mark.parametrize("dur0,blank", [(50.0, 0.0), (50.0, 50.0), (0.0, 50.0)])
def test_greedy_device_edge_paths(gdec, dur0, blank):
    """The zero-duration / max-symbols path (every frame emits max_symbols tokens) and the all-blank path (the
    prediction output reused across frames), as the CPU tests, on the GPU."""
    import torch

    import oracle
    from voxrt_b200.decoder import TdtDecoder

    m = dict(gdec[0])
    hb = np.array(m["head_b"], np.float32).copy()
    hb[m["vocab"]] += dur0
    hb[m["blank"]] += blank
    m["head_b"] = hb
    P, O = TdtDecoder(m, device=torch.cuda.current_device()), oracle.TdtDecoder(m)
    lens = [6, 1, 11]
    projs = [np.random.default_rng(5 + i).standard_normal((t, m["hidden"])).astype(np.float32)
             for i, t in enumerate(lens)]
    got = P.greedy_device(_stack(projs), lens)
    for p, g, t in zip(projs, got, lens):
        np.testing.assert_array_equal(g, O.greedy(p))
        if dur0 and not blank:
            assert g.shape[0] == t * m["max_symbols"] and (g[:, 2] == 0).all()
        if blank:
            assert g.shape[0] == 0


def test_greedy_device_truncated_then_redone(gdec):
    """Utterances that emit more than their first capacity are decoded again with the full bound."""
    m, P, _ = gdec
    lens = [40, 5, 30]
    projs = [np.random.default_rng(300 + i).standard_normal((t, m["hidden"])).astype(np.float32)
             for i, t in enumerate(lens)]
    got = P.greedy_device(_stack(projs), lens, per_frame=0)  # room for 16 at first
    for p, g in zip(projs, got):
        np.testing.assert_array_equal(g, P.greedy(p))
    assert max(g.shape[0] for g in got) > 16


def test_greedy_device_config5_sizes(gdec):
    """Config 5's decoder on 300 utterances of 12-750 frames (1-60 s of audio), log-uniform like the box workload,
    decoded in one lockstep batch, against the host decoder's threaded batch."""
    m, P, _ = gdec
    rng = np.random.default_rng(55)
    lens = np.exp(rng.uniform(np.log(12), np.log(750), 300)).astype(int).tolist()
    projs = [(0.5 * rng.standard_normal((t, m["hidden"]))).astype(np.float32) for t in lens]
    got = P.greedy_device(_stack(projs), lens)
    want = P.greedy_batch(projs)
    for i, (g, w) in enumerate(zip(got, want)):
        np.testing.assert_array_equal(g, w, err_msg=f"utterance {i} ({lens[i]} frames)")


def test_rank_pipeline_gpu_decode_equals_host_decode():
    """voxrt_b200.box.RankPipeline.transcribe: encoder (2 layers) + projection + TDT greedy decode over several
    length buckets, with the batched GPU decode on its own stream against the host decoder threads: identical
    emissions for every utterance."""
    torch = _gpu_or_skip()
    from voxrt_b200 import box, synth
    from voxrt_b200.decoder import TdtDecoder
    from voxrt_b200.encoder import CudaEncoder

    dev = torch.cuda.current_device()
    enc = CudaEncoder.load(synth.encoder(2), device=dev)
    dec = TdtDecoder(synth.decoder(seed=7), device=dev)
    rng = np.random.default_rng(77)
    t_in = [int(x) for x in rng.integers(40, 900, 14)]
    feats = [synth.feats(rng, t) for t in t_in]
    buckets = box.plan(t_in, 1, budget=250)[0]
    assert len(buckets) >= 3
    pipe = box.RankPipeline(enc, dec, decode_threads=4)
    got = pipe.transcribe(feats, buckets, decode="gpu")
    want = pipe.transcribe(feats, buckets, decode="host")
    assert sorted(got) == list(range(len(t_in)))
    for u in range(len(t_in)):
        np.testing.assert_array_equal(got[u], want[u], err_msg=f"utterance {u}")
    assert sum(len(g) for g in got.values()) > 0


def test_rank_pipeline_encode_two_handles():
    """RankPipeline.encode with a second encoder handle (alternate buckets on two host threads, two host-buffer C ABI
    calls in flight on one GPU) returns the same frames, bit for bit, as one handle taking the buckets in turn."""
    torch = _gpu_or_skip()
    from voxrt_b200 import box, synth
    from voxrt_b200.encoder import CudaEncoder

    dev = torch.cuda.current_device()
    m = synth.encoder(2)
    rng = np.random.default_rng(78)
    t_in = [int(x) for x in rng.integers(40, 900, 14)]
    feats = [synth.feats(rng, t) for t in t_in]
    buckets = box.plan(t_in, 1, budget=250)[0]
    assert len(buckets) >= 3
    one = box.RankPipeline(CudaEncoder.load(m, device=dev)).encode(feats, buckets)
    two_pipe = box.RankPipeline(CudaEncoder.load(m, device=dev), second_encoder=CudaEncoder.load(m, device=dev))
    for _ in range(2):
        two = two_pipe.encode(feats, buckets)
        assert sorted(two) == list(range(len(t_in)))
        for u in range(len(t_in)):
            np.testing.assert_array_equal(two[u].view(np.uint32), one[u].view(np.uint32), err_msg=f"utterance {u}")


@pytest.mark.parametrize("hidden,vocab,layers,durations,max_symbols", [
    (384, 1000, 1, (0, 2, 5), 3),
    (128, 64, 3, (0, 1), 5),
    (256, 8193, 4, (0, 1, 2, 3, 4), 10),
])
def test_greedy_device_other_decoder_shapes(hidden, vocab, layers, durations, max_symbols):
    """The GPU decode for other decoder shapes (1, 3 and 4 LSTM layers, hidden 128 / 256 / 384, other duration sets
    and symbol caps, head rows not a multiple of 64) against the oracle on ragged utterances."""
    torch = _gpu_or_skip()
    import oracle
    from voxrt_b200 import synth
    from voxrt_b200.decoder import TdtDecoder

    m = synth.decoder(seed=hidden + layers, hidden=hidden, vocab=vocab, n_layers=layers, durations=durations,
                      max_symbols=max_symbols)
    P, O = TdtDecoder(m, device=torch.cuda.current_device()), oracle.TdtDecoder(m)
    lens = [13, 1, 70, 0, 129]
    projs = [np.random.default_rng(40 + i).standard_normal((t, hidden)).astype(np.float32) for i, t in enumerate(lens)]
    got = P.greedy_device(_stack(projs), lens)
    for i, (p, g) in enumerate(zip(projs, got)):
        np.testing.assert_array_equal(g, O.greedy(p), err_msg=f"utterance {i}")
    P.close()
