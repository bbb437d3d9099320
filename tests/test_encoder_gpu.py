"""GPU parity of the whole encoder path against the oracle (bit for bit): layers on subsampled input for a
token-stacked batch, and subsampling + layers through the host-buffer entry points, in both weight formats."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_LAYERS = 2


@pytest.fixture(scope="module")
def model():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voxrt_b200 import synth

    return {"sub": synth.subsampling(99), "layers": [synth.layer(100 + i) for i in range(N_LAYERS)]}


@pytest.fixture(scope="module")
def oracle_model(model, oracle_lib):
    return oracle_lib.OracleSubsampling(model["sub"]), [oracle_lib.OracleLayer(lw) for lw in model["layers"]]


def _bits(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("weights", ["2bit", "int8"])
def test_layers_stacked_batch(model, oracle_model, oracle_lib, weights):
    import torch

    from voxrt_b200.encoder import CudaEncoder

    enc = CudaEncoder.load(model, weights=weights)
    rng = np.random.default_rng(5)
    lengths = [37, 130, 5, 64]
    xs = [rng.standard_normal((t, 1024)).astype(np.float32) for t in lengths]
    out = enc.forward(torch.from_numpy(np.concatenate(xs)).cuda(), lengths).cpu().numpy()
    _, layers = oracle_model
    r = 0
    for x, t in zip(xs, lengths):
        pos = oracle_lib.rel_pos_table(t)
        want = x
        for L in layers:
            want = L.forward(want, pos)
        got = out[r:r + t]
        r += t
        bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
        assert bad.size == 0, f"[{weights}] t={t}: {bad.size} mismatches, max abs {np.abs(got - want).max()}"
    enc.close()


def test_forward_feats_and_batch(model, oracle_model, oracle_lib):
    from voxrt_b200 import synth
    from voxrt_b200.encoder import CudaEncoder

    enc = CudaEncoder.load(model)
    sub, layers = oracle_model
    rng = np.random.default_rng(6)
    feats = [synth.feats(rng, t) for t in (161, 400, 97)]
    want = [oracle_lib.encoder_forward(sub, layers, f) for f in feats]
    one, te = enc.forward_feats(feats[0])
    assert te == want[0].shape[0] and _bits(one, want[0])
    outs = enc.forward_batch(feats)
    for g, w in zip(outs, want):
        assert _bits(g, w)
    for o in outs:  # caller-owned outputs, reused: every frame is written again
        o.fill(np.nan)
    again = enc.forward_batch(feats, outs)
    assert all(a is o for a, o in zip(again, outs))
    for g, w in zip(outs, want):
        assert _bits(g, w)
    # page-locked feats and outputs: direct DMA, inputs in groups overlapped with the front end
    feats_p = [enc.pinned_array(f.shape) for f in feats]
    for a, f in zip(feats_p, feats):
        a[...] = f
    outs_p = [enc.pinned_array(o.shape) for o in outs]
    for o in outs_p:
        o.fill(np.nan)
    enc.forward_batch(feats_p, outs_p)
    for g, w in zip(outs_p, want):
        assert _bits(g, w)
    for o in outs:
        o.fill(np.nan)
    enc.forward_batch(feats_p, outs)  # page-locked inputs, pageable outputs
    for g, w in zip(outs, want):
        assert _bits(g, w)
    enc.close()


def test_config2_one_block_t375(oracle_lib):
    """one FastConformer block (d 1024, FF 4096, 8 heads x 128, conv kernel 9) on one utterance
    of T = 375 frames of N(0, 1), batch 1, seed 2 (ConformerLayer::forward_profiled, encoder.rs:706-756)."""
    import torch

    from voxrt_b200 import synth
    from voxrt_b200.encoder import CudaEncoder

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lw = synth.layer(2)
    enc = CudaEncoder.load({"sub": synth.subsampling(99), "layers": [lw]})
    x = np.random.default_rng(2).standard_normal((375, 1024)).astype(np.float32)
    got = enc.forward(torch.from_numpy(x).cuda(), [375]).cpu().numpy()
    want = oracle_lib.OracleLayer(lw).prepare().forward(x, oracle_lib.rel_pos_table(375))
    bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{bad.size} mismatches, max abs {np.abs(got - want).max()}"
    enc.close()


def test_config3_full_encoder_bench_workload(oracle_lib):
    """BASELINE config 3 exactly as bench.py times it: rank 0's 64 utterances (U(2, 30) s, 12,955 encoder frames
    token-stacked), the conv-subsampling front end and all 24 layers, through the device-resident batch entry.
    Every GEMM then runs with many tiles per CTA (weight slabs reused across m-tiles, TMEM phases carried over),
    including the fused q|k|v-quantising, GLU and SiLU -> int8 epilogues. Every utterance is compared bit for bit
    with the oracle's Encoder::forward (encoder.rs:816-856)."""
    import torch

    from voxrt_b200 import synth
    from voxrt_b200.encoder import CudaEncoder

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    mdl = synth.encoder(24)
    secs, t_in, feats = synth.config3_workload(0, 64)
    te = np.array([CudaEncoder.out_frames(int(t)) for t in t_in])
    assert te.sum() == 12955
    enc = CudaEncoder.load(mdl)
    out = torch.empty((int(te.sum()), 1024), dtype=torch.float32, device="cuda")
    enc.forward_device(torch.from_numpy(np.concatenate(feats)).cuda(), t_in, out)
    got = out.cpu().numpy()
    enc.close()
    sub = oracle_lib.OracleSubsampling(mdl["sub"])
    layers = [oracle_lib.OracleLayer(lw).prepare() for lw in mdl["layers"]]
    oracle_lib.set_threads(0)
    offs = np.concatenate([[0], np.cumsum(te)])
    for u, f in enumerate(feats):
        want = oracle_lib.encoder_forward(sub, layers, f)
        g = got[offs[u]:offs[u + 1]]
        bad = np.flatnonzero(g.view(np.uint32) != want.view(np.uint32))
        assert bad.size == 0, f"utterance {u} (t_e={te[u]}): {bad.size} mismatches, max abs {np.abs(g - want).max()}"


def test_encoder_from_model_dir(tmp_path, oracle_lib):
    """GpuEncoder::load from a thrush-ternary-v2 directory (vxg_encoder_create_from_model) produces the same frames,
    bit for bit, as the encoder built from the arrays the directory was written from, and both match the oracle."""
    import torch

    from voxrt_b200 import synth
    from voxrt_b200.encoder import CudaEncoder

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    enc_w = synth.encoder(2)
    path = synth.write_model_dir(str(tmp_path / "m"), enc_w, synth.decoder(seed=7))
    a = CudaEncoder.load(enc_w)
    b = CudaEncoder.from_model(path)
    feats = synth.feats(np.random.default_rng(8), 333)
    ya, _ = a.forward_feats(feats)
    yb, _ = b.forward_feats(feats)
    assert _bits(ya, yb)
    sub = oracle_lib.OracleSubsampling(enc_w["sub"])
    layers = [oracle_lib.OracleLayer(lw) for lw in enc_w["layers"]]
    assert _bits(yb, oracle_lib.encoder_forward(sub, layers, feats))
    a.close()
    b.close()
