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
