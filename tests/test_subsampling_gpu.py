"""GPU parity: the f32 subsampling front end against the oracle's Subsampling::forward, bit for bit."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voxrt_b200 import kernels

    return kernels


def test_linear_f32_lane_order(K, oracle_lib):
    import torch

    rng = np.random.default_rng(0)
    # small M, an N tail, a long K, and several 128-row blocks with tails in both M and N
    for M, Kd, N in ((2, 256, 256), (37, 256, 256), (100, 4096, 1024), (5, 64, 300), (300, 96, 130)):
        x = rng.standard_normal((M, Kd)).astype(np.float32)
        w = (rng.standard_normal((N, Kd)) / np.sqrt(Kd)).astype(np.float32)
        b = rng.standard_normal(N).astype(np.float32)
        want = oracle_lib.linear(x, w, b)
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        T = lambda a: torch.from_numpy(a).cuda()
        from voxrt_b200._lib import check, lib
        from voxrt_b200.kernels import _ptr, _stream_ptr

        xt, wt, bt = T(x), T(w), T(b)  # keep the device buffers alive until the kernel has run
        check(lib().vxg_linear_f32(_ptr(xt), M, Kd, _ptr(wt), _ptr(bt), N, 0, _ptr(y), _stream_ptr()))
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (M, Kd, N)


@pytest.mark.parametrize("lengths", [[9], [17], [100], [301], [3001], [17, 250, 64, 1201]])
def test_subsampling_matches_oracle(K, oracle_lib, lengths):
    import torch

    from voxrt_b200 import synth

    sw = synth.subsampling(99)
    S = K.Subsampling(sw)
    O = oracle_lib.OracleSubsampling(sw)
    rng = np.random.default_rng(sum(lengths))
    feats = [synth.feats(rng, t) for t in lengths]
    out = S.forward(torch.from_numpy(np.concatenate(feats)).cuda(), lengths).cpu().numpy()
    r = 0
    for f in feats:
        want = O.forward(f)
        got = out[r:r + want.shape[0]]
        r += want.shape[0]
        bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
        assert bad.size == 0, f"t_in={f.shape[0]}: {bad.size} mismatches"
    assert r == out.shape[0]
