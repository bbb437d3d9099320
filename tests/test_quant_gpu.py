"""GPU parity: quantisation and the fused LayerNorm -> int8 pass against the oracle, bit for bit."""
import numpy as np
import pytest

from conftest import LCG

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voxrt_b200 import kernels

    return kernels


def _bits_equal(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_quantize_rows_ties_zero_and_sizes(K, oracle_lib):
    import torch

    rng = np.random.default_rng(0)
    for n, inp, group in ((1, 128, 128), (7, 1024, 128), (333, 4096, 128), (5, 384, 384), (3, 1024, 1024)):
        x = (rng.standard_normal((n, inp)) * rng.uniform(0.1, 10)).astype(np.float32)
        x[0, :group] = 0.0                                              # all-zero group -> scale 1
        x[-1, ::5] = (np.arange(len(x[-1, ::5])) + 0.5).astype(np.float32) * np.float32(0.1)  # .5 ties
        q, s = oracle_lib.quantize_rows(x, group)
        A = K.quantize(torch.from_numpy(x).cuda(), group)
        np.testing.assert_array_equal(A.x.cpu().numpy(), q)
        assert _bits_equal(A.scales.cpu().numpy(), s)


def test_ln_quant_matches_oracle(K, oracle_lib):
    import torch

    rng = np.random.default_rng(1)
    for n, d in ((1, 1024), (37, 1024), (1000, 1024), (9, 4096), (4, 1000)):
        x = (rng.standard_normal((n, d)) * 3 + 1).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
        b = (0.1 * rng.standard_normal(d)).astype(np.float32)
        group = 128 if d % 128 == 0 else 8
        q, s = oracle_lib.ln_quant_rows(x, g, b, group)
        xt = torch.from_numpy(x).cuda()
        A = K.ln_quant(xt, torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda(), group)
        np.testing.assert_array_equal(A.x.cpu().numpy(), q)
        assert _bits_equal(A.scales.cpu().numpy(), s)


def test_norm_out_then_ln_quant_fused(K, oracle_lib):
    """norm_out (f32, written back to x) followed by the next layer's LayerNorm -> int8, in one pass."""
    import torch

    rng = np.random.default_rng(2)
    n, d = 257, 1024
    x = rng.standard_normal((n, d)).astype(np.float32)
    g0, b0, g1, b1 = [(1 + 0.1 * rng.standard_normal(d)).astype(np.float32) if i % 2 == 0 else
                      (0.1 * rng.standard_normal(d)).astype(np.float32) for i in range(4)]
    y = np.stack([oracle_lib.layer_norm_row(x[t], g0, b0) for t in range(n)])
    q, s = oracle_lib.ln_quant_rows(y, g1, b1, 128)
    xt = torch.from_numpy(x).cuda()
    T = lambda a: torch.from_numpy(a).cuda()
    A = K.ln_quant(xt, T(g1), T(b1), 128, pre=(T(g0), T(b0)), x_out=xt)
    assert _bits_equal(xt.cpu().numpy(), y)
    np.testing.assert_array_equal(A.x.cpu().numpy(), q)
    assert _bits_equal(A.scales.cpu().numpy(), s)
