"""GPU parity: conv module middle (GLU -> depthwise conv with folded BN -> SiLU -> int8) against the oracle."""
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


def test_fold_bn_matches_oracle(oracle_lib):
    from voxrt_b200 import kernels, synth

    L = synth.layer(3)
    a = kernels.fold_bn(L["dw_weight"], L["bn_w"], L["bn_b"], L["bn_mean"], L["bn_var"])
    b = oracle_lib.fold_bn(L["dw_weight"], L["bn_w"], L["bn_b"], L["bn_mean"], L["bn_var"], 9)
    assert np.array_equal(a[0].view(np.uint32), b[0].view(np.uint32))
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))


@pytest.mark.parametrize("lengths", [[1], [4], [9], [64], [65], [375], [375, 3, 130, 64, 7]])
def test_conv_middle(K, oracle_lib, lengths):
    import torch

    from voxrt_b200 import synth
    from voxrt_b200._lib import check_device

    rng = np.random.default_rng(len(lengths) * 1000 + sum(lengths))
    d = 1024
    L = synth.layer(4)
    dw_t, dw_b = K.fold_bn(L["dw_weight"], L["bn_w"], L["bn_b"], L["bn_mean"], L["bn_var"])
    rows = sum(lengths)
    offs = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
    g = (2.0 * rng.standard_normal((rows, 2 * d))).astype(np.float32)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    hb, q = K.conv_glu_dw_silu(T(g), offs, lengths, T(dw_t), T(dw_b))
    check_device()
    hb, gq, gs = hb.cpu().numpy(), q.x.cpu().numpy(), q.scales.cpu().numpy()
    for o, t in zip(offs, lengths):
        want = oracle_lib.conv_middle(g[o:o + t], dw_t, dw_b)
        assert np.array_equal(hb[o:o + t].view(np.uint32), want.view(np.uint32)), f"t={t}"
        wq, ws = oracle_lib.quantize_rows(want, 128)
        np.testing.assert_array_equal(gq[o:o + t], wq)
        assert np.array_equal(gs[o:o + t].view(np.uint32), ws.view(np.uint32))
