"""GPU parity: the tcgen05 ternary GEMM against the scalar oracle, bit for bit (int32 group sums and f32 outputs),
on the reference's own kernel-test shapes and vectors plus BASELINE config 1."""
import numpy as np
import pytest

from conftest import LCG
from refgen import acts_f32, random_matrix, x86_ternary

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voxrt_b200 import kernels

    return kernels


def _run(K, oracle, trits_or_q, s16, out, inp, group, xf, ep, ep_scale=0.0, y0=None, want_sums=True, bias=None,
         fmts=("2bit", "int8")):
    import torch

    from voxrt_b200.synth import pack_trits

    if trits_or_q.dtype == np.int8:
        q = pack_trits(trits_or_q)
    else:
        q = trits_or_q
    w_rows, sw = oracle.unpack_matrix(q, s16, out, inp, group)
    xq, sx = oracle.quantize_rows(xf, group)
    n = xf.shape[0]
    y_init = np.zeros((n, out), np.float32) if y0 is None else y0
    want, ref_sums = oracle.gemm(w_rows, sw, xq, sx, group, ep, ep_scale, y=y_init, bias=bias, want_sums=True)
    from voxrt_b200._lib import check_device

    X = K.QuantAct(torch.from_numpy(xq).cuda(), torch.from_numpy(sx).cuda(), group)
    b = None if bias is None else torch.from_numpy(bias).cuda()
    # with the group sums requested the kernel takes its generic group loop; without, the unrolled one (when
    # K / G is a multiple of 8): both must match the oracle bit for bit
    for fmt in fmts:
        W = K.TernaryMatrix.from_packed(q, s16, out, inp, group, fmt=fmt)
        for with_sums in ((True, False) if want_sums else (False,)):
            y = torch.from_numpy(y_init.copy()).cuda()
            sums = torch.zeros((n, out, inp // group), dtype=torch.int32, device="cuda") if with_sums else None
            K.gemm_ep(W, X, y, b, K.Epilogue(ep, ep_scale), group_sums=sums)
            torch.cuda.synchronize()
            check_device()
            got = y.cpu().numpy()
            if with_sums:
                np.testing.assert_array_equal(sums.cpu().numpy(), ref_sums, err_msg=fmt)
            bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
            assert bad.size == 0, f"[{fmt}, sums={with_sums}] {bad.size} f32 mismatches, first at " \
                                  f"{np.unravel_index(bad[0], got.shape)}: {got.flat[bad[0]]} vs {want.flat[bad[0]]}"


def test_simd_equals_scalar_shapes(K, oracle_lib):
    """kernels.rs:35-53 shapes and vectors: (7,128) (9,256) (64,1024) (130,4096) x n in {1,3,4,5,17}."""
    rng = LCG(42)
    for out, inp in ((7, 128), (9, 256), (64, 1024), (130, 4096)):
        q, s16, _ = random_matrix(out, inp, rng)
        for n in (1, 3, 4, 5, 17):
            xf = acts_f32(n, inp, rng)
            _run(K, oracle_lib, q, s16, out, inp, 128, xf, 0)


def test_epilogues_identical(K, oracle_lib):
    """kernels.rs:91-112: Store / Silu / AddScaled(0.5) on a pre-filled y."""
    rng = LCG(5)
    out, inp, n = 64, 1024, 13
    q, s16, _ = random_matrix(out, inp, rng)
    xf = acts_f32(n, inp, rng)
    base = np.array([(i % 7) - 3.0 for i in range(n * out)], np.float32).reshape(n, out)
    for ep, s in ((0, 0.0), (1, 0.0), (2, 0.5)):
        _run(K, oracle_lib, q, s16, out, inp, 128, xf, ep, s, y0=base.copy())


def test_x86_list_and_extremes(K, oracle_lib):
    """x86_kernels.rs ternary shapes and the saturation extremes, all three epilogues, with a bias."""
    rng = LCG(3)
    for out, inp in ((7, 128), (16, 256), (33, 1024), (130, 4096)):
        trits, _, s16 = x86_ternary(out, inp, rng)
        for n in (1, 2, 9, 17):
            xf = acts_f32(n, inp, rng)
            init = np.array([np.float32(rng.next() % 100) * np.float32(0.01) for _ in range(n * out)],
                            np.float32).reshape(n, out)
            for ep, s in ((0, 0.0), (1, 0.0), (2, 0.37)):
                _run(K, oracle_lib, trits, s16, out, inp, 128, xf, ep, s, y0=init.copy())
    trits, _, s16 = x86_ternary(32, 1024, rng, extreme=True)
    xf = acts_f32(5, 1024, rng, extreme=True)
    bias = np.linspace(-1, 1, 32).astype(np.float32)
    _run(K, oracle_lib, trits, s16, 32, 1024, 128, xf, 0, bias=bias)


def test_config1_gemm_bit_exact(K, oracle_lib):
    """M=250, K=1024, N=4096, trits P=(.3,.4,.3), scales U(0.01,0.05) (f16), N(0,1)
    activations per-token quantised; both G=128 and G=K=1024."""
    from voxrt_b200 import synth

    rng = np.random.default_rng(1)
    M, Kd, N = 250, 1024, 4096
    for G in (128, 1024):
        mod = synth.ternary_module(rng, N, Kd, G)
        xf = rng.standard_normal((M, Kd)).astype(np.float32)
        _run(K, oracle_lib, mod["qweight"], mod["scales"], N, Kd, G, xf, 0)


def test_large_m_multi_tile(K, oracle_lib):
    """Persistent scheduling over many tiles and a ragged last tile: M=1000, N=1024+64, K=4096."""
    from voxrt_b200 import synth

    rng = np.random.default_rng(7)
    M, Kd, N = 1000, 4096, 1088
    mod = synth.ternary_module(rng, N, Kd, 128)
    xf = rng.standard_normal((M, Kd)).astype(np.float32)
    _run(K, oracle_lib, mod["qweight"], mod["scales"], N, Kd, 128, xf, 2, 0.5,
         y0=rng.standard_normal((M, N)).astype(np.float32), want_sums=False)


@pytest.mark.parametrize("G", [256, 1024])
def test_multi_chunk_groups_many_tiles(K, oracle_lib, G):
    """Groups wider than one 128-column chunk (G = 256, G = K = 1024) with several tiles per CTA (M = 4000,
    N = 1024: 256 tiles over at most 148 CTAs), both weight formats; the scalar-equivalent VNNI oracle is the
    checker."""
    import torch

    from voxrt_b200 import synth
    from voxrt_b200._lib import check_device

    rng = np.random.default_rng(G)
    M, Kd, N = 4000, 1024, 1024
    mod = synth.ternary_module(rng, N, Kd, G)
    w_rows, sw = oracle_lib.unpack_matrix(mod["qweight"], mod["scales"], N, Kd, G)
    xq, sx = oracle_lib.quantize_rows(rng.standard_normal((M, Kd)).astype(np.float32), G)
    want = oracle_lib.Q16(w_rows, sw, G).gemm(xq, sx)
    X = K.QuantAct(torch.from_numpy(xq).cuda(), torch.from_numpy(sx).cuda(), G)
    for fmt in ("2bit", "int8"):
        W = K.TernaryMatrix.from_packed(mod["qweight"], mod["scales"], N, Kd, G, fmt=fmt)
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        K.gemm_ep(W, X, y)
        torch.cuda.synchronize()
        check_device()
        got = y.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), fmt


@pytest.mark.parametrize("M,N,Kd", [(1, 128, 1024), (250, 4096, 1024), (1000, 1024, 4096), (300, 256, 128)])
def test_silu_quant_fused(K, oracle_lib, M, N, Kd):
    """linear1 + Silu + quantize_group(128) fused: int8 codes and scales identical to the Silu GEMM followed by
    the reference quantiser, for both weight formats (resident and streamed slabs)."""
    import torch

    from voxrt_b200 import synth
    from voxrt_b200._lib import check_device

    rng = np.random.default_rng(M + N + Kd)
    mod = synth.ternary_module(rng, N, Kd, 128)
    w_rows, sw = oracle_lib.unpack_matrix(mod["qweight"], mod["scales"], N, Kd, 128)
    xf = (3.0 * rng.standard_normal((M, Kd))).astype(np.float32)
    xq, sx = oracle_lib.quantize_rows(xf, 128)
    h = oracle_lib.gemm(w_rows, sw, xq, sx, 128, 1, 0.0, y=np.zeros((M, N), np.float32))
    want_q, want_s = oracle_lib.quantize_rows(h, 128)
    X = K.QuantAct(torch.from_numpy(xq).cuda(), torch.from_numpy(sx).cuda(), 128)
    for fmt in ("2bit", "int8"):
        W = K.TernaryMatrix.from_packed(mod["qweight"], mod["scales"], N, Kd, 128, fmt=fmt)
        got = K.gemm_silu_quant(W, X)
        torch.cuda.synchronize()
        check_device()
        np.testing.assert_array_equal(got.x.cpu().numpy(), want_q, err_msg=fmt)
        assert np.array_equal(got.scales.cpu().numpy().view(np.uint32), want_s.view(np.uint32)), fmt


def _big_case(oracle_lib, seed, M, N, Kd):
    from voxrt_b200 import synth

    rng = np.random.default_rng(seed)
    mod = synth.ternary_module(rng, N, Kd, 128)
    w_rows, sw = oracle_lib.unpack_matrix(mod["qweight"], mod["scales"], N, Kd, 128)
    xq, sx = oracle_lib.quantize_rows((2.0 * rng.standard_normal((M, Kd))).astype(np.float32), 128)
    y = oracle_lib.Q16(w_rows, sw, 128).gemm(xq, sx)
    return rng, mod, xq, sx, y


def test_qkv_quant_epilogue_many_tiles(K, oracle_lib):
    """The q|k|v projection's quantising epilogue (per-head Qu = quant(q + bias_u), Qv = quant(q + bias_v),
    K = quant(k), v as f32; encoder.rs:349-377) at M = 4000: 32 x 24 tiles over at most 148 CTAs, so every CTA
    walks several tiles, reuses its weight slab across m-tiles and carries TMEM buffer phases from tile to tile."""
    import torch

    from voxrt_b200._lib import check_device

    M, H, Kd = 4000, 8, 1024
    N = 3 * H * 128
    rng, mod, xq, sx, y = _big_case(oracle_lib, 11, M, N, Kd)
    bu = (0.1 * rng.standard_normal((H, 128))).astype(np.float16).astype(np.float32)
    bv = (0.1 * rng.standard_normal((H, 128))).astype(np.float16).astype(np.float32)
    W = K.TernaryMatrix.from_module(mod)
    X = K.QuantAct(torch.from_numpy(xq).cuda(), torch.from_numpy(sx).cuda(), 128)
    qu, squ, qv, sqv, kk, sk, yv = K.gemm_qkv_quant(W, X, H, torch.from_numpy(bu).cuda(), torch.from_numpy(bv).cuda())
    torch.cuda.synchronize()
    check_device()
    d = H * 128
    got_v = yv.cpu().numpy()[:, 2 * d:]
    assert np.array_equal(got_v.view(np.uint32), y[:, 2 * d:].view(np.uint32)), "v columns"
    for h in range(H):
        q = y[:, h * 128:(h + 1) * 128]
        k = y[:, d + h * 128:d + (h + 1) * 128]
        for name, src, codes, scales in (("Qu", q + bu[h], qu, squ), ("Qv", q + bv[h], qv, sqv),
                                         ("K", k, kk, sk)):
            wq, ws = oracle_lib.quantize_rows(np.ascontiguousarray(src, np.float32), 128)
            np.testing.assert_array_equal(codes[h].cpu().numpy(), wq, err_msg=f"{name} head {h}")
            assert np.array_equal(scales[h].cpu().numpy().view(np.uint32), ws[:, 0].view(np.uint32)), (name, h)


def test_glu_epilogue_many_tiles(K, oracle_lib):
    """pointwise_conv1 with the GLU in the epilogue (rows interleaved at load time) at M = 4000, N = 2048: 32 x 16
    tiles, several per CTA. Expected: the Store GEMM in the reference's row order, then a * sigmoid_fast(b)."""
    import torch

    from voxrt_b200 import synth
    from voxrt_b200._lib import check_device

    M, N, Kd = 4000, 2048, 1024
    rng, mod, xq, sx, y = _big_case(oracle_lib, 12, M, N, Kd)
    want = oracle_lib.glu_rows(y)
    order = K.glu_row_order(N)
    assert sorted(order.tolist()) == list(range(N))
    trits = np.stack([oracle_lib.unpack_row(r, Kd) for r in mod["qweight"]])[order]
    perm = {"qweight": synth.pack_trits(trits), "scales": mod["scales"][order], "out": N, "in": Kd, "group": 128}
    W = K.TernaryMatrix.from_module(perm)
    X = K.QuantAct(torch.from_numpy(xq).cuda(), torch.from_numpy(sx).cuda(), 128)
    got = K.gemm_glu(W, X)
    torch.cuda.synchronize()
    check_device()
    got = got.cpu().numpy()
    bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{bad.size} mismatches, first at {np.unravel_index(bad[0], got.shape)}"


def test_silu_quant_epilogue_many_tiles(K, oracle_lib):
    """ff*.linear1's SiLU -> int8 epilogue at the encoder's own row count (M = 12955, N = 4096): 102 x 32 tiles, 22
    per CTA, every CTA crossing weight-slab boundaries."""
    import torch

    from voxrt_b200._lib import check_device

    M, N, Kd = 12955, 4096, 1024
    rng, mod, xq, sx, _ = _big_case(oracle_lib, 13, M, N, Kd)
    w_rows, sw = oracle_lib.unpack_matrix(mod["qweight"], mod["scales"], N, Kd, 128)
    h = oracle_lib.Q16(w_rows, sw, 128).gemm(xq, sx, ep=1)
    want_q, want_s = oracle_lib.quantize_rows(h, 128)
    W = K.TernaryMatrix.from_module(mod)
    X = K.QuantAct(torch.from_numpy(xq).cuda(), torch.from_numpy(sx).cuda(), 128)
    got = K.gemm_silu_quant(W, X)
    torch.cuda.synchronize()
    check_device()
    np.testing.assert_array_equal(got.x.cpu().numpy(), want_q)
    assert np.array_equal(got.scales.cpu().numpy().view(np.uint32), want_s.view(np.uint32))
