"""GPU parity: int8 relative-position attention against the oracle's attn_core_int8, bit for bit, for single
utterances of ragged lengths and for batches of stacked utterances sharing one relative table."""
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


def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def _case(K, oracle, lengths, tmax=None, seed=0, scale=1.0):
    import torch

    from voxrt_b200._lib import check_device

    rng = np.random.default_rng(seed)
    H, d = 8, 1024
    tmax = tmax or max(lengths)
    rows = int(sum(lengths))
    offs = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
    qkv = (rng.standard_normal((rows, 3 * d)) * scale).astype(np.float32)
    rel = rng.standard_normal((2 * tmax - 1, d)).astype(np.float32)
    bu, bv = _f16(0.1 * rng.standard_normal((H, 128))), _f16(0.1 * rng.standard_normal((H, 128)))
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ctx, cq = K.attention_i8(T(qkv), T(rel), tmax, offs, lengths, T(bu), T(bv), H)
    check_device()
    got = ctx.cpu().numpy()
    gq, gs = cq.x.cpu().numpy(), cq.scales.cpu().numpy()
    for u, (o, t) in enumerate(zip(offs, lengths)):
        rk = rel[tmax - t: tmax + t - 1]
        want = oracle.attn_core_int8(qkv[o:o + t], rk, t, bu, bv)
        g = got[o:o + t]
        bad = np.flatnonzero(g.view(np.uint32) != want.view(np.uint32))
        assert bad.size == 0, f"utt {u} (t={t}): {bad.size} mismatches, first {np.unravel_index(bad[0], g.shape)}" \
                              f" {g.flat[bad[0]]} vs {want.flat[bad[0]]}"
        wq, ws = oracle.quantize_rows(want, 128)
        np.testing.assert_array_equal(gq[o:o + t], wq)
        assert np.array_equal(gs[o:o + t].view(np.uint32), ws.view(np.uint32))


@pytest.mark.parametrize("t", [1, 2, 5, 37, 128, 129, 300, 375])
def test_single_utterance(K, oracle_lib, t):
    _case(K, oracle_lib, [t], seed=t)


def test_batch_shared_rel_table(K, oracle_lib):
    _case(K, oracle_lib, [375, 17, 200, 128, 259, 1, 64], seed=11)


def test_rel_table_longer_than_batch(K, oracle_lib):
    _case(K, oracle_lib, [100, 33], tmax=300, seed=12)


def test_large_scores(K, oracle_lib):
    """Peaked softmax rows (large-magnitude q/k) still match bit for bit."""
    _case(K, oracle_lib, [150, 90], seed=13, scale=6.0)


def _long_case(K, oracle, t, n_utt, seed, blocks=None):
    """8 heads x 128, utterances of t frames stacked (batch n_utt), per-token-quantised N(0, 1)
    q/k/v, rel_k N(0, 1) [2t-1, 1024], bias_u / bias_v as config 2. With `blocks`, only those 8-row query blocks of
    every utterance are checked (rows are independent given the per-head operands, which the oracle still quantises
    over all frames)."""
    import torch

    from voxrt_b200._lib import check_device

    rng = np.random.default_rng(seed)
    H, d = 8, 1024
    lengths = [t] * n_utt
    offs = np.arange(n_utt, dtype=np.int32) * t
    qkv = rng.standard_normal((t * n_utt, 3 * d), dtype=np.float32)
    rel = rng.standard_normal((2 * t - 1, d), dtype=np.float32)
    bu, bv = _f16(0.1 * rng.standard_normal((H, 128))), _f16(0.1 * rng.standard_normal((H, 128)))
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ctx, _ = K.attention_i8(T(qkv), T(rel), t, offs, lengths, T(bu), T(bv), H)
    check_device()
    got = ctx.cpu().numpy()
    for u in range(n_utt):
        q = qkv[u * t:(u + 1) * t]
        if blocks is None:
            want = oracle.attn_core_int8(q, rel, t, bu, bv)
            rows = np.arange(t)
        else:
            want = oracle.attn_core_int8_rows(q, rel, t, bu, bv, blocks)
            rows = np.concatenate([np.arange(8 * b, min(t, 8 * b + 8)) for b in blocks])
        g, w = got[u * t + rows], want[rows]
        bad = np.flatnonzero(g.view(np.uint32) != w.view(np.uint32))
        assert bad.size == 0, f"utt {u} (t={t}): {bad.size} mismatches, first row {rows[bad[0] // d]}"


def test_long_form_t1500_batch8(K, oracle_lib):
    """Config 4, T = 1500 (2 min), batch 8: every row of every utterance."""
    _long_case(K, oracle_lib, 1500, 8, seed=41)


def test_long_form_t7500_batch8_sampled_rows(K, oracle_lib):
    """Config 4, T = 7500 (10 min), batch 8: 1024 sampled query rows per utterance (128 blocks of 8, always
    including the first and the last block)."""
    nb = (7500 + 7) // 8
    blocks = np.unique(np.concatenate([[0, nb - 1], np.random.default_rng(42).choice(nb, 126, replace=False)]))
    _long_case(K, oracle_lib, 7500, 8, seed=42, blocks=blocks)
