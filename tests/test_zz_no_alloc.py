"""GPU: the allocation-free conv-module entry (static device index table, for callers that cannot allocate device
memory while they run) against the workspace entry, through the C ABI, on two calls in a row with different batches,
for both conv kernels and at the table's size limit. The tolerance is the conv tests' own: bit-identical."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(lib, fn, g, offs, lens, dw_t, dw_b, torch, workspace):
    rows, ld = g.shape
    k, d = dw_t.shape
    hb = torch.full((rows, d), float("nan"), dtype=torch.float32, device=g.device)
    q = torch.zeros((rows, d), dtype=torch.int8, device=g.device)
    s = torch.zeros((rows, d // 128), dtype=torch.float32, device=g.device)
    off = np.ascontiguousarray(offs, np.int32)
    ln = np.ascontiguousarray(lens, np.int32)
    P = lambda t: C.c_void_p(t.data_ptr())
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if workspace:
        nb = lib.vxg_conv_workspace_bytes(rows, len(ln))
        ws = torch.empty(nb, dtype=torch.uint8, device=g.device)
        st = lib.vxg_conv_glu_dw_silu_quant(P(g), ld, off.ctypes.data, ln.ctypes.data, len(ln), P(dw_t), P(dw_b), d,
                                            k, P(hb), P(q), P(s), P(ws), nb, stream)
    else:
        st = lib.vxg_conv_glu_dw_silu_quant_static(P(g), ld, off.ctypes.data, ln.ctypes.data, len(ln), P(dw_t),
                                                   P(dw_b), d, k, P(hb), P(q), P(s), stream)
    torch.cuda.synchronize()
    return st, hb.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy()


def _check_pair(L, g, lens, dw_t, dw_b, torch):
    from voxrt_b200._lib import VXG_OK, check_device

    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int32)
    st0, hb0, q0, s0 = _run(L, None, g, offs, lens, dw_t, dw_b, torch, workspace=True)
    st1, hb1, q1, s1 = _run(L, None, g, offs, lens, dw_t, dw_b, torch, workspace=False)
    check_device()
    assert st0 == VXG_OK and st1 == VXG_OK, (st0, st1, L.vxg_last_error())
    assert np.array_equal(hb1.view(np.uint32), hb0.view(np.uint32)), len(lens)
    np.testing.assert_array_equal(q1, q0)
    assert np.array_equal(s1.view(np.uint32), s0.view(np.uint32)), len(lens)


def _dw(torch, seed, k):
    from voxrt_b200 import kernels, synth

    lw = synth.layer(seed, k=k)
    dw_t, dw_b = kernels.fold_bn(lw["dw_weight"], lw["bn_w"], lw["bn_b"], lw["bn_mean"], lw["bn_var"])
    return torch.from_numpy(dw_t).cuda(), torch.from_numpy(dw_b).cuda()


def test_static_entry_matches_workspace_entry():
    """Two calls in a row with different batches (the second must not see the first's tables), for the specialised
    9-tap kernel and for the generic kernel at k = 5 and k = 15."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voxrt_b200._lib import lib

    L = lib()
    rng = np.random.default_rng(7)
    for k in (9, 5, 15):
        dw_t, dw_b = _dw(torch, 4 + k, k)
        d = dw_t.shape[1]
        for lens in ([375, 3, 130, 64, 7], [200, 1, 65, 1000]):
            g = torch.from_numpy((2.0 * rng.standard_normal((sum(lens), 2 * d))).astype(np.float32)).cuda()
            _check_pair(L, g, lens, dw_t, dw_b, torch)


def test_static_entry_at_the_table_limit():
    """A batch whose tables need exactly the 16384 entries of the static array: 1000 utterances (the most the entry
    takes) with 7192 row tiles of 64 (each utterance's last tile one row long)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voxrt_b200._lib import lib

    L = lib()
    lens = [64 * 7 + 1] * 192 + [64 * 6 + 1] * 808
    tiles = sum((t + 63) // 64 for t in lens)
    assert 2 * len(lens) + 2 * tiles == 16384
    dw_t, dw_b = _dw(torch, 21, 9)
    d = dw_t.shape[1]
    torch.manual_seed(0)
    g = 2.0 * torch.randn((sum(lens), 2 * d), dtype=torch.float32, device="cuda")
    _check_pair(L, g, lens, dw_t, dw_b, torch)


def test_static_entry_rejects_oversized_batch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from voxrt_b200._lib import VXG_ERR_ARG, lib

    L = lib()
    dummy = torch.empty(16, dtype=torch.float32, device="cuda")
    P = C.c_void_p(dummy.data_ptr())
    # no output pointers: even if the size checks let a batch through, the call would stop before any launch
    lens = np.full(999, 64 * 8, np.int32)  # 2 * 999 + 2 * 999 * 8 entries > 16384
    offs = (np.arange(999) * 512).astype(np.int32)
    st = L.vxg_conv_glu_dw_silu_quant_static(P, 2048, offs.ctypes.data, lens.ctypes.data, len(lens), P, P, 1024, 9,
                                             None, None, None, None)
    assert st == VXG_ERR_ARG
    assert "static table holds 16384" in L.vxg_last_error().decode()
    lens = np.full(1001, 1, np.int32)  # more utterances than the build kernel's parameters carry
    offs = np.arange(1001, dtype=np.int32)
    st = L.vxg_conv_glu_dw_silu_quant_static(P, 2048, offs.ctypes.data, lens.ctypes.data, len(lens), P, P, 1024, 9,
                                             None, None, None, None)
    assert st == VXG_ERR_ARG
    assert "at most 1000" in L.vxg_last_error().decode()
