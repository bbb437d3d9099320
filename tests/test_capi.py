"""CPU checks of the C ABI boundary: the library loads and exports every function include/vxg.h declares, the
binding declares each with its signature, and host-side helpers behave (no GPU compute)."""
import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "vxg.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vxg_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from voxrt_b200 import _lib

    L = _lib.lib()
    names = _declared()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    unbound = [n for n in names if n not in _lib.SIGNATURES]
    assert not unbound, unbound


def test_errors_are_reported_not_raised():
    from voxrt_b200 import _lib

    L = _lib.lib()
    st = L.vxg_ternary_repack(None, None, 4, 128, 128, None, None)
    assert st == _lib.VXG_ERR_ARG
    assert b"NULL" in L.vxg_last_error()
    q = np.zeros((1, 26), np.uint8)
    s = np.zeros((1, 1), np.uint16)
    codes = np.zeros(4096, np.uint8)
    sc = np.zeros(128, np.float32)
    assert L.vxg_ternary_repack(q.ctypes.data, s.ctypes.data, 1, 130, 128, codes.ctypes.data, sc.ctypes.data) == \
        _lib.VXG_ERR_ARG  # in % 128 != 0
    assert L.vxg_version() == b"0.1.0"


def test_repack_roundtrip_matches_oracle_trits(oracle_lib):
    """The device-format repack (host side) encodes the same trits and scales the oracle unpacks."""
    from voxrt_b200 import _lib, synth

    L = _lib.lib()
    rng = np.random.default_rng(0)
    out, inp = 200, 256
    m = synth.ternary_module(rng, out, inp, 128)
    w8 = np.zeros(L.vxg_ternary_i8_bytes(out, inp), np.int8)
    st = np.zeros(L.vxg_ternary_scales_count(out, inp, 128), np.float32)
    assert L.vxg_ternary_repack_i8(m["qweight"].ctypes.data, m["scales"].ctypes.data, out, inp, 128,
                                   w8.ctypes.data, st.ctypes.data) == 0
    w, sw = oracle_lib.unpack_matrix(m["qweight"], m["scales"], out, inp, 128)
    np.testing.assert_array_equal(w8.reshape(-1, inp)[:out], w)
    pad = L.vxg_ternary_out_pad(out)
    st = st.reshape(pad // 128, inp // 128, 128).transpose(0, 2, 1).reshape(pad, inp // 128)
    assert np.array_equal(st[:out].view(np.uint32), sw.view(np.uint32))
    # 2-bit codes decode to the same trits (code = trit + 1 at the PRMT bit positions)
    codes = np.zeros(L.vxg_ternary_codes_bytes(out, inp), np.uint8)
    assert L.vxg_ternary_repack(m["qweight"].ctypes.data, m["scales"].ctypes.data, out, inp, 128,
                                codes.ctypes.data, st.ctypes.data) == 0
    words = codes.view(np.uint32).reshape(pad // 128, inp // 128, 128, 8)
    pos = [(16 if (e >> 2) & 2 else 0) + (2 if (e >> 2) & 1 else 0) + 4 * (e & 3) for e in range(16)]
    dec = np.zeros((pad, inp), np.int8)
    for e, b in enumerate(pos):
        v = ((words >> b) & 3).astype(np.int8) - 1  # [nt, chunk, row, word]
        for c in range(inp // 128):
            dec.reshape(pad // 128, 128, inp)[:, :, c * 128 + np.arange(8) * 16 + e] = v[:, c]
    np.testing.assert_array_equal(dec[:out], w)
    assert not dec[out:].any()


def test_fold_bn_host(oracle_lib):
    from voxrt_b200 import kernels, synth

    L = synth.layer(1)
    a = kernels.fold_bn(L["dw_weight"], L["bn_w"], L["bn_b"], L["bn_mean"], L["bn_var"])
    b = oracle_lib.fold_bn(L["dw_weight"], L["bn_w"], L["bn_b"], L["bn_mean"], L["bn_var"], 9)
    assert np.array_equal(a[0].view(np.uint32), b[0].view(np.uint32))
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))


def test_out_frames_matches_reference_formula(oracle_lib):
    from voxrt_b200 import _lib, synth

    for t in (1, 2, 8, 9, 17, 100, 3001):
        assert _lib.lib().vxg_sub_out_frames(t) == oracle_lib.lib().vxo_sub_out_frames(t, 3, 2) == synth.out_frames(t)
