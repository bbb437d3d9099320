"""CPU tests: pin the oracle against the reference's golden vectors and known answers, and check the restated x86
baseline kernels against the scalar oracle on the reference's own test lists (no GPU needed)."""
import json
import os

import numpy as np
import pytest

from conftest import LCG
from refgen import acts_f32, random_matrix, x86_int8, x86_ternary

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


# ------------------------------------------------------------------------------------------------- codec

def test_codec_matches_reference_fixtures(oracle_lib):
    """tests/fixtures_trits.rs:13-47 on the reference's real-weight fixture rows: trits and dequant exact."""
    o = oracle_lib
    meta = json.load(open(os.path.join(GOLD, "ternary_fixtures.json")))
    assert len(meta) == 3
    for tag, m in meta.items():
        rows, inf, g = m["rows"], m["in_features"], m["group_size"]
        q = np.fromfile(os.path.join(GOLD, f"{tag}.qweight.bin"), np.uint8).reshape(rows, -1)
        s = np.fromfile(os.path.join(GOLD, f"{tag}.scales.f16.bin"), np.uint16).reshape(rows, -1)
        want_t = np.fromfile(os.path.join(GOLD, f"{tag}.trits.i8.bin"), np.int8).reshape(rows, inf)
        want_w = np.fromfile(os.path.join(GOLD, f"{tag}.weight.f32.bin"), "<f4").reshape(rows, inf)
        w, sc = o.unpack_matrix(q, s, rows, inf, g)
        np.testing.assert_array_equal(w, want_t, err_msg=tag)
        deq = w.astype(np.float32) * np.repeat(sc, g, axis=1)
        assert np.array_equal(deq.view(np.uint32), want_w.view(np.uint32)), tag
        zf = float(np.mean(w == 0))
        assert abs(zf - m["zero_fraction_rows"]) < 1e-9


def test_codec_matches_reference_python_codec(oracle_lib):
    """Vectors from the reference's reference-py/trits.py (pack / unpack / dequant), ragged widths."""
    o = oracle_lib
    v = np.load(os.path.join(GOLD, "codec_vectors.npz"))
    for n in (1, 4, 5, 6, 127, 128, 1024, 4096):
        t, q = v[f"pack_in_{n}"], v[f"pack_out_{n}"]
        for r in range(t.shape[0]):
            np.testing.assert_array_equal(o.pack_row(t[r]), q[r])
            np.testing.assert_array_equal(o.unpack_row(q[r], n), v[f"unpack_{n}"][r])
    w, s = o.unpack_matrix(v["dequant_q"], v["dequant_s"], 5, 256, 128)
    deq = w.astype(np.float32) * np.repeat(s, 128, axis=1)
    assert np.array_equal(deq.view(np.uint32), v["dequant_w"].astype(np.float32).view(np.uint32))


def test_codec_lsd_first_kat(oracle_lib):
    """trits.rs:103-109: byte 196 -> [0, 1, -1, 0, 1]."""
    np.testing.assert_array_equal(oracle_lib.unpack_row(np.array([196], np.uint8), 5), [0, 1, -1, 0, 1])


def test_synth_packer_matches_oracle_codec(oracle_lib):
    """The product-side synthetic packer (numpy) agrees with the restated pack_row on ragged widths."""
    from voxrt_b200.synth import pack_trits

    rng = np.random.default_rng(1)
    for n in (1, 4, 5, 6, 127, 128, 1024):
        t = rng.integers(-1, 2, size=(3, n), dtype=np.int8)
        q = pack_trits(t)
        for r in range(3):
            np.testing.assert_array_equal(q[r], oracle_lib.pack_row(t[r]))
            np.testing.assert_array_equal(oracle_lib.unpack_row(q[r], n), t[r])


def test_f16_conversion_exact(oracle_lib):
    bits = np.arange(0, 65536, 7, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle_lib.f16_to_f32(b) for b in bits], np.float32)
    fin = np.isfinite(want)
    assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))


# ------------------------------------------------------------------------------------------ quantisation

def _quant_numpy(src):
    """Independent numpy statement of quantize_group_portable (packed.rs:527-535)."""
    src = np.asarray(src, np.float32)
    amax = np.float32(np.max(np.abs(src))) if len(src) else np.float32(0)
    s = np.float32(1.0) if amax == 0 else np.float32(amax / np.float32(127.0))
    inv = np.float32(np.float32(1.0) / s)
    q = np.clip(np.rint(src * inv), -127, 127).astype(np.int8)
    return s, q


def test_quantizer_ties_and_sizes(oracle_lib):
    """packed.rs:606-630: inputs with exact .5 ties after scaling, sizes 1..4096."""
    seed = 3
    for n in (1, 7, 8, 15, 16, 17, 128, 133, 384, 4096):
        src = []
        for i in range(n):
            seed = (seed * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
            if i % 5 == 0:
                src.append(np.float32(np.float32(i) + np.float32(0.5)) * np.float32(0.1))
            else:
                src.append(np.float32(seed >> 40) / np.float32(1e6) - np.float32(8.0))
        src = np.array(src, np.float32)
        s, q = oracle_lib.quantize_group(src)
        s2, q2 = _quant_numpy(src)
        assert np.float32(s).view(np.uint32) == s2.view(np.uint32)
        np.testing.assert_array_equal(q, q2)
    s, q = oracle_lib.quantize_group(np.zeros(128, np.float32))
    assert s == 1.0 and not q.any()


# --------------------------------------------------------------------------------------------- f32 math

def test_exp_poly_error_bound(oracle_lib):
    """tensor.rs:1017-1030: within 3e-7 relative of f64 exp after the [-87, 88] clamp."""
    xs = [i * np.float32(0.05) for i in range(-2000, 2000)] + [-87.0, -100.0, 88.0, 1e3, 0.0, -0.0]
    for x in xs:
        x = np.float32(x)
        got = float(oracle_lib.exp_poly(x))
        want = np.exp(float(np.clip(x, -87.0, 88.0)))
        assert abs((got - want) / want) < 3e-7, x


def test_softmax_tolerance(oracle_lib):
    """tensor.rs:1051-1079 with the portable row: |p - p_f64| <= 2e-6 + 4e-6 |p|."""
    seed = 1
    for n in (1, 3, 4, 7, 64, 333):
        x = []
        for _ in range(n):
            seed = (seed * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
            x.append(np.float32((seed >> 33) % 20001) / np.float32(100.0) - np.float32(100.0))
        x = np.array(x, np.float32)
        e, s = oracle_lib.exp_row_scaled(x, 0.0884)
        got = e * (np.float32(1.0) / s)
        mx = np.max(x * np.float32(0.0884))
        ef = np.exp((x * np.float32(0.0884) - mx).astype(np.float64))
        want = (ef / ef.sum()).astype(np.float32)
        assert np.all(np.abs(got - want) <= 2e-6 + np.abs(want) * 4e-6)


# ------------------------------------------------------------------------------------------------- GEMM

def test_accumulation_cannot_overflow(oracle_lib):
    """kernels.rs:176-200: all trits +1, x = 127, scale 1 -> y = 4096 * 127 exactly."""
    o = oracle_lib
    inp = 4096
    w = np.ones((1, inp), np.int8)
    sw = np.ones((1, inp // 128), np.float32)
    xq, sx = o.quantize_rows(np.full((1, inp), 127.0, np.float32))
    y = o.gemm(w, sw, xq, sx, 128)
    assert y[0, 0] == np.float32(inp * 127)
    if o.cpu_has_vnni():
        assert o.Q16(w, sw, 128).gemm(xq, sx)[0, 0] == np.float32(inp * 127)


def test_quantised_path_tracks_f32_path(oracle_lib):
    """kernels.rs:149-174: int8 per-group-128 vs the dequantised f32 linear, relative error < 1e-2."""
    o = oracle_lib
    rng = LCG(7)
    q, s16, trits = random_matrix(256, 1024, rng)
    w, sw = o.unpack_matrix(q, s16, 256, 1024, 128)
    wf = w.astype(np.float32) * np.repeat(sw, 128, axis=1)
    x = acts_f32(16, 1024, rng, div=1000.0, off=1.0)
    yf = o.linear(x, wf)
    xq, sx = o.quantize_rows(x)
    yq = o.gemm(w, sw, xq, sx, 128)
    assert np.max(np.abs(yf - yq)) / np.max(np.abs(yf)) < 1e-2


def _check_ranges(o, name, W, w_rows, sw, x, sx, group, rng):
    """x86_kernels.rs:90-124: partial row/token ranges x 3 epilogues, bit for bit vs the scalar oracle."""
    out, n = w_rows.shape[0], x.shape[0]
    ranges = [(0, out, 0, n), (min(1, out), out, 0, n), (0, min(out, 17), n // 2, n),
              (out // 3, out - out // 4, 0, (n + 1) // 2)]
    for ep, es in ((o.EP_STORE, 0.0), (o.EP_SILU, 0.0), (o.EP_ADD_SCALED, 0.37)):
        for r0, r1, t0, t1 in ranges:
            if r0 >= r1 or t0 >= t1:
                continue
            init = np.array([np.float32(rng.next() % 100) * np.float32(0.01) for _ in range(n * out)],
                            np.float32).reshape(n, out)
            want = o.gemm(w_rows, sw, x, sx, group, ep, es, y=init, rows=(r0, r1), toks=(t0, t1))
            got = W.gemm_range(x, sx, init.copy(), r0, r1, t0, t1, ep, es)
            assert np.array_equal(want.view(np.uint32), got.view(np.uint32)), (name, out, n, r0, r1, t0, t1, ep)


def _kernels(o):
    ks = []
    if o.cpu_has_avx2():
        ks.append(("avx2", 1))
    if o.cpu_has_vnni():
        ks.append(("vnni", 2))
    return ks


def test_x86_ternary_equals_scalar_exactly(oracle_lib):
    """x86_kernels.rs:140-152."""
    o = oracle_lib
    ks = _kernels(o)
    if not ks:
        pytest.skip("no AVX2/VNNI")
    rng = LCG(3)
    try:
        for name, k in ks:
            o.force_kernel(k)
            for out, inp in ((7, 128), (16, 256), (33, 1024), (130, 4096)):
                trits, sw, _ = x86_ternary(out, inp, rng)
                W = o.Q16(trits, sw, 128, ternary=True)
                for n in (1, 2, 3, 4, 5, 8, 9, 17):
                    xq, sx = o.quantize_rows(acts_f32(n, inp, rng), 128)
                    _check_ranges(o, name, W, trits, sw, xq, sx, 128, rng)
    finally:
        o.force_kernel(-1)


def test_x86_int8_equals_scalar_exactly(oracle_lib):
    """x86_kernels.rs:154-172: arbitrary int8 weights, groups 128 / 384 / 1024."""
    o = oracle_lib
    ks = _kernels(o)
    if not ks:
        pytest.skip("no AVX2/VNNI")
    rng = LCG(5)
    try:
        for name, k in ks:
            o.force_kernel(k)
            for out, inp, group in ((7, 128, 128), (40, 640, 128), (128, 384, 384), (19, 1024, 1024)):
                rows, sw = x86_int8(out, inp, group, rng)
                W = o.Q16(rows, sw, group, ternary=False)
                for n in (1, 2, 5, 8, 11):
                    xq, sx = o.quantize_rows(acts_f32(n, inp, rng), group)
                    _check_ranges(o, name, W, rows, sw, xq, sx, group, rng)
    finally:
        o.force_kernel(-1)


def test_x86_extremes_do_not_saturate(oracle_lib):
    """x86_kernels.rs:174-185."""
    o = oracle_lib
    ks = _kernels(o)
    if not ks:
        pytest.skip("no AVX2/VNNI")
    rng = LCG(9)
    try:
        for name, k in ks:
            o.force_kernel(k)
            trits, sw, _ = x86_ternary(32, 1024, rng, extreme=True)
            xq, sx = o.quantize_rows(acts_f32(5, 1024, rng, extreme=True), 128)
            _check_ranges(o, name, o.Q16(trits, sw, 128, True), trits, sw, xq, sx, 128, rng)
            rows, sw = x86_int8(32, 1024, 1024, rng, extreme=True)
            xq, sx = o.quantize_rows(acts_f32(5, 1024, rng, extreme=True), 1024)
            _check_ranges(o, name, o.Q16(rows, sw, 1024, False), rows, sw, xq, sx, 1024, rng)
    finally:
        o.force_kernel(-1)


def test_ln_quant_matches_unfused(oracle_lib):
    """prepare_normed == layer_norm_row then quantize (ternary_linear.rs:132-158)."""
    o = oracle_lib
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 1024)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.1 * rng.standard_normal(1024)).astype(np.float32)
    q, s = o.ln_quant_rows(x, g, b)
    for t in range(5):
        y = o.layer_norm_row(x[t], g, b)
        q2, s2 = o.quantize_rows(y[None], 128)
        np.testing.assert_array_equal(q[t], q2[0])
        assert np.array_equal(s[t].view(np.uint32), s2[0].view(np.uint32))


def test_layer_forward_runs_and_is_thread_invariant(oracle_lib):
    """One int8 layer at a small T is finite and does not depend on the oracle's thread count."""
    o = oracle_lib
    from voxrt_b200 import synth

    L = o.OracleLayer(synth.layer(2))
    rng = np.random.default_rng(2)
    t = 37
    x = rng.standard_normal((t, 1024)).astype(np.float32)
    pos = o.rel_pos_table(t)
    n0 = o.get_threads()
    try:
        o.set_threads(1)
        a = L.forward(x, pos)
        o.set_threads(4)
        b = L.forward(x, pos)
    finally:
        o.set_threads(n0 if n0 else 0)
    assert np.isfinite(a).all()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
