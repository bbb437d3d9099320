"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against, and the timed CPU baseline. Only the
test suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this module; the product
package ``voxrt_b200`` never does. See oracle/oracle.h for what each function restates and how it is pinned.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

EP_STORE, EP_SILU, EP_ADD_SCALED = 0, 1, 2


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (g++ only)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_P = C.c_void_p
_I = C.c_int
_F = C.c_float


def _declare(L):
    sig = {
        "vxo_unpack_row": (None, [_P, _I, _P]),
        "vxo_pack_row": (None, [_P, _I, _P]),
        "vxo_f16_to_f32": (_F, [C.c_uint16]),
        "vxo_unpack_matrix": (None, [_P, _P, _I, _I, _I, _P, _P]),
        "vxo_quantize_group": (_F, [_P, _I, _P]),
        "vxo_quantize_rows": (None, [_P, _I, _I, _I, _P, _P]),
        "vxo_layer_norm_row": (None, [_P, _P, _P, _I, _P]),
        "vxo_ln_quant_rows": (None, [_P, _I, _I, _P, _P, _I, _P, _P]),
        "vxo_gemm": (None, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _I, _I, _I, _I]),
        "vxo_exp_poly": (_F, [_F]),
        "vxo_silu_fast": (_F, [_F]),
        "vxo_sigmoid_fast": (_F, [_F]),
        "vxo_glu_rows": (None, [_P, _I, _I, _P]),
        "vxo_vad_probs": (None, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _F, _P]),
        "vxo_segment": (_I, [_P, _I, _F, _I, _I, _I, _I, _P, _I]),
        "vxo_math_cr": (None, [_I, _P, C.c_size_t, _P]),
        "vxo_exp_row_scaled": (_F, [_P, _I, _F]),
        "vxo_linear": (None, [_P, _I, _I, _P, _P, _I, _P]),
        "vxo_rel_pos_table": (None, [_I, _I, _P]),
        "vxo_fold_bn": (None, [_P, _P, _P, _P, _P, _I, _I, _P, _P]),
        "vxo_attn_core_int8": (None, [_P, _P, _I, _I, _I, _I, _P, _P, _F, _P]),
        "vxo_attn_core_int8_rows": (None, [_P, _P, _I, _I, _I, _I, _P, _P, _F, _P, _P, _I]),
        "vxo_conv_middle": (None, [_P, _I, _I, _I, _P, _P, _P]),
        "vxo_layer_forward": (None, [_P, _I, _I, _I, _P, _I, _P]),
        "vxo_layer_prepare": (_P, [_P]),
        "vxo_layer_free": (None, [_P]),
        "vxo_layer_forward_prepared": (None, [_P, _P, _I, _I, _I, _P, _I, _P]),
        "vxo_sub_out_frames": (_I, [_I, _I, _I]),
        "vxo_subsampling_forward": (None, [_P, _P, _I, _P]),
        "vxo_set_threads": (None, [_I]),
        "vxo_get_threads": (_I, []),
        "vxo_q16_prepare": (_P, [_P, _P, _I, _I, _I, _I]),
        "vxo_q16_free": (None, [_P]),
        "vxo_q16_gemm": (None, [_P, _P, _P, _I, _I, _F, _P, _P]),
        "vxo_q16_gemm_range": (None, [_P, _P, _P, _I, _I, _F, _P, _I, _I, _I, _I]),
        "vxo_q16_bench_range": (C.c_double, [_P, _P, _P, _I, _P, _I, _I]),
        "vxo_force_kernel": (_I, [_I]),
        "vxo_cpu_has_vnni": (_I, []),
        "vxo_cpu_has_avx2": (_I, []),
        "vxo_tdt_int8_rows": (None, [_P, _I, _I, _P, _P]),
        "vxo_tdt_pred_step": (None, [_P, _I, _P, _P, _P, _P, _P]),
        "vxo_tdt_joint": (None, [_P, _P, _P, _P]),
        "vxo_tdt_project": (None, [_P, _P, _I, _P]),
        "vxo_tdt_greedy": (_I, [_P, _P, _I, _P, _P, _P, _I]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def _p(a):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------------------------------------- codec

def unpack_row(packed, in_features):
    packed = _c(packed, np.uint8)
    out = np.empty(in_features, np.int8)
    lib().vxo_unpack_row(_p(packed), in_features, _p(out))
    return out


def pack_row(trits):
    trits = _c(trits, np.int8)
    out = np.empty((len(trits) + 4) // 5, np.uint8)
    lib().vxo_pack_row(_p(trits), len(trits), _p(out))
    return out


def pack_matrix(trits):
    trits = _c(trits, np.int8)
    out, n = trits.shape
    q = np.empty((out, (n + 4) // 5), np.uint8)
    for r in range(out):
        q[r] = pack_row(trits[r])
    return q


def f16_to_f32(h):
    return lib().vxo_f16_to_f32(int(h))


def unpack_matrix(qweight, scales_f16, out, inp, group):
    """thrush-ternary-v2 -> (int8 rows [out, inp], f32 scales [out, inp/group])."""
    qweight = _c(qweight, np.uint8)
    scales_f16 = _c(scales_f16, np.uint16)
    w = np.empty((out, inp), np.int8)
    s = np.empty((out, inp // group), np.float32)
    lib().vxo_unpack_matrix(_p(qweight), _p(scales_f16), out, inp, group, _p(w), _p(s))
    return w, s


# ------------------------------------------------------------------------------------------ quantisation

def quantize_group(src):
    src = _c(src, np.float32)
    dst = np.empty(len(src), np.int8)
    s = lib().vxo_quantize_group(_p(src), len(src), _p(dst))
    return np.float32(s), dst


def quantize_rows(x, group=128):
    x = _c(x, np.float32)
    n, inp = x.shape
    q = np.empty((n, inp), np.int8)
    s = np.empty((n, inp // group), np.float32)
    lib().vxo_quantize_rows(_p(x), n, inp, group, _p(q), _p(s))
    return q, s


def layer_norm_row(x, g, b):
    x, g, b = _c(x, np.float32), _c(g, np.float32), _c(b, np.float32)
    y = np.empty_like(x)
    lib().vxo_layer_norm_row(_p(x), _p(g), _p(b), len(x), _p(y))
    return y


def ln_quant_rows(x, g, b, group=128):
    x, g, b = _c(x, np.float32), _c(g, np.float32), _c(b, np.float32)
    n, d = x.shape
    q = np.empty((n, d), np.int8)
    s = np.empty((n, d // group), np.float32)
    lib().vxo_ln_quant_rows(_p(x), n, d, _p(g), _p(b), group, _p(q), _p(s))
    return q, s


# -------------------------------------------------------------------------------------------------- GEMM

def gemm(w, sw, x, sx, group, ep=EP_STORE, ep_scale=0.0, y=None, bias=None, want_sums=False, rows=None, toks=None):
    """Scalar reference GEMM (gemm_scalar_range). Returns y (and the int32 group sums [M, N, K/G])."""
    w, sw, x, sx = _c(w, np.int8), _c(sw, np.float32), _c(x, np.int8), _c(sx, np.float32)
    N, K = w.shape
    M = x.shape[0]
    y = np.zeros((M, N), np.float32) if y is None else _c(y, np.float32).copy()
    sums = np.zeros((M, N, K // group), np.int32) if want_sums else None
    r0, r1 = rows if rows else (0, N)
    t0, t1 = toks if toks else (0, M)
    bias = None if bias is None else _c(bias, np.float32)
    lib().vxo_gemm(_p(w), _p(sw), _p(x), _p(sx), M, N, K, group, ep, float(ep_scale), _p(bias), _p(y), _p(sums),
                   r0, r1, t0, t1)
    return (y, sums) if want_sums else y


class Q16:
    """Quad16 weights for the restated x86 kernels (the timed CPU baseline)."""

    def __init__(self, w, sw, group, ternary=True):
        self._w = _c(w, np.int8)
        self._s = _c(sw, np.float32)
        self.out, self.inp = self._w.shape
        self.group = group
        self.h = lib().vxo_q16_prepare(_p(self._w), _p(self._s), self.out, self.inp, group, int(ternary))

    def gemm(self, x, sx, ep=EP_STORE, ep_scale=0.0, y=None, bias=None):
        x, sx = _c(x, np.int8), _c(sx, np.float32)
        n = x.shape[0]
        y = np.zeros((n, self.out), np.float32) if y is None else y
        bias = None if bias is None else _c(bias, np.float32)
        lib().vxo_q16_gemm(self.h, _p(x), _p(sx), n, ep, float(ep_scale), _p(bias), _p(y))
        return y

    def gemm_range(self, x, sx, y, r0, r1, t0, t1, ep=EP_STORE, ep_scale=0.0):
        x, sx = _c(x, np.int8), _c(sx, np.float32)
        lib().vxo_q16_gemm_range(self.h, _p(x), _p(sx), x.shape[0], ep, float(ep_scale), _p(y), r0, r1, t0, t1)
        return y

    def bench_range(self, x, sx, rows, reps=5):
        """Best-of-`reps` seconds of the selected x86 kernel, single-threaded, on weight rows [0, rows) x all tokens
        (x86_bench.rs:31-71)."""
        x, sx = _c(x, np.int8), _c(sx, np.float32)
        y = np.zeros((x.shape[0], self.out), np.float32)
        return lib().vxo_q16_bench_range(self.h, _p(x), _p(sx), x.shape[0], _p(y), rows, reps)

    def __del__(self):
        try:
            lib().vxo_q16_free(self.h)
        except Exception:
            pass


def force_kernel(k: int) -> int:
    """-1 auto, 0 scalar, 1 AVX2, 2 AVX-512 VNNI; returns the kernel that will run."""
    return lib().vxo_force_kernel(k)


def cpu_info() -> dict:
    """The host CPU as the baselines report it: model string, logical CPUs, physical cores, VNNI / AVX2 support."""
    import os

    model, cores = "unknown", set()
    phys = core = None
    try:
        for line in open("/proc/cpuinfo"):
            k, _, v = line.partition(":")
            k, v = k.strip(), v.strip()
            if k == "model name" and model == "unknown":
                model = v
            elif k == "physical id":
                phys = v
            elif k == "core id":
                core = v
            elif not k and phys is not None and core is not None:
                cores.add((phys, core))
                phys = core = None
        if phys is not None and core is not None:
            cores.add((phys, core))
    except OSError:
        pass
    return {"cpu_model": model, "logical_cpus": os.cpu_count(), "physical_cores": len(cores) or None,
            "avx512_vnni": cpu_has_vnni(), "avx2": cpu_has_avx2()}


def cpu_has_vnni() -> bool:
    return bool(lib().vxo_cpu_has_vnni())


def cpu_has_avx2() -> bool:
    return bool(lib().vxo_cpu_has_avx2())


def set_threads(n: int):
    lib().vxo_set_threads(n)


def get_threads() -> int:
    return lib().vxo_get_threads()


# --------------------------------------------------------------------------------------------- f32 math

def exp_poly(x):
    return np.float32(lib().vxo_exp_poly(float(x)))


def silu_fast(x):
    return np.float32(lib().vxo_silu_fast(float(x)))


def sigmoid_fast(x):
    return np.float32(lib().vxo_sigmoid_fast(float(x)))


def math_cr(fn, x):
    """Correctly rounded f32 exp (fn 0) / tanh (fn 1) by extended-precision evaluation."""
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().vxo_math_cr(fn, _p(x), x.size, _p(y))
    return y


def vad_probs(sub, w):
    """VadHead::probs (vad.rs:39-82) for one utterance: sub [t, d] -> p [t]. w: proj_w [h, d], proj_b [h],
    ctx_w [h, h, k], ctx_b [h], out_w [h], out_b (float)."""
    sub = _c(sub, np.float32)
    t, d = sub.shape
    pw, pb = _c(w["proj_w"], np.float32).reshape(-1, d), _c(w["proj_b"], np.float32)
    h = pw.shape[0]
    cw, cb, ow = _c(w["ctx_w"], np.float32), _c(w["ctx_b"], np.float32), _c(w["out_w"], np.float32).reshape(h)
    k = cw.size // (h * h)
    p = np.empty(t, np.float32)
    lib().vxo_vad_probs(_p(sub), t, d, h, k, _p(pw), _p(pb), _p(cw), _p(cb), _p(ow), float(w["out_b"]), _p(p))
    return p


SEGMENT_DEFAULTS = {"threshold": 0.5, "min_pause_frames": 8, "max_frames": 750, "min_frames": 125, "pad_frames": 2}


def segment(p, cfg=None):
    """segment (vad.rs:140-240): list of (start, end) encoder-frame pairs."""
    c = dict(SEGMENT_DEFAULTS, **(cfg or {}))
    p = _c(p, np.float32)
    cap = max(1, p.size + 1)
    out = np.empty(2 * cap, np.int32)
    n = lib().vxo_segment(_p(p), p.size, float(np.float32(c["threshold"])), c["min_pause_frames"], c["max_frames"],
                          c["min_frames"], c["pad_frames"], _p(out), cap)
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(n)]


def glu_rows(g):
    """glu_row_portable (tensor.rs:917-924) over every row of g [n, 2d] -> [n, d]."""
    g = _c(g, np.float32)
    n, d2 = g.shape
    out = np.empty((n, d2 // 2), np.float32)
    lib().vxo_glu_rows(_p(g), n, d2 // 2, _p(out))
    return out


def exp_row_scaled(row, scale):
    row = _c(row, np.float32).copy()
    s = lib().vxo_exp_row_scaled(_p(row), len(row), float(scale))
    return row, np.float32(s)


def linear(x, w, b=None):
    x, w = _c(x, np.float32), _c(w, np.float32)
    n, in_f = x.shape
    out_f = w.shape[0]
    y = np.empty((n, out_f), np.float32)
    b = None if b is None else _c(b, np.float32)
    lib().vxo_linear(_p(x), n, in_f, _p(w), _p(b), out_f, _p(y))
    return y


# ---------------------------------------------------------------------------------------------- encoder

def rel_pos_table(t, d=1024):
    out = np.empty((2 * t - 1, d), np.float32)
    lib().vxo_rel_pos_table(t, d, _p(out))
    return out


def fold_bn(dw, gamma, beta, mean, var, k):
    dw = _c(dw, np.float32).reshape(-1)
    d = len(gamma)
    dw_t = np.empty((k, d), np.float32)
    dw_b = np.empty(d, np.float32)
    args = [_c(a, np.float32) for a in (gamma, beta, mean, var)]
    lib().vxo_fold_bn(_p(dw), *[_p(a) for a in args], d, k, _p(dw_t), _p(dw_b))
    return dw_t, dw_b


def attn_core_int8(qkv, rel_k, t, bias_u, bias_v, d=1024, h=8):
    dh = d // h
    qkv, rel_k = _c(qkv, np.float32), _c(rel_k, np.float32)
    bu, bv = _c(bias_u, np.float32), _c(bias_v, np.float32)
    ctx = np.zeros((t, d), np.float32)
    scaling = np.float32(1.0) / np.sqrt(np.float32(dh), dtype=np.float32)
    lib().vxo_attn_core_int8(_p(qkv), _p(rel_k), t, d, h, dh, _p(bu), _p(bv), float(scaling), _p(ctx))
    return ctx


def attn_core_int8_rows(qkv, rel_k, t, bias_u, bias_v, blocks, d=1024, h=8):
    """attn_core_int8 on the listed 8-row query blocks only (rows 8b .. 8b+7); other rows of the result are zero."""
    dh = d // h
    qkv, rel_k = _c(qkv, np.float32), _c(rel_k, np.float32)
    bu, bv = _c(bias_u, np.float32), _c(bias_v, np.float32)
    blk = _c(blocks, np.int32)
    ctx = np.zeros((t, d), np.float32)
    scaling = np.float32(1.0) / np.sqrt(np.float32(dh), dtype=np.float32)
    lib().vxo_attn_core_int8_rows(_p(qkv), _p(rel_k), t, d, h, dh, _p(bu), _p(bv), float(scaling), _p(ctx),
                                  _p(blk), len(blk))
    return ctx


def conv_middle(g, dw_t, dw_b):
    """g [t, 2d] -> SiLU(depthwise conv(GLU(g))) [t, d] (encoder.rs:596-624)."""
    g = _c(g, np.float32)
    t, d2 = g.shape
    d = d2 // 2
    dw_t, dw_b = _c(dw_t, np.float32), _c(dw_b, np.float32)
    hb = np.empty((t, d), np.float32)
    lib().vxo_conv_middle(_p(g), t, d, dw_t.shape[0], _p(dw_t), _p(dw_b), _p(hb))
    return hb


class _Tern(C.Structure):
    _fields_ = [("w", _P), ("s", _P), ("out", _I), ("inp", _I), ("group", _I)]


class _Layer(C.Structure):
    _fields_ = [(n, _Tern) for n in ("ff1_1", "ff1_2", "qkv", "o", "relk", "pw1", "pw2", "ff2_1", "ff2_2")] + [
        ("ln_g", _P * 5), ("ln_b", _P * 5), ("bias_u", _P), ("bias_v", _P), ("dw_w", _P), ("dw_b", _P)]


class _Sub(C.Structure):
    _fields_ = [("channels", _I), ("kernel", _I), ("stride", _I), ("n_mels", _I), ("d_model", _I),
                ("conv0_w", _P), ("conv0_b", _P), ("dw_w", _P * 2), ("dw_b", _P * 2), ("pw_w", _P * 2),
                ("pw_b", _P * 2), ("lin_w", _P), ("lin_b", _P)]


LAYER_MODULES = ("ff1_1", "ff1_2", "qkv", "o", "relk", "pw1", "pw2", "ff2_1", "ff2_2")


class OracleLayer:
    """One FastConformer layer's weights in the oracle's form (int8 rows + f32 scales, folded BN)."""

    def __init__(self, lw):
        """lw: voxrt_b200.synth layer dict (base-3 packed ternary tensors, f16 scales, f32 dense params)."""
        self._keep = []
        self.s = _Layer()
        for name in LAYER_MODULES:
            m = lw[name]
            w, sc = unpack_matrix(m["qweight"], m["scales"], m["out"], m["in"], m["group"])
            self._keep += [w, sc]
            setattr(self.s, name, _Tern(_p(w), _p(sc), m["out"], m["in"], m["group"]))
        for i, n in enumerate(("norm_ff1", "norm_attn", "norm_conv", "norm_ff2", "norm_out")):
            g, b = _c(lw[n + "_w"], np.float32), _c(lw[n + "_b"], np.float32)
            self._keep += [g, b]
            self.s.ln_g[i], self.s.ln_b[i] = _p(g), _p(b)
        bu, bv = _c(lw["bias_u"], np.float32), _c(lw["bias_v"], np.float32)
        k = lw["dw_weight"].shape[-1]
        dw_t, dw_b = fold_bn(lw["dw_weight"], lw["bn_w"], lw["bn_b"], lw["bn_mean"], lw["bn_var"], k)
        self._keep += [bu, bv, dw_t, dw_b]
        self.s.bias_u, self.s.bias_v, self.s.dw_w, self.s.dw_b = _p(bu), _p(bv), _p(dw_t), _p(dw_b)
        self.k = k

    def forward(self, x, pos_emb, d=1024, heads=8):
        x = _c(x, np.float32).copy()
        pos_emb = _c(pos_emb, np.float32)
        if getattr(self, "_prep", None):
            lib().vxo_layer_forward_prepared(self._prep, C.byref(self.s), d, heads, self.k, _p(x), x.shape[0],
                                             _p(pos_emb))
        else:
            lib().vxo_layer_forward(C.byref(self.s), d, heads, self.k, _p(x), x.shape[0], _p(pos_emb))
        return x

    def prepare(self):
        """Repack the weights once (load time), so forwards time only the layer arithmetic."""
        if not getattr(self, "_prep", None):
            self._prep = lib().vxo_layer_prepare(C.byref(self.s))
        return self

    def __del__(self):
        try:
            if getattr(self, "_prep", None):
                lib().vxo_layer_free(self._prep)
        except Exception:
            pass


class OracleSubsampling:
    def __init__(self, sw):
        """sw: voxrt_b200.synth subsampling dict in HF layout; permuted here as Subsampling::load does."""
        c = sw["conv0_w"].shape[0]
        k = sw["conv0_w"].shape[-1]
        f3 = sw["lin_w"].shape[1] // c
        d = sw["lin_w"].shape[0]
        tap = lambda w: np.ascontiguousarray(np.asarray(w, np.float32).reshape(c, k * k).T)  # [k*k, C]
        lw = np.asarray(sw["lin_w"], np.float32).reshape(d, c, f3).transpose(0, 2, 1).reshape(d, f3 * c)
        self._keep = [tap(sw["conv0_w"]), _c(sw["conv0_b"], np.float32),
                      tap(sw["dw1_w"]), _c(sw["dw1_b"], np.float32), tap(sw["dw2_w"]), _c(sw["dw2_b"], np.float32),
                      _c(np.asarray(sw["pw1_w"]).reshape(c, c), np.float32), _c(sw["pw1_b"], np.float32),
                      _c(np.asarray(sw["pw2_w"]).reshape(c, c), np.float32), _c(sw["pw2_b"], np.float32),
                      _c(lw, np.float32), _c(sw["lin_b"], np.float32)]
        K = self._keep
        s = _Sub()
        s.channels, s.kernel, s.stride, s.n_mels, s.d_model = c, k, 2, sw["n_mels"], d
        s.conv0_w, s.conv0_b = _p(K[0]), _p(K[1])
        s.dw_w[0], s.dw_b[0], s.dw_w[1], s.dw_b[1] = _p(K[2]), _p(K[3]), _p(K[4]), _p(K[5])
        s.pw_w[0], s.pw_b[0], s.pw_w[1], s.pw_b[1] = _p(K[6]), _p(K[7]), _p(K[8]), _p(K[9])
        s.lin_w, s.lin_b = _p(K[10]), _p(K[11])
        self.s = s
        self.d = d
        self.k = k

    def out_frames(self, t):
        return lib().vxo_sub_out_frames(t, self.k, 2)

    def forward(self, feats):
        feats = _c(feats, np.float32)
        t = feats.shape[0]
        out = np.empty((self.out_frames(t), self.d), np.float32)
        lib().vxo_subsampling_forward(C.byref(self.s), _p(feats), t, _p(out))
        return out


def encoder_forward(sub: OracleSubsampling, layers, feats, d=1024, heads=8):
    """Encoder::forward (encoder.rs:816-856): subsampling, rel-pos table, layers."""
    x = sub.forward(feats)
    te = x.shape[0]
    pos = rel_pos_table(te, d)
    for L in layers:
        x = L.forward(x, pos, d, heads)
    return x


# ------------------------------------------------------------------------------------------------- TDT decoder
class _Tdt(C.Structure):
    _fields_ = [("hidden", _I), ("vocab", _I), ("n_dur", _I), ("blank", _I), ("max_symbols", _I), ("d_model", _I),
                ("n_layers", _I), ("durations", _P), ("embedding", _P), ("w_ih", _P * 4), ("s_ih", _P * 4),
                ("w_hh", _P * 4), ("s_hh", _P * 4), ("b", _P * 4), ("proj_w", _P), ("proj_b", _P), ("head_w", _P),
                ("head_s", _P), ("head_b", _P), ("enc_w", _P), ("enc_b", _P)]


def tdt_int8_rows(w_f16):
    """int8_rows (decoder.rs:270-303): per-row int8 codes + the row scale replicated per 128-group."""
    w = np.ascontiguousarray(w_f16).view(np.uint16)
    out, inp = w.shape
    rows = np.empty((out, inp), np.int8)
    sc = np.empty((out, inp // 128), np.float32)
    lib().vxo_tdt_int8_rows(_p(w), out, inp, _p(rows), _p(sc))
    return rows, sc


class TdtDecoder:
    """The reference decoder (decoder.rs) in int8 mode, from a weight dict with f16 LSTM / projector / head weights."""

    def __init__(self, m: dict):
        self._keep = []

        def keep(a, dtype):
            a = np.ascontiguousarray(a, dtype=dtype)
            self._keep.append(a)
            return a.ctypes.data

        h, v, nd = m["hidden"], m["vocab"], len(m["durations"])
        self.hidden, self.vocab, self.n_dur = h, v, nd
        st = _Tdt()
        st.hidden, st.vocab, st.n_dur, st.blank = h, v, nd, m["blank"]
        st.max_symbols, st.d_model, st.n_layers = m["max_symbols"], m["d_model"], len(m["lstm"])
        st.durations = keep(m["durations"], np.int32)
        st.embedding = keep(m["embedding"], np.float32)
        for l, layer in enumerate(m["lstm"]):
            wi, si = tdt_int8_rows(layer["w_ih"])
            wh, sh = tdt_int8_rows(layer["w_hh"])
            st.w_ih[l], st.s_ih[l] = keep(wi, np.int8), keep(si, np.float32)
            st.w_hh[l], st.s_hh[l] = keep(wh, np.int8), keep(sh, np.float32)
            st.b[l] = keep(np.asarray(layer["b_ih"], np.float32) + np.asarray(layer["b_hh"], np.float32),
                           np.float32)
        st.proj_w = keep(np.asarray(m["proj_w"]).view(np.uint16), np.uint16)
        st.proj_b = keep(m["proj_b"], np.float32)
        hw, hs = tdt_int8_rows(m["head_w"])
        st.head_w, st.head_s = keep(hw, np.int8), keep(hs, np.float32)
        st.head_b = keep(m["head_b"], np.float32)
        st.enc_w = keep(m["enc_w"], np.float32)
        st.enc_b = keep(m["enc_b"], np.float32)
        self._st = st
        self.n_layers = len(m["lstm"])

    def _ref(self):
        return C.byref(self._st)

    def project(self, enc):
        enc = np.ascontiguousarray(enc, np.float32)
        t = enc.shape[0]
        out = np.empty((t, self.hidden), np.float32)
        lib().vxo_tdt_project(self._ref(), _p(enc), t, _p(out))
        return out

    def joint(self, enc_t, g):
        out = np.empty(self.vocab + self.n_dur, np.float32)
        lib().vxo_tdt_joint(self._ref(), _p(_c(enc_t, np.float32)), _p(_c(g, np.float32)), _p(out))
        return out

    def pred_step(self, token, h, c):
        g = np.empty(self.hidden, np.float32)
        hn = np.empty_like(_c(h, np.float32))
        cn = np.empty_like(hn)
        lib().vxo_tdt_pred_step(self._ref(), int(token), _p(_c(h, np.float32)), _p(_c(c, np.float32)), _p(g),
                                _p(hn), _p(cn))
        return g, hn, cn

    def greedy(self, proj):
        proj = np.ascontiguousarray(proj, np.float32)
        t = proj.shape[0]
        cap = max(1, t * 10 + 16)
        tok, fr, du = (np.empty(cap, np.int32) for _ in range(3))
        n = lib().vxo_tdt_greedy(self._ref(), _p(proj), t, _p(tok), _p(fr), _p(du), cap)
        assert n <= cap
        return np.stack([tok[:n], fr[:n], du[:n]], axis=1)


# ------------------------------------------------------------------------------------------------ frontend
# NeMo log-mel (crates/voxrt/src/frontend.rs), restated in numpy for the GPU frontend's parity tests. The FFT is
# numpy's (f64, then the bins rounded to f32), not realfft's f32 transform, so agreement with the reference and with
# the GPU is to f32 rounding of the spectrum, not bit for bit.
def _hz_to_mel(f):
    """frontend.rs:45-56 (librosa Slaney, htk=False)"""
    f_sp, min_log_hz = 200.0 / 3.0, 1000.0
    min_log_mel, logstep = min_log_hz / f_sp, np.log(6.4) / 27.0
    return min_log_mel + np.log(f / min_log_hz) / logstep if f >= min_log_hz else f / f_sp


def _mel_to_hz(m):
    """frontend.rs:58-71"""
    f_sp, min_log_hz = 200.0 / 3.0, 1000.0
    min_log_mel, logstep = min_log_hz / f_sp, np.log(6.4) / 27.0
    return min_log_hz * np.exp(logstep * (m - min_log_mel)) if m >= min_log_mel else f_sp * m


def mel_filterbank(sr=16000, n_fft=512, n_mels=128):
    """slaney_mel_filterbank (frontend.rs:74-90): f64, cast to f32. [n_mels, n_fft/2 + 1]"""
    n_bins = n_fft // 2 + 1
    fftf = np.arange(n_bins, dtype=np.float64) * sr / n_fft
    lo, hi = _hz_to_mel(0.0), _hz_to_mel(sr / 2.0)
    mel_f = np.array([_mel_to_hz(lo + (hi - lo) * i / (n_mels + 1)) for i in range(n_mels + 2)])
    fb = np.zeros((n_mels, n_bins), np.float32)
    for i in range(n_mels):
        enorm = 2.0 / (mel_f[i + 2] - mel_f[i])
        lower = (fftf - mel_f[i]) / (mel_f[i + 1] - mel_f[i])
        upper = (mel_f[i + 2] - fftf) / (mel_f[i + 2] - mel_f[i + 1])
        fb[i] = (np.maximum(np.minimum(lower, upper), 0.0) * enorm).astype(np.float32)
    return fb


def mel_power(samples, n_mels=128, sr=16000, n_fft=512, win=400, hop=160, preemph=0.97):
    """log_mel's steps up to the f64 mel sums (frontend.rs:112-160): [n_frames, n_mels] f64."""
    s = np.asarray(samples, np.float32)
    x = s.copy()
    x[1:] = s[1:] - np.float32(preemph) * s[:-1]  # product, then difference, in f32
    pad = n_fft // 2
    padded = np.concatenate([np.zeros(pad, np.float32), x, np.zeros(pad, np.float32)])
    n = len(s) // hop
    k = np.arange(win, dtype=np.float64)
    window = (0.5 - 0.5 * np.cos(2.0 * np.pi * k / (win - 1))).astype(np.float32)
    woff = (n_fft - win) // 2
    frames = np.zeros((n, n_fft), np.float32)
    for t in range(n):
        frames[t, woff:woff + win] = padded[t * hop + woff:t * hop + woff + win] * window
    spec = np.fft.rfft(frames.astype(np.float64), axis=1)
    re, im = spec.real.astype(np.float32), spec.imag.astype(np.float32)
    power = re * re + im * im
    return power.astype(np.float64) @ mel_filterbank(sr, n_fft, n_mels).astype(np.float64).T


def log_mel(samples, n_mels=128):
    """frontend.rs:112-166: logf(f32(mel sum) + 2^-24)."""
    return np.log(mel_power(samples, n_mels).astype(np.float32) + np.float32(5.9604645e-8)).astype(np.float32)


def normalize_feats(feats):
    """Frontend::normalize (frontend.rs:169-191): per feature, f64 mean and unbiased variance, std + 1e-5 in f32."""
    f = np.asarray(feats, np.float32).copy()
    n = f.shape[0]
    if n < 2:
        return f
    mean = f.astype(np.float64).mean(axis=0)
    var = ((f.astype(np.float64) - mean) ** 2).sum(axis=0) / (n - 1.0)
    std = np.sqrt(var).astype(np.float32) + np.float32(1e-5)
    return ((f - mean.astype(np.float32)) / std).astype(np.float32)
