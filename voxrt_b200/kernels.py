"""Kernel-level API mirroring the reference's kernel trait (crates/voxrt/src/kernels/mod.rs, packed.rs): device
TernaryMatrix / QuantAct operands, the Epilogue enum and gemm_ep, each a thin call into libvxg.so's C ABI.

Device memory and streams are torch CUDA tensors / streams (plumbing only); the arithmetic runs in the library's
sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import check, lib

GROUP = 128


@dataclass(frozen=True)
class Epilogue:
    """kernels/mod.rs:14-21: Store, Silu, AddScaled(s)."""

    kind: int
    scale: float = 0.0

    @staticmethod
    def AddScaled(s: float) -> "Epilogue":
        return Epilogue(2, float(s))


Epilogue.Store = Epilogue(0)
Epilogue.Silu = Epilogue(1)


def _stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


class TernaryMatrix:
    """Ternary weights [out, inp] resident on the GPU in one of the kernels' formats, chosen at load time like the
    reference's Layout (packed.rs:8-27): "2bit" = 2-bit codes tiled per 128 rows x 128 columns, unpacked to int8
    inside the SM; "int8" = int8 rows (4x the bytes, no unpack). f32 scales tile-major in both.
    TernaryMatrix::from_packed_layout (packed.rs:73-130)."""

    def __init__(self, out, inp, group, weights, scales_t, fmt="2bit"):
        self.out, self.inp, self.group, self.fmt = out, inp, group, fmt
        self.weights, self.scales_t = weights, scales_t

    @property
    def codes(self):
        return self.weights

    @classmethod
    def from_packed(cls, qweight, scales_f16, out, inp, group=GROUP, device=None, fmt="2bit"):
        L = lib()
        q = np.ascontiguousarray(qweight, np.uint8)
        s = np.ascontiguousarray(scales_f16).view(np.uint16)
        ns = L.vxg_ternary_scales_count(out, inp, group)
        st = np.empty(ns, np.float32)
        if fmt == "2bit":
            w = np.empty(L.vxg_ternary_codes_bytes(out, inp), np.uint8)
            check(L.vxg_ternary_repack(q.ctypes.data, s.ctypes.data, out, inp, group, w.ctypes.data, st.ctypes.data))
        elif fmt == "int8":
            w = np.empty(L.vxg_ternary_i8_bytes(out, inp), np.int8)
            check(L.vxg_ternary_repack_i8(q.ctypes.data, s.ctypes.data, out, inp, group, w.ctypes.data,
                                          st.ctypes.data))
        else:
            raise ValueError(f"unknown weight format {fmt!r}")
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        return cls(out, inp, group, torch.from_numpy(w).to(dev), torch.from_numpy(st).to(dev), fmt)

    @classmethod
    def from_module(cls, m: dict, device=None, fmt="2bit"):
        """From a synthetic / model-file module dict {qweight, scales, out, in, group}."""
        return cls.from_packed(m["qweight"], m["scales"], m["out"], m["in"], m["group"], device, fmt)


class QuantAct:
    """int8 activations [n, inp] + f32 scales [n, inp/group] on the GPU (QuantAct, packed.rs:286-298)."""

    def __init__(self, x: torch.Tensor, scales: torch.Tensor, group: int = GROUP):
        assert x.dtype == torch.int8 and x.is_cuda and x.is_contiguous()
        assert scales.dtype == torch.float32 and scales.is_cuda and scales.is_contiguous()
        self.x, self.scales, self.group = x, scales, group
        self.n, self.inp = x.shape


def gemm_ep(w: TernaryMatrix, x: QuantAct, y: torch.Tensor, bias: torch.Tensor | None = None,
            ep: Epilogue = Epilogue.Store, group_sums: torch.Tensor | None = None, stream=None):
    """y[n, out] = epilogue(x x w^T) (+ bias): kernels::gemm_ep (kernels/mod.rs:324-362), on the tensor cores."""
    assert x.inp == w.inp and x.group == w.group, "input width / group mismatch"
    assert y.dtype == torch.float32 and y.is_contiguous() and tuple(y.shape) == (x.n, w.out)
    fn = lib().vxg_gemm_ternary_i8 if w.fmt == "2bit" else lib().vxg_gemm_ternary_i8w
    check(fn(_ptr(x.x), _ptr(x.scales), _ptr(w.weights), _ptr(w.scales_t), x.n, w.out, w.inp, w.group, ep.kind,
             ep.scale, _ptr(bias), _ptr(y), _ptr(group_sums), _stream_ptr(stream)))
    return y


def gemm_silu_quant(w: TernaryMatrix, x: QuantAct, stream=None) -> QuantAct:
    """FeedForward::forward_fused's linear1 (encoder.rs:79-94): Silu GEMM, then per-(row, 128) int8 for linear2,
    fused in one kernel; returns the int8 activations linear2 consumes."""
    assert x.inp == w.inp and x.group == w.group, "input width / group mismatch"
    q = torch.empty((x.n, w.out), dtype=torch.int8, device=x.x.device)
    s = torch.empty((x.n, w.out // GROUP), dtype=torch.float32, device=x.x.device)
    fn = lib().vxg_gemm_ternary_silu_q if w.fmt == "2bit" else lib().vxg_gemm_ternary_silu_q_w
    check(fn(_ptr(x.x), _ptr(x.scales), _ptr(w.weights), _ptr(w.scales_t), x.n, w.out, w.inp, w.group, _ptr(q),
             _ptr(s), _stream_ptr(stream)))
    return QuantAct(q, s, GROUP)


def gemm_qkv_quant(w: TernaryMatrix, x: QuantAct, heads: int, bias_u: torch.Tensor, bias_v: torch.Tensor,
                   stream=None):
    """The stacked q|k|v projection with the attention's per-head operands quantised in the epilogue (encoder.rs:
    138-187, :349-377). Returns (qu, squ, qv, sqv, k, sk, y): int8 [heads, n, 128] codes with f32 [heads, n] scales
    for q + bias_u, q + bias_v and k, and y [n, 3 * heads * 128] f32 whose v columns hold the v projection."""
    assert w.fmt == "2bit" and w.out == 3 * heads * 128 and x.inp == w.inp and x.group == w.group
    dev = x.x.device
    q8 = [torch.empty((heads, x.n, 128), dtype=torch.int8, device=dev) for _ in range(3)]
    sc = [torch.empty((heads, x.n), dtype=torch.float32, device=dev) for _ in range(3)]
    y = torch.empty((x.n, w.out), dtype=torch.float32, device=dev)
    check(lib().vxg_gemm_ternary_qkv_quant(_ptr(x.x), _ptr(x.scales), _ptr(w.weights), _ptr(w.scales_t), x.n, heads,
                                           w.inp, w.group, _ptr(bias_u), _ptr(bias_v), _ptr(q8[0]), _ptr(q8[1]),
                                           _ptr(q8[2]), _ptr(sc[0]), _ptr(sc[1]), _ptr(sc[2]), _ptr(y),
                                           _stream_ptr(stream)))
    return q8[0], sc[0], q8[1], sc[1], q8[2], sc[2], y


def glu_row_order(n: int) -> np.ndarray:
    """Source rows (the reference's [value; gate] order) of the rows of a GLU projection as its GEMM expects them."""
    L = lib()
    order = np.array([L.vxg_glu_source_row(r, n) for r in range(n)], np.int64)
    assert order.min() >= 0, f"GLU projection width {n} unsupported"
    return order


def gemm_glu(w: TernaryMatrix, x: QuantAct, stream=None) -> torch.Tensor:
    """pointwise_conv1 + glu_row (encoder.rs:594-596, tensor.rs:936-940) fused: `w` holds the projection's rows in
    glu_row_order; returns y [n, out / 2] f32."""
    assert w.fmt == "2bit" and x.inp == w.inp and x.group == w.group
    y = torch.empty((x.n, w.out // 2), dtype=torch.float32, device=x.x.device)
    check(lib().vxg_gemm_ternary_glu(_ptr(x.x), _ptr(x.scales), _ptr(w.weights), _ptr(w.scales_t), x.n, w.out, w.inp,
                                     w.group, _ptr(y), _stream_ptr(stream)))
    return y


def gemm(w: TernaryMatrix, x: QuantAct, y: torch.Tensor, bias: torch.Tensor | None = None, stream=None):
    """kernels::gemm (kernels/mod.rs:319-321)."""
    return gemm_ep(w, x, y, bias, Epilogue.Store, stream=stream)


def quantize(x: torch.Tensor, group: int = GROUP, stream=None) -> QuantAct:
    """QuantAct::quantize (packed.rs:302-312) on the GPU: per-(token, group) absmax/127 int8."""
    assert x.dtype == torch.float32 and x.is_cuda and x.is_contiguous() and x.dim() == 2
    n, inp = x.shape
    q = torch.empty((n, inp), dtype=torch.int8, device=x.device)
    s = torch.empty((n, inp // group), dtype=torch.float32, device=x.device)
    check(lib().vxg_quantize_rows(_ptr(x), n, inp, group, _ptr(q), _ptr(s), _stream_ptr(stream)))
    return QuantAct(q, s, group)


def ln_quant(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, group: int = GROUP, pre=None,
             x_out: torch.Tensor | None = None, stream=None) -> QuantAct:
    """TernaryLinear::prepare_normed (ternary_linear.rs:132-158): LayerNorm(x) -> int8, fused. `pre` = (g0, b0)
    applies a first LayerNorm whose f32 output goes to x_out (norm_out of the previous layer)."""
    n, d = x.shape
    q = torch.empty((n, d), dtype=torch.int8, device=x.device)
    s = torch.empty((n, d // group), dtype=torch.float32, device=x.device)
    g0, b0 = pre if pre is not None else (None, None)
    check(lib().vxg_ln_quant(_ptr(x), n, d, _ptr(g0), _ptr(b0), _ptr(x_out), _ptr(gamma), _ptr(beta), group,
                             _ptr(q), _ptr(s), _stream_ptr(stream)))
    return QuantAct(q, s, group)


def layer_norm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, out: torch.Tensor, stream=None):
    """LayerNormP::forward (encoder.rs:60-62) -> out (may be x)."""
    n, d = x.shape
    check(lib().vxg_ln_quant(_ptr(x), n, d, _ptr(gamma), _ptr(beta), _ptr(out), None, None, GROUP, None, None,
                             _stream_ptr(stream)))
    return out


def attention_i8(qkv: torch.Tensor, rel_k: torch.Tensor, tmax: int, offsets, lengths, bias_u: torch.Tensor,
                 bias_v: torch.Tensor, heads: int = 8, scaling: float | None = None, want_f32: bool = True,
                 want_q: bool = True, workspace: torch.Tensor | None = None, stream=None):
    """attn_core_int8 (encoder.rs:317-534) for utterances stacked in qkv rows. Returns (ctx f32 | None,
    QuantAct of ctx per head | None)."""
    rows, ld = qkv.shape
    d = heads * 128
    if scaling is None:
        scaling = float(np.float32(1.0) / np.sqrt(np.float32(128.0), dtype=np.float32))
    off = np.ascontiguousarray(offsets, np.int32)
    ln = np.ascontiguousarray(lengths, np.int32)
    nb = lib().vxg_attention_workspace_bytes(rows, tmax, len(ln), heads)
    if workspace is None or workspace.numel() < nb:
        workspace = torch.empty(nb, dtype=torch.uint8, device=qkv.device)
    ctx = torch.zeros((rows, d), dtype=torch.float32, device=qkv.device) if want_f32 else None
    cq = torch.zeros((rows, d), dtype=torch.int8, device=qkv.device) if want_q else None
    cs = torch.zeros((rows, heads), dtype=torch.float32, device=qkv.device) if want_q else None
    check(lib().vxg_attention_i8(_ptr(qkv), ld, _ptr(rel_k), tmax, off.ctypes.data, ln.ctypes.data, len(ln),
                                 _ptr(bias_u), _ptr(bias_v), heads, 128, float(scaling), _ptr(ctx), _ptr(cq),
                                 _ptr(cs), _ptr(workspace), workspace.numel(), _stream_ptr(stream)))
    return ctx, (QuantAct(cq, cs, 128) if want_q else None)


def fold_bn(dw, gamma, beta, mean, var):
    """ConvModule::load (encoder.rs:546-579): BN(eval) folded into the depthwise conv -> (dw_t [k, d], bias [d])."""
    dw = np.ascontiguousarray(dw, np.float32)
    d, k = dw.shape[0], dw.shape[-1]
    dw_t = np.empty((k, d), np.float32)
    dw_b = np.empty(d, np.float32)
    args = [np.ascontiguousarray(a, np.float32) for a in (gamma, beta, mean, var)]
    check(lib().vxg_fold_bn(dw.ctypes.data, *[a.ctypes.data for a in args], d, k, dw_t.ctypes.data,
                            dw_b.ctypes.data))
    return dw_t, dw_b


def conv_glu_dw_silu(g: torch.Tensor, offsets, lengths, dw_t: torch.Tensor, dw_b: torch.Tensor, want_f32=True,
                     want_q=True, stream=None):
    """ConvModule middle (encoder.rs:596-626): GLU -> depthwise conv -> SiLU (-> int8 for pointwise_conv2)."""
    rows, ld = g.shape
    k, d = dw_t.shape
    off = np.ascontiguousarray(offsets, np.int32)
    ln = np.ascontiguousarray(lengths, np.int32)
    nb = lib().vxg_conv_workspace_bytes(rows, len(ln))
    ws = torch.empty(nb, dtype=torch.uint8, device=g.device)
    hb = torch.zeros((rows, d), dtype=torch.float32, device=g.device) if want_f32 else None
    q = torch.zeros((rows, d), dtype=torch.int8, device=g.device) if want_q else None
    s = torch.zeros((rows, d // 128), dtype=torch.float32, device=g.device) if want_q else None
    check(lib().vxg_conv_glu_dw_silu_quant(_ptr(g), ld, off.ctypes.data, ln.ctypes.data, len(ln), _ptr(dw_t),
                                           _ptr(dw_b), d, k, _ptr(hb), _ptr(q), _ptr(s), _ptr(ws), nb,
                                           _stream_ptr(stream)))
    return hb, (QuantAct(q, s, 128) if want_q else None)


class Subsampling:
    """Device weights of the dw-striding Conv2d x8 front end in the layouts Subsampling::load prepares
    (subsampling.rs:31-96): 3x3 kernels tap-major [9][C], pointwise [C][C], final linear with its columns permuted
    to channels-last (f*C + c)."""

    def __init__(self, sw: dict, device=None):
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        c = sw["conv0_w"].shape[0]
        k = sw["conv0_w"].shape[-1]
        d = sw["lin_w"].shape[0]
        f3 = sw["lin_w"].shape[1] // c
        tap = lambda w: np.ascontiguousarray(np.asarray(w, np.float32).reshape(c, k * k).T)
        lw = np.asarray(sw["lin_w"], np.float32).reshape(d, c, f3).transpose(0, 2, 1).reshape(d, f3 * c)
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
        self.t = [T(tap(sw["conv0_w"])), T(sw["conv0_b"]), T(tap(sw["dw1_w"])), T(sw["dw1_b"]),
                  T(np.asarray(sw["pw1_w"]).reshape(c, c)), T(sw["pw1_b"]), T(tap(sw["dw2_w"])), T(sw["dw2_b"]),
                  T(np.asarray(sw["pw2_w"]).reshape(c, c)), T(sw["pw2_b"]), T(lw), T(sw["lin_b"])]
        self.n_mels, self.d_model = int(sw["n_mels"]), d

    @staticmethod
    def out_frames(t_in: int) -> int:
        return lib().vxg_sub_out_frames(int(t_in))

    def forward(self, feats: torch.Tensor, t_in, stream=None) -> torch.Tensor:
        """Stacked feats [sum t_in, n_mels] -> stacked [sum out_frames, d_model] (Subsampling::forward)."""
        t_in = np.ascontiguousarray(t_in, np.int32)
        rows = sum(self.out_frames(t) for t in t_in)
        out = torch.empty((rows, self.d_model), dtype=torch.float32, device=feats.device)
        nb = lib().vxg_subsampling_workspace_bytes(t_in.ctypes.data, len(t_in), self.n_mels)
        ws = torch.empty(nb, dtype=torch.uint8, device=feats.device)
        check(lib().vxg_subsampling(_ptr(feats), t_in.ctypes.data, len(t_in), self.n_mels,
                                    *[_ptr(a) for a in self.t], self.d_model, _ptr(out), _ptr(ws), nb,
                                    _stream_ptr(stream)))
        return out
