"""The encoder on one GPU, mirroring the reference's GPU encoder boundary (GpuEncoder, crates/voxrt/src/metal/
mod.rs:451-640; Transcriber::encode, transcriber.rs:194-225): load from model tensors, forward (layers on
subsampled input), forward_feats (log-mel in, encoder frames out), warm_up, plus a token-stacked batch form.
All arithmetic runs in libvxg.so's sm_100a kernels; this module only marshals tensors through the C ABI."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib

_P, _I = C.c_void_p, C.c_int

WEIGHTS_2BIT, WEIGHTS_INT8 = 0, 1


class _Tern(C.Structure):
    _fields_ = [("qweight", _P), ("scales", _P), ("out", _I), ("inp", _I), ("group", _I)]


_TERN_FIELDS = ("ff1_linear1", "ff1_linear2", "q_proj", "k_proj", "v_proj", "o_proj", "relative_k_proj",
                "pointwise_conv1", "pointwise_conv2", "ff2_linear1", "ff2_linear2")
_DENSE_FIELDS = ("norm_ff1_w", "norm_ff1_b", "norm_attn_w", "norm_attn_b", "norm_conv_w", "norm_conv_b",
                 "norm_ff2_w", "norm_ff2_b", "norm_out_w", "norm_out_b", "bias_u", "bias_v", "dw_weight",
                 "bn_weight", "bn_bias", "bn_mean", "bn_var")


class _Layer(C.Structure):
    _fields_ = [(n, _Tern) for n in _TERN_FIELDS] + [(n, _P) for n in _DENSE_FIELDS]


_SUB_FIELDS = ("conv0_w", "conv0_b", "dw1_w", "dw1_b", "pw1_w", "pw1_b", "dw2_w", "dw2_b", "pw2_w", "pw2_b",
               "lin_w", "lin_b")


class _Sub(C.Structure):
    _fields_ = [(n, _P) for n in _SUB_FIELDS]


class _Desc(C.Structure):
    _fields_ = [("d_model", _I), ("ff", _I), ("heads", _I), ("conv_kernel", _I), ("n_layers", _I), ("n_mels", _I),
                ("sub_channels", _I), ("weight_format", _I), ("layers", C.POINTER(_Layer)),
                ("sub", C.POINTER(_Sub))]


def _split_qkv(m):
    """The synthetic / model-file q|k|v stack -> three modules (rows 0..d, d..2d, 2d..3d)."""
    d = m["out"] // 3
    return [{"qweight": m["qweight"][i * d:(i + 1) * d], "scales": m["scales"][i * d:(i + 1) * d], "out": d,
             "in": m["in"], "group": m["group"]} for i in range(3)]


class CudaEncoder:
    """GpuEncoder equivalent on one B200. `model` is a dict {"sub": subsampling tensors, "layers": [layer dicts]}
    in the model file's layouts (voxrt_b200.synth produces one)."""

    def __init__(self, handle, d_model, n_mels, device):
        self._h = handle
        self.d_model, self.n_mels, self.device = d_model, n_mels, device

    @classmethod
    def load(cls, model: dict, device: int = 0, weights: str = "2bit") -> "CudaEncoder":
        keep = []

        def arr(a, dtype):
            a = np.ascontiguousarray(a, dtype)
            keep.append(a)
            return a.ctypes.data

        layers = model["layers"]
        L = (_Layer * len(layers))()
        names = {"ff1_linear1": "ff1_1", "ff1_linear2": "ff1_2", "o_proj": "o", "relative_k_proj": "relk",
                 "pointwise_conv1": "pw1", "pointwise_conv2": "pw2", "ff2_linear1": "ff2_1", "ff2_linear2": "ff2_2"}
        dense = {"norm_ff1_w": "norm_ff1_w", "norm_ff1_b": "norm_ff1_b", "norm_attn_w": "norm_attn_w",
                 "norm_attn_b": "norm_attn_b", "norm_conv_w": "norm_conv_w", "norm_conv_b": "norm_conv_b",
                 "norm_ff2_w": "norm_ff2_w", "norm_ff2_b": "norm_ff2_b", "norm_out_w": "norm_out_w",
                 "norm_out_b": "norm_out_b", "bias_u": "bias_u", "bias_v": "bias_v", "dw_weight": "dw_weight",
                 "bn_weight": "bn_w", "bn_bias": "bn_b", "bn_mean": "bn_mean", "bn_var": "bn_var"}
        for i, lw in enumerate(layers):
            mods = dict(lw)
            if "qkv" in lw:
                mods["q_proj"], mods["k_proj"], mods["v_proj"] = _split_qkv(lw["qkv"])
            for f in _TERN_FIELDS:
                m = mods[names.get(f, f)]
                setattr(L[i], f, _Tern(arr(m["qweight"], np.uint8), arr(np.asarray(m["scales"]).view(np.uint16),
                                                                        np.uint16), m["out"], m["in"], m["group"]))
            for f in _DENSE_FIELDS:
                setattr(L[i], f, arr(lw[dense[f]], np.float32))
        sw = model["sub"]
        S = _Sub(*[arr(sw[f], np.float32) for f in _SUB_FIELDS])
        l0 = layers[0]
        desc = _Desc(d_model=l0["ff1_1"]["in"], ff=l0["ff1_1"]["out"], heads=np.asarray(l0["bias_u"]).shape[0],
                     conv_kernel=np.asarray(l0["dw_weight"]).shape[-1], n_layers=len(layers),
                     n_mels=int(sw["n_mels"]), sub_channels=np.asarray(sw["conv0_w"]).shape[0],
                     weight_format=WEIGHTS_2BIT if weights == "2bit" else WEIGHTS_INT8, layers=L, sub=C.pointer(S))
        h = C.c_void_p()
        check(lib().vxg_encoder_create(C.byref(desc), device, C.byref(h)))
        return cls(h, desc.d_model, desc.n_mels, device)

    @classmethod
    def from_model(cls, model, device: int = 0, weights: str = "2bit") -> "CudaEncoder":
        """GpuEncoder::load from a model directory (a path or an open voxrt_b200.model.ModelFile)."""
        from .model import ModelFile

        mf = model if isinstance(model, ModelFile) else ModelFile.open(model)
        cfg = mf.config()
        h = C.c_void_p()
        check(lib().vxg_encoder_create_from_model(mf._h, WEIGHTS_2BIT if weights == "2bit" else WEIGHTS_INT8, device,
                                                  C.byref(h)))
        if mf is not model:
            mf.close()
        return cls(h, cfg["d_model"], cfg["n_mels"], device)

    def close(self):
        if self._h:
            lib().vxg_encoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def out_frames(t_in: int) -> int:
        return lib().vxg_encoder_out_frames(int(t_in))

    def forward_feats(self, feats: np.ndarray):
        """GpuEncoder::forward_feats: log-mel [t_in, n_mels] (host) -> (encoder output [t_e, d], t_e)."""
        feats = np.ascontiguousarray(feats, np.float32)
        te = self.out_frames(feats.shape[0])
        out = np.empty((te, self.d_model), np.float32)
        t_e = C.c_int()
        check(lib().vxg_encoder_forward_feats(self._h, feats.ctypes.data, feats.shape[0], out.ctypes.data, out.size,
                                              C.byref(t_e)))
        return out, t_e.value

    @staticmethod
    def pinned_array(shape, dtype=np.float32):
        """A numpy array in page-locked host memory (torch's pinned allocator). forward_batch moves page-locked
        feats and output arrays with the DMA engines directly, with no staging copy on the host."""
        import torch

        return torch.empty(tuple(shape), dtype=torch.from_numpy(np.empty(0, dtype)).dtype, pin_memory=True).numpy()

    def forward_batch(self, feats_list, outs=None):
        """Token-stacked forward of several utterances: host arrays in, host arrays out (one copy each way).

        `outs` (optional) are caller-owned C-contiguous float32 arrays of shape [out_frames(t_in[u]), d_model] that
        receive the frames, so a caller that runs many batches of the same lengths reuses its buffers."""
        feats_list = [np.ascontiguousarray(f, np.float32) for f in feats_list]
        n = len(feats_list)
        t_in = np.array([f.shape[0] for f in feats_list], np.int32)
        if outs is None:
            outs = [np.empty((self.out_frames(t), self.d_model), np.float32) for t in t_in]
        else:
            if len(outs) != n:
                raise ValueError(f"{len(outs)} output arrays for {n} utterances")
            for u, (o, t) in enumerate(zip(outs, t_in)):
                want = (self.out_frames(int(t)), self.d_model)
                if o.dtype != np.float32 or o.shape != want or not o.flags["C_CONTIGUOUS"] or not o.flags["WRITEABLE"]:
                    raise ValueError(f"outs[{u}]: need a writeable C-contiguous float32 array of shape {want}")
        fp = (C.c_void_p * n)(*[f.ctypes.data for f in feats_list])
        op = (C.c_void_p * n)(*[o.ctypes.data for o in outs])
        te = np.empty(n, np.int32)
        check(lib().vxg_encoder_forward_batch(self._h, fp, t_in.ctypes.data, n, op, te.ctypes.data))
        return outs

    def forward_device(self, feats, t_in, out, stream=None):
        """Device-resident batch: feats [sum t_in, n_mels] and out [sum t_e, d] are torch CUDA tensors."""
        import torch

        t_in = np.ascontiguousarray(t_in, np.int32)
        te = np.empty(len(t_in), np.int32)
        s = stream if stream is not None else torch.cuda.current_stream()
        check(lib().vxg_encoder_forward_device(self._h, C.c_void_p(feats.data_ptr()), t_in.ctypes.data, len(t_in),
                                               C.c_void_p(out.data_ptr()), te.ctypes.data,
                                               C.c_void_p(s.cuda_stream)))
        return te

    def subsample_device(self, feats, t_in, out=None, stream=None):
        """GpuEncoder::subsample / Transcriber::subsample (transcriber.rs:182-192): the subsampling front end alone
        on stacked feats [sum t_in, n_mels] (torch CUDA) -> [sum t_e, d] (the VAD head's input)."""
        import torch

        t_in = np.ascontiguousarray(t_in, np.int32)
        te = np.array([self.out_frames(int(t)) for t in t_in], np.int32)
        if out is None:
            out = torch.empty((int(te.sum()), self.d_model), dtype=torch.float32, device=feats.device)
        s = stream if stream is not None else torch.cuda.current_stream()
        check(lib().vxg_encoder_subsample_device(self._h, C.c_void_p(feats.data_ptr()), t_in.ctypes.data, len(t_in),
                                                 C.c_void_p(out.data_ptr()), te.ctypes.data,
                                                 C.c_void_p(s.cuda_stream)))
        return out

    def forward(self, x, t):
        """GpuEncoder::forward: layers on subsampled input x [sum t, d] (torch CUDA, stacked) -> new tensor."""
        import torch

        t = np.ascontiguousarray(np.atleast_1d(t), np.int32)
        out = torch.empty_like(x)
        check(lib().vxg_encoder_forward_layers_device(self._h, C.c_void_p(x.data_ptr()), t.ctypes.data, len(t),
                                                      C.c_void_p(out.data_ptr()),
                                                      C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return out

    PROF_CLASSES = ("subsampling", "ln_quant", "gemm", "attention", "conv", "quantize")

    def set_profiling(self, on: bool):
        check(lib().vxg_encoder_set_profiling(self._h, int(bool(on))))

    def profile(self) -> dict:
        """Device ms and launch counts per kernel class since the last call, plus the GEMMs' int8 ops."""
        ms = (C.c_double * 6)()
        n = (C.c_int * 6)()
        ops = C.c_double()
        check(lib().vxg_encoder_profile(self._h, ms, n, C.byref(ops)))
        return {"ms": dict(zip(self.PROF_CLASSES, list(ms))), "steps": dict(zip(self.PROF_CLASSES, list(n))),
                "gemm_ops": ops.value}

    def warm_up(self, t: int):
        """GpuEncoder::warm_up: run once on silence to size the workspace for inputs up to t encoder frames."""
        self.forward_feats(np.zeros((t * 8, self.n_mels), np.float32))
