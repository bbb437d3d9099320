"""VAD head and segmentation behind libvxg's C ABI, mirroring the reference's crates/voxrt/src/vad.rs: VadHead
(load, probs) on the GPU and segment() with SegmentConfig on the host."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import check, lib

_P, _I = C.c_void_p, C.c_int


class _Desc(C.Structure):
    _fields_ = [("d_model", _I), ("hidden", _I), ("kernel", _I), ("proj_w", _P), ("proj_b", _P), ("ctx_w", _P),
                ("ctx_b", _P), ("out_w", _P), ("out_b", C.c_float), ("frame_seconds", C.c_double), ("device", _I)]


class SegmentConfig(C.Structure):
    """SegmentConfig (vad.rs:86-103); SegmentConfig() holds the reference's defaults."""
    _fields_ = [("threshold", C.c_float), ("min_pause_frames", _I), ("max_frames", _I), ("min_frames", _I),
                ("pad_frames", _I)]

    def __init__(self, **kw):
        super().__init__()
        lib().vxg_segment_cfg_default(C.byref(self))
        for k, v in kw.items():
            setattr(self, k, v)

    def as_dict(self) -> dict:
        return {n: getattr(self, n) for n, _ in self._fields_}


class _Seg(C.Structure):
    _fields_ = [("start", _I), ("end", _I)]


def segment(probs, cfg: SegmentConfig | None = None) -> list[tuple[int, int]]:
    """segment (vad.rs:140-240): speech segments [start, end) in encoder frames."""
    p = np.ascontiguousarray(probs, np.float32)
    cfg = cfg or SegmentConfig()
    cap = p.size + 1
    out = (_Seg * cap)()
    n = C.c_size_t(0)
    check(lib().vxg_segment(p.ctypes.data, p.size, C.byref(cfg), out, cap, C.byref(n)))
    return [(out[i].start, out[i].end) for i in range(n.value)]


class VadHead:
    """VadHead (vad.rs:7-82) on GPU `device`. Weights: proj_w [h, d(, 1)], proj_b [h], ctx_w [h, h, k], ctx_b [h],
    out_w [(1, )h(, 1)], out_b (float), as float arrays."""

    def __init__(self, w: dict, device: int = 0, frame_seconds: float = 0.08):
        pw = np.ascontiguousarray(w["proj_w"], np.float32)
        h = pw.shape[0]
        pw = pw.reshape(h, -1)
        cw = np.ascontiguousarray(w["ctx_w"], np.float32)
        self._keep = [pw, np.ascontiguousarray(w["proj_b"], np.float32), cw,
                      np.ascontiguousarray(w["ctx_b"], np.float32),
                      np.ascontiguousarray(w["out_w"], np.float32).reshape(h)]
        d = _Desc()
        d.d_model, d.hidden, d.kernel = pw.shape[1], h, cw.shape[2]
        d.proj_w, d.proj_b, d.ctx_w, d.ctx_b, d.out_w = [a.ctypes.data for a in self._keep]
        d.out_b, d.frame_seconds, d.device = float(np.float32(w["out_b"])), frame_seconds, int(device)
        h_ = _P()
        check(lib().vxg_vad_create(C.byref(d), C.byref(h_)))
        self._h, self.device = h_, int(device)
        self.d_model, self.hidden, self.kernel = d.d_model, h, d.kernel
        del self._keep

    @classmethod
    def from_model(cls, model, device: int = 0) -> "VadHead":
        """VadHead::load (vad.rs:21-36) from a model directory (a path or an open ModelFile)."""
        from .model import ModelFile

        mf = model if isinstance(model, ModelFile) else ModelFile.open(model)
        h = _P()
        check(lib().vxg_vad_create_from_model(mf._h, int(device), C.byref(h)))
        if mf is not model:
            mf.close()
        self = cls.__new__(cls)
        self._h, self.device = h, int(device)
        d, hid, k, fs = _I(), _I(), _I(), C.c_double()
        check(lib().vxg_vad_info(h, C.byref(d), C.byref(hid), C.byref(k), C.byref(fs)))
        self.d_model, self.hidden, self.kernel = d.value, hid.value, k.value
        return self

    def close(self):
        if getattr(self, "_h", None):
            lib().vxg_vad_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def probs_device(self, sub: torch.Tensor, frames=None) -> torch.Tensor:
        """VadHead::probs on stacked subsampler outputs sub [sum t, d_model] (CUDA f32), utterances of `frames`
        rows each (default: one utterance). Returns probs [sum t] on the device."""
        assert sub.is_cuda and sub.dtype == torch.float32 and sub.is_contiguous()
        t = np.ascontiguousarray([sub.shape[0]] if frames is None else frames, np.int32)
        out = torch.empty(sub.shape[0], dtype=torch.float32, device=sub.device)
        s = torch.cuda.current_stream(sub.device)
        check(lib().vxg_vad_probs_device(self._h, C.c_void_p(sub.data_ptr()), t.ctypes.data, len(t),
                                         C.c_void_p(out.data_ptr()), C.c_void_p(s.cuda_stream)))
        return out
