"""Long-form / streaming transcription behind libvxg's C ABI, mirroring crates/voxrt/src/longform.rs (LongForm:
push, flush, the closed segments' ranges) and Transcriber::transcribe_long (transcriber.rs:356-420). Segments are
absolute sample ranges; transcriptions are TDT emissions in absolute encoder frames (text is out of scope)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib
from .vad import SegmentConfig

_P, _I = C.c_void_p, C.c_int
BLOCK_FN = C.CFUNCTYPE(C.c_longlong, C.c_void_p, C.POINTER(C.c_float), C.c_longlong, C.c_longlong, C.c_longlong,
                       C.POINTER(C.c_float))


class LongFormConfig(C.Structure):
    _fields_ = [("seg", SegmentConfig), ("block_samples", C.c_longlong), ("ctx_samples", C.c_longlong),
                ("samples_per_frame", _I), ("sample_rate", _I), ("long_form_threshold_s", C.c_double),
                ("collect_only", _I)]

    def __init__(self, **kw):
        super().__init__()
        lib().vxg_longform_cfg_default(C.byref(self))
        for k, v in kw.items():
            if k in SegmentConfig().as_dict():
                setattr(self.seg, k, v)
            else:
                setattr(self, k, v)


class _Em(C.Structure):
    _fields_ = [("token", C.c_int32), ("frame", C.c_int32), ("duration", C.c_int32)]


def _ems(buf, n):
    return np.array([(e.token, e.frame, e.duration) for e in buf[:n]], np.int32).reshape(-1, 3)


class LongForm:
    """LongForm over the library's GPU components (frontend, encoder, VAD head, decoder), or, with `vad_fn`, over
    an external VAD: vad_fn(block: np.ndarray f32, skip, want) -> probabilities of frames [skip, skip + want) of the
    block (collect-only)."""

    def __init__(self, frontend=None, encoder=None, vad=None, decoder=None, cfg: LongFormConfig | None = None,
                 vad_fn=None):
        self.cfg = cfg or LongFormConfig()
        h = _P()
        if vad_fn is not None:
            def cb(user, samples, n, skip, want, out):
                try:
                    blk = np.ctypeslib.as_array(samples, shape=(n,)).copy() if n else np.zeros(0, np.float32)
                    p = np.ascontiguousarray(vad_fn(blk, int(skip), int(want)), np.float32)[:want]
                    for i, v in enumerate(p):
                        out[i] = float(v)
                    return len(p)
                except Exception:  # reported as a failed call
                    return -1
            self._cb = BLOCK_FN(cb)
            check(lib().vxg_longform_create_with_vad(self._cb, None, C.byref(self.cfg), C.byref(h)))
        else:
            check(lib().vxg_longform_create(frontend._h, encoder._h, vad._h, decoder._h if decoder else None,
                                            C.byref(self.cfg), C.byref(h)))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().vxg_longform_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _pairs(buf, n):
        return [(int(buf[2 * i]), int(buf[2 * i + 1])) for i in range(n)]

    def push(self, samples) -> list[tuple[int, int]]:
        """Feed audio; returns the segments (absolute sample ranges) this call closed."""
        x = np.ascontiguousarray(samples, np.float32)
        cap = 64
        buf = (C.c_longlong * (2 * cap))()
        n = C.c_size_t(0)
        check(lib().vxg_longform_push(self._h, x.ctypes.data, x.size, buf, cap, C.byref(n)))
        if n.value > cap:
            return self.ranges()[-n.value:]
        return self._pairs(buf, n.value)

    def flush(self) -> list[tuple[int, int]]:
        cap = 64
        buf = (C.c_longlong * (2 * cap))()
        n = C.c_size_t(0)
        check(lib().vxg_longform_flush(self._h, buf, cap, C.byref(n)))
        if n.value > cap:
            return self.ranges()[-n.value:]
        return self._pairs(buf, n.value)

    def ranges(self) -> list[tuple[int, int]]:
        n = C.c_size_t(0)
        check(lib().vxg_longform_ranges(self._h, None, 0, C.byref(n)))
        buf = (C.c_longlong * (2 * max(1, n.value)))()
        check(lib().vxg_longform_ranges(self._h, buf, n.value, C.byref(n)))
        return self._pairs(buf, n.value)

    def emissions(self) -> np.ndarray:
        n = C.c_size_t(0)
        check(lib().vxg_longform_emissions(self._h, None, 0, C.byref(n)))
        buf = (_Em * max(1, n.value))()
        check(lib().vxg_longform_emissions(self._h, buf, n.value, C.byref(n)))
        return _ems(buf, n.value)

    def stats(self) -> dict:
        mp, bs, npb = C.c_longlong(), C.c_longlong(), C.c_longlong()
        check(lib().vxg_longform_stats(self._h, C.byref(mp), C.byref(bs), C.byref(npb)))
        return {"max_pending": mp.value, "base_sample": bs.value, "n_probs": npb.value}


def transcribe_long(frontend, encoder, vad, decoder, samples, cfg: LongFormConfig | None = None):
    """Transcriber::transcribe_long: (emissions [n, 3] in absolute encoder frames, segment sample ranges)."""
    cfg = cfg or LongFormConfig()
    x = np.ascontiguousarray(samples, np.float32)
    spf = cfg.samples_per_frame
    cap = max(16, (x.size // spf + 2) * 10 + 64)
    rcap = max(4, x.size // spf + 4)
    em = (_Em * cap)()
    rg = (C.c_longlong * (2 * rcap))()
    n, nr = C.c_size_t(0), C.c_size_t(0)
    check(lib().vxg_transcribe_long(frontend._h, encoder._h, vad._h, decoder._h, x.ctypes.data, x.size,
                                    C.byref(cfg), em, cap, C.byref(n), rg, rcap, C.byref(nr)))
    assert n.value <= cap and nr.value <= rcap
    return _ems(em, n.value), LongForm._pairs(rg, nr.value)
