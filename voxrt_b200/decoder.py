"""TDT decoder behind libvxg's C ABI, mirroring the reference's Decoder (crates/voxrt/src/decoder.rs): load from a
model dict, project_encoder (on the GPU), greedy (host threads, as the reference), pred_step and joint for parity
checks. Weight dict keys follow the model file's tensor names (decoder.lstm.*, joint.head.*, encoder_projector.*).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import check, lib

_P, _I = C.c_void_p, C.c_int


class _Desc(C.Structure):
    _fields_ = [("hidden", _I), ("vocab", _I), ("n_durations", _I), ("blank", _I), ("max_symbols", _I),
                ("d_model", _I), ("n_layers", _I), ("durations", _P), ("embedding", _P), ("w_ih", _P * 4),
                ("w_hh", _P * 4), ("b_ih", _P * 4), ("b_hh", _P * 4), ("proj_w", _P), ("proj_b", _P),
                ("head_w", _P), ("head_b", _P), ("enc_w", _P), ("enc_b", _P), ("device", _I)]


class _Emission(C.Structure):
    _fields_ = [("token", C.c_int32), ("frame", C.c_int32), ("duration", C.c_int32)]


def _arr(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class TdtDecoder:
    """Decoder::load (decoder.rs:61-110) in int8 mode. `device` is the GPU for project_device (None: host only)."""

    def __init__(self, m: dict, device: int | None = None):
        keep = []

        def ptr(a, dtype):
            a = _arr(a, dtype)
            keep.append(a)
            return a.ctypes.data

        d = _Desc()
        d.hidden, d.vocab, d.n_durations = m["hidden"], m["vocab"], len(m["durations"])
        d.blank, d.max_symbols, d.d_model, d.n_layers = m["blank"], m["max_symbols"], m["d_model"], len(m["lstm"])
        d.durations = ptr(m["durations"], np.int32)
        d.embedding = ptr(m["embedding"], np.float32)
        for l, layer in enumerate(m["lstm"]):
            d.w_ih[l] = ptr(np.asarray(layer["w_ih"]).view(np.uint16), np.uint16)
            d.w_hh[l] = ptr(np.asarray(layer["w_hh"]).view(np.uint16), np.uint16)
            d.b_ih[l] = ptr(layer["b_ih"], np.float32)
            d.b_hh[l] = ptr(layer["b_hh"], np.float32)
        d.proj_w = ptr(np.asarray(m["proj_w"]).view(np.uint16), np.uint16)
        d.proj_b = ptr(m["proj_b"], np.float32)
        d.head_w = ptr(np.asarray(m["head_w"]).view(np.uint16), np.uint16)
        d.head_b = ptr(m["head_b"], np.float32)
        d.enc_w = ptr(m["enc_w"], np.float32)
        d.enc_b = ptr(m["enc_b"], np.float32)
        d.device = -1 if device is None else int(device)
        h = _P()
        check(lib().vxg_tdt_create(C.byref(d), C.byref(h)))
        self._h = h
        self.hidden, self.vocab, self.n_dur = d.hidden, d.vocab, d.n_durations
        self.n_layers, self.device, self.max_symbols = d.n_layers, device, d.max_symbols

    @classmethod
    def from_model(cls, model, device: int | None = None) -> "TdtDecoder":
        """Decoder::load (decoder.rs:57-110) from a model directory (a path or an open ModelFile)."""
        from .model import ModelFile

        mf = model if isinstance(model, ModelFile) else ModelFile.open(model)
        cfg = mf.config()
        h = _P()
        check(lib().vxg_tdt_create_from_model(mf._h, -1 if device is None else int(device), C.byref(h)))
        if mf is not model:
            mf.close()
        self = cls.__new__(cls)
        self._h = h
        self.hidden, self.vocab, self.n_dur = cfg["dec_hidden"], cfg["vocab"], cfg["n_durations"]
        self.n_layers, self.device, self.max_symbols = cfg["dec_layers"], device, cfg["max_symbols"]
        return self

    def close(self):
        if getattr(self, "_h", None):
            lib().vxg_tdt_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def project_device(self, enc: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Decoder::project_encoder (decoder.rs:123-134) on the GPU: enc [t, d_model] -> [t, hidden] (f32)."""
        assert enc.is_cuda and enc.dtype == torch.float32 and enc.is_contiguous()
        t = enc.shape[0]
        if out is None:
            out = torch.empty((t, self.hidden), dtype=torch.float32, device=enc.device)
        s = stream if stream is not None else torch.cuda.current_stream()
        check(lib().vxg_tdt_project_device(self._h, C.c_void_p(enc.data_ptr()), t, C.c_void_p(out.data_ptr()),
                                           C.c_void_p(s.cuda_stream)))
        return out

    @staticmethod
    def _cap(t: int) -> int:
        return max(1, t * 10 + 16)

    def greedy(self, proj: np.ndarray) -> np.ndarray:
        """Decoder::greedy (decoder.rs:204-266): [n, 3] int32 rows of (token, frame, duration)."""
        proj = _arr(proj, np.float32)
        t = proj.shape[0]
        cap = self._cap(t)
        out = (_Emission * cap)()
        n = C.c_size_t(0)
        check(lib().vxg_tdt_greedy(self._h, proj.ctypes.data, t, out, cap, C.byref(n)))
        assert n.value <= cap
        return np.array([(e.token, e.frame, e.duration) for e in out[:n.value]], np.int32).reshape(-1, 3)

    def greedy_batch(self, projs, threads: int = 0):
        """Many utterances on host threads; the same results as greedy() per utterance."""
        projs = [_arr(p, np.float32) for p in projs]
        n = len(projs)
        t = np.array([p.shape[0] for p in projs], np.int32)
        caps = np.array([self._cap(int(x)) for x in t], np.uint64)
        outs = [(_Emission * int(c))() for c in caps]
        pp = (_P * n)(*[p.ctypes.data for p in projs])
        op = (_P * n)(*[C.cast(o, _P) for o in outs])
        nout = np.zeros(n, np.uint64)
        check(lib().vxg_tdt_greedy_batch(self._h, n, pp, t.ctypes.data, op, caps.ctypes.data, nout.ctypes.data,
                                         int(threads)))
        res = []
        for o, k in zip(outs, nout):
            assert k <= len(o)
            res.append(np.array([(e.token, e.frame, e.duration) for e in o[:int(k)]], np.int32).reshape(-1, 3))
        return res

    def greedy_device(self, proj: torch.Tensor, frames, stream=None, per_frame: int = 2, timings: dict | None = None):
        """Decoder::greedy for every utterance of a stacked projection proj [sum frames, hidden] (CUDA, f32) on the
        decoder's GPU, in lockstep rounds (vxg_tdt_greedy_device). Each utterance first gets room for
        per_frame * frames + 16 emissions; utterances that emitted more are decoded again with room for the most
        the loop can emit (frames * max_symbols). Returns a list of [n, 3] int32 arrays like greedy(). `timings`
        (a dict) receives the wall seconds of the decode call(s), of the copies to the host and the number of
        utterances decoded again."""
        import time
        assert proj.is_cuda and proj.dtype == torch.float32 and proj.is_contiguous()
        frames = np.ascontiguousarray(frames, np.int32)
        n = len(frames)
        offs = np.concatenate([[0], np.cumsum(frames, dtype=np.int64)])
        assert proj.shape[0] >= offs[-1] and (n == 0 or proj.shape[1] == self.hidden)
        s = stream if stream is not None else torch.cuda.current_stream(proj.device)

        def run(idx, caps):
            fr = np.ascontiguousarray(frames[idx], np.int32)
            if len(idx) == n:
                pr = proj
            else:
                pr = torch.cat([proj[int(offs[u]):int(offs[u + 1])] for u in idx]) if len(idx) else proj[:0]
            caps = np.ascontiguousarray(caps, np.uint64)
            eo = np.concatenate([[0], np.cumsum(caps.astype(np.int64))]).astype(np.int64)
            out = torch.empty((max(1, int(eo[-1])), 3), dtype=torch.int32, device=proj.device)
            cnt = torch.empty(max(1, len(idx)), dtype=torch.int32, device=proj.device)
            t0 = time.perf_counter()
            with torch.cuda.stream(s):
                check(lib().vxg_tdt_greedy_device(self._h, len(idx), C.c_void_p(pr.data_ptr()), fr.ctypes.data,
                                                  C.c_void_p(out.data_ptr()), caps.ctypes.data,
                                                  C.c_void_p(cnt.data_ptr()), C.c_void_p(s.cuda_stream)))
            s.synchronize()
            t1 = time.perf_counter()
            res = out.cpu().numpy(), cnt.cpu().numpy()[:len(idx)], eo
            if timings is not None:
                timings["decode_call_s"] = timings.get("decode_call_s", 0.0) + t1 - t0
                timings["to_host_s"] = timings.get("to_host_s", 0.0) + time.perf_counter() - t1
            return res

        caps = frames.astype(np.int64) * per_frame + 16
        out, cnt, eo = run(np.arange(n), caps)
        res = [out[eo[u]:eo[u] + min(int(cnt[u]), int(caps[u]))].copy() for u in range(n)]
        again = [u for u in range(n) if cnt[u] > caps[u]]
        if timings is not None:
            timings["redecoded"] = len(again)
        if again:
            full = frames[again].astype(np.int64) * self.max_symbols + 16
            out2, cnt2, eo2 = run(np.array(again), full)
            for i, u in enumerate(again):
                assert cnt2[i] <= full[i]
                res[u] = out2[eo2[i]:eo2[i] + int(cnt2[i])].copy()
        return res

    def pred_step_device(self, tokens: torch.Tensor, h: torch.Tensor, c: torch.Tensor):
        """The GPU decode's prediction-network step for n inputs: tokens [n] int32, h, c [n, n_layers, hidden]."""
        n = tokens.shape[0]
        g = torch.empty((n, self.hidden), dtype=torch.float32, device=h.device)
        hn, cn = torch.empty_like(h), torch.empty_like(c)
        s = torch.cuda.current_stream(h.device)
        check(lib().vxg_tdt_pred_step_device(self._h, n, *[C.c_void_p(x.data_ptr()) for x in (tokens, h, c, g, hn, cn)],
                                             C.c_void_p(s.cuda_stream)))
        return g, hn, cn

    def joint_device(self, enc: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
        """The GPU decode's joint evaluation for n inputs: enc, g [n, hidden] -> logits [n, vocab + n_durations]."""
        n = enc.shape[0]
        out = torch.empty((n, self.vocab + self.n_dur), dtype=torch.float32, device=enc.device)
        s = torch.cuda.current_stream(enc.device)
        check(lib().vxg_tdt_joint_device(self._h, n, C.c_void_p(enc.data_ptr()), C.c_void_p(g.data_ptr()),
                                         C.c_void_p(out.data_ptr()), C.c_void_p(s.cuda_stream)))
        return out

    def pred_step(self, token: int, h: np.ndarray, c: np.ndarray):
        h, c = _arr(h, np.float32), _arr(c, np.float32)
        g = np.empty(self.hidden, np.float32)
        hn, cn = np.empty_like(h), np.empty_like(c)
        check(lib().vxg_tdt_pred_step(self._h, int(token), h.ctypes.data, c.ctypes.data, g.ctypes.data,
                                      hn.ctypes.data, cn.ctypes.data))
        return g, hn, cn

    def joint(self, enc_t: np.ndarray, g: np.ndarray) -> np.ndarray:
        enc_t, g = _arr(enc_t, np.float32), _arr(g, np.float32)
        out = np.empty(self.vocab + self.n_dur, np.float32)
        check(lib().vxg_tdt_joint(self._h, enc_t.ctypes.data, g.ctypes.data, out.ctypes.data))
        return out
