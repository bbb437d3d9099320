"""A thrush-ternary-v2 model directory behind libvxg's C ABI, mirroring the reference's ModelFile
(crates/voxrt/src/format.rs:76-309): open (format / naming checks, safetensors header), validate (every tensor the
loaders read, by dtype and shape), config, tensor access; the encoder and decoder load from it directly
(CudaEncoder.from_model, TdtDecoder.from_model). All parsing runs in the library (C++)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib

_DTYPES = {0: np.float16, 1: None, 2: np.float32, 3: np.uint8, 4: np.int8}


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("d_model", "ff", "n_layers", "heads", "n_mels", "conv_kernel", "sub_channels",
                                        "group", "dec_hidden", "dec_layers", "vocab", "blank", "max_symbols",
                                        "n_durations", "vad_hidden", "vad_kernel")] + [("vad_frame_seconds",
                                                                                       C.c_double)]


class ModelFile:
    def __init__(self, handle, path):
        self._h, self.path = handle, path

    @classmethod
    def open(cls, path) -> "ModelFile":
        h = C.c_void_p()
        check(lib().vxg_model_open(str(path).encode(), C.byref(h)))
        return cls(h, str(path))

    def close(self):
        if self._h:
            lib().vxg_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def validate(self) -> list[str]:
        """ModelFile::validate: the mismatches (empty when every tensor is as the loaders expect)."""
        buf = C.create_string_buffer(1 << 20)
        n = lib().vxg_model_validate(self._h, buf, len(buf))
        return [s for s in buf.value.decode().split("\n") if s][:n]

    def config(self) -> dict:
        c = _Cfg()
        check(lib().vxg_model_config(self._h, C.byref(c)))
        return {n: getattr(c, n) for n, _ in _Cfg._fields_}

    def tensor(self, name: str) -> np.ndarray:
        """A copy of one tensor's data in its stored dtype and shape (BF16 as uint16 bits)."""
        dt, nd = C.c_int(), C.c_int()
        shape = (C.c_int64 * 8)()
        data, nbytes = C.c_void_p(), C.c_size_t()
        check(lib().vxg_model_tensor(self._h, name.encode(), C.byref(dt), shape, C.byref(nd), C.byref(data),
                                     C.byref(nbytes)))
        np_dt = _DTYPES.get(dt.value) or np.uint16
        raw = C.string_at(data.value, nbytes.value)
        return np.frombuffer(raw, np_dt).reshape([shape[i] for i in range(nd.value)]).copy()

    def tensor_f32(self, name: str) -> np.ndarray:
        """load_f32: the tensor widened to f32 (exactly, from F16 / BF16)."""
        t = self.tensor(name)
        out = np.empty(t.shape, np.float32)
        check(lib().vxg_model_tensor_f32(self._h, name.encode(), out.ctypes.data, out.size))
        return out
