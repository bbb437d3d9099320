"""The NeMo log-mel frontend on the GPU behind libvxg's C ABI, mirroring the reference's Frontend
(crates/voxrt/src/frontend.rs:36-200): compute (normalised features) and log_mel (before normalisation) for a batch
of utterances stacked along the sample axis."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib

HOP = 160


class Frontend:
    def __init__(self, n_mels: int = 128, device: int = 0, sample_rate: int = 16000):
        h = C.c_void_p()
        check(lib().vxg_frontend_create(sample_rate, n_mels, device, C.byref(h)))
        self._h, self.n_mels, self.device = h, n_mels, device

    def close(self):
        if self._h:
            lib().vxg_frontend_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def n_frames(n_samples: int) -> int:
        return int(n_samples) // HOP

    def compute_device(self, samples, lengths, feats=None, normalize: bool = True, stream=None):
        """samples: torch CUDA f32 tensor of the stacked utterances; lengths: samples per utterance. Returns
        (feats [sum frames, n_mels] CUDA tensor, frames per utterance)."""
        import torch

        lengths = np.ascontiguousarray(lengths, np.int64)
        nfr = lengths // HOP
        if feats is None:
            feats = torch.empty((int(nfr.sum()), self.n_mels), dtype=torch.float32, device=samples.device)
        out_n = np.empty(len(lengths), np.int32)
        s = stream if stream is not None else torch.cuda.current_stream()
        check(lib().vxg_frontend_device(self._h, C.c_void_p(samples.data_ptr()), lengths.ctypes.data, len(lengths),
                                        int(bool(normalize)), C.c_void_p(feats.data_ptr()), out_n.ctypes.data,
                                        C.c_void_p(s.cuda_stream)))
        return feats, out_n

    def compute(self, waves, normalize: bool = True):
        """Frontend::compute for host arrays: a list of 1-D f32 sample arrays -> list of [frames, n_mels] arrays."""
        import torch

        lens = np.array([len(w) for w in waves], np.int64)
        dev = torch.device("cuda", self.device)
        x = torch.from_numpy(np.concatenate([np.asarray(w, np.float32) for w in waves])).to(dev)
        f, n = self.compute_device(x, lens, normalize=normalize)
        f = f.cpu().numpy()
        offs = np.concatenate([[0], np.cumsum(n)])
        return [f[offs[i]:offs[i + 1]] for i in range(len(waves))]


def filterbank(sample_rate: int = 16000, n_fft: int = 512, n_mels: int = 128) -> np.ndarray:
    """slaney_mel_filterbank as the library computes it (host)."""
    fb = np.empty((n_mels, n_fft // 2 + 1), np.float32)
    check(lib().vxg_mel_filterbank(sample_rate, n_fft, n_mels, fb.ctypes.data))
    return fb
