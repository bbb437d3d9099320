"""The correctly rounded f32 exp and tanh (crmath.cuh) that replace the reference's libm calls in the decoder and the
VAD head: the library's host evaluation against the oracle's extended-precision one on a strided sample of all f32
inputs plus every input of the tie tables and the special values (CPU; the full 2^32 comparison is recorded in the
design notes), and the device evaluation against the host one on every f32 input (GPU)."""
import os
import re

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
TABLES = os.path.join(os.path.dirname(HERE), "voxrt_b200", "csrc", "crmath_tables.h")


def _tie_inputs():
    src = open(TABLES).read()
    out = {}
    for name in ("Exp", "Tanh"):
        m = re.search(r"k%sTieTable\[\d+\] = \{([^}]*)\}" % name, src)
        vals = [int(v.rstrip("u"), 16) for v in re.findall(r"0x[0-9a-f]+u", m.group(1))]
        out[name] = np.array(vals[0::2], np.uint32) if len(vals) > 2 or vals[0] != 0xFFFFFFFF else np.zeros(0, np.uint32)
    return out


def _same(a, b):
    na = np.isnan(a)
    return bool(np.array_equal(na, np.isnan(b)) and np.array_equal(a[~na].view(np.uint32), b[~na].view(np.uint32)))


def _host(fn, x):
    from voxrt_b200._lib import check, lib

    y = np.empty_like(x)
    check(lib().vxg_math_host(fn, x.ctypes.data, x.size, y.ctypes.data))
    return y


def test_host_matches_extended_precision_sample(oracle_lib):
    ties = _tie_inputs()
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1.17549435e-38, 88.7228, 88.72284,
                        -87.33654, -103.9720, -103.97208, -104.0, 89.0, 9.01, 9.02, 0.25, 0.2499999, 20.0, 3.4e38,
                        -3.4e38], np.float32)
    stride = (np.arange(0, 1 << 32, 97, dtype=np.uint64)).astype(np.uint32)
    for fn, name in ((0, "Exp"), (1, "Tanh")):
        x = np.concatenate([stride, ties[name], special.view(np.uint32)]).view(np.float32)
        assert _same(_host(fn, x), oracle_lib.math_cr(fn, x)), name
    assert len(ties["Exp"]) > 0 and len(ties["Tanh"]) > 0


@pytest.mark.gpu
def test_device_matches_host_on_every_input():
    import torch

    from voxrt_b200._lib import check, check_device, lib

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ch = 1 << 28
    xd = torch.empty(ch, dtype=torch.float32, device="cuda")
    yd = torch.empty_like(xd)
    for c in range(1 << 32 >> 28):
        x = (np.arange(ch, dtype=np.uint64) + c * ch).astype(np.uint32).view(np.float32)
        xd.copy_(torch.from_numpy(x))
        for fn in (0, 1):
            check(lib().vxg_math_device(fn, xd.data_ptr(), ch, yd.data_ptr(), None))
            assert _same(yd.cpu().numpy(), _host(fn, x)), (fn, c)
    check_device()
