"""Stand-alone timing of single kernels on cuda:0, for profiling them in isolation (ncu -k ... python -m
voxrt_b200.kernel_bench ...).

  ln      one LayerNorm -> int8 pass at the config-3 token count: vxg_ln_quant on x [12955, 1024] with a first
          LayerNorm written to x_out, then the second LayerNorm and the per-128 quantisation (the pass that opens
          every encoder layer after the first)
  linear  the subsampling's f32 linear in the reference's lane order: vxg_linear_f32 on x [M, K] (default the
          pointwise-conv shape 131072 x 256 -> 256, bias, ReLU)

Prints the CUDA-event time of `--reps` back-to-back launches after `--warmup` launches, and the throughput.
"""
from __future__ import annotations

import argparse
import ctypes as C

import torch

from voxrt_b200 import kernels
from voxrt_b200._lib import check, check_device, lib


def _time(fn, warmup: int, reps: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / max(1, reps)  # ms per launch


def bench_ln(rows: int, warmup: int, reps: int) -> None:
    d = 1024
    x = torch.randn((rows, d), device="cuda")
    g0, b0 = 1 + 0.1 * torch.randn(d, device="cuda"), 0.1 * torch.randn(d, device="cuda")
    g1, b1 = 1 + 0.1 * torch.randn(d, device="cuda"), 0.1 * torch.randn(d, device="cuda")
    x_out = torch.empty_like(x)
    ms = _time(lambda: kernels.ln_quant(x, g1, b1, pre=(g0, b0), x_out=x_out), warmup, reps)
    nbytes = rows * d * 4 * 2 + rows * d + rows * (d // 128) * 4  # x in, x_out + int8 codes + scales out
    print(f"ln_quant {rows}x{d}: {ms * 1e3:.1f} us per launch, {nbytes / ms / 1e6:.0f} GB/s of algorithmic bytes")


def bench_linear(m: int, k: int, n: int, warmup: int, reps: int) -> None:
    x = torch.randn((m, k), device="cuda")
    w = torch.randn((n, k), device="cuda") / k ** 0.5
    b = torch.randn(n, device="cuda")
    y = torch.empty((m, n), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())
    ms = _time(lambda: check(lib().vxg_linear_f32(P(x), m, k, P(w), P(b), n, 1, P(y), None)), warmup, reps)
    print(f"linear {m}x{n}x{k}: {ms * 1e3:.1f} us per launch, {2.0 * m * n * k / ms / 1e9:.1f} TFLOP/s")


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("kernel", choices=["ln", "linear"])
    ap.add_argument("--rows", type=int, default=12955, help="ln: rows")
    ap.add_argument("--mkn", type=int, nargs=3, default=[131072, 256, 256], help="linear: M K N")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args()
    assert torch.cuda.is_available(), "kernel_bench needs a CUDA device"
    torch.cuda.set_device(0)
    torch.manual_seed(0)
    if a.kernel == "ln":
        bench_ln(a.rows, a.warmup, a.reps)
    else:
        bench_linear(*a.mkn, a.warmup, a.reps)
    check_device()


if __name__ == "__main__":
    main()
