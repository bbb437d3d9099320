"""Input generators restating the reference's own kernel tests, so the parity cases use the same vectors.

crates/voxrt/tests/kernels.rs:14-33 (random_matrix) and crates/voxrt/tests/x86_kernels.rs:27-86
(ternary / int8 / acts), all driven by the reference's 64-bit LCG (kernels.rs:7-12).
"""
import numpy as np

from conftest import LCG
from voxrt_b200.synth import pack_trits


def lcg_trits(rng: LCG, out, inp, extreme=False):
    if extreme:
        return np.ones((out, inp), np.int8)
    return np.array([[rng.next() % 3 - 1 for _ in range(inp)] for _ in range(out)], np.int8)


def random_matrix(out, inp, rng: LCG):
    """kernels.rs:14-33: per row the trits, then per group one f16 scale 0.01 + (lcg % 100) * 0.001."""
    ng = inp // 128
    trits = np.zeros((out, inp), np.int8)
    s16 = np.zeros((out, ng), np.float16)
    for r in range(out):
        trits[r] = [rng.next() % 3 - 1 for _ in range(inp)]
        for g in range(ng):
            s16[r, g] = np.float16(np.float32(0.01) + np.float32(rng.next() % 100) * np.float32(0.001))
    return pack_trits(trits), s16.view(np.uint16), trits


def x86_ternary(out, inp, rng: LCG, extreme=False):
    """x86_kernels.rs:27-48: per row the trits then ng f16 scales."""
    ng = inp // 128
    trits = np.zeros((out, inp), np.int8)
    s16 = np.zeros((out, ng), np.float16)
    for r in range(out):
        trits[r] = 1 if extreme else [rng.next() % 3 - 1 for _ in range(inp)]
        for g in range(ng):
            s16[r, g] = np.float16(np.float32(0.01) + np.float32(rng.next() % 100) * np.float32(0.001))
    return trits, s16.astype(np.float32), s16.view(np.uint16)


def x86_int8(out, inp, group, rng: LCG, extreme=False):
    """x86_kernels.rs:50-68: arbitrary int8 rows (not ternary) with f32 scales."""
    n = out * inp
    if extreme:
        rows = np.where(np.arange(n) % 2 == 0, 127, -127).astype(np.int8)
    else:
        rows = np.array([(rng.next() % 255) - 127 for _ in range(n)], np.int32).astype(np.int8)
    scales = np.array([np.float32(0.001) + np.float32(rng.next() % 1000) * np.float32(1e-5)
                       for _ in range(out * (inp // group))], np.float32)
    return rows.reshape(out, inp), scales.reshape(out, inp // group)


def acts_f32(n, inp, rng: LCG, extreme=False, div=100.0, off=10.0):
    """x86_kernels.rs:70-85 / kernels.rs:42-44: (lcg % 2001) / 100 - 10 (or +-5 extremes)."""
    if extreme:
        return np.where(np.arange(n * inp) % 2 == 0, 5.0, -5.0).astype(np.float32).reshape(n, inp)
    v = [np.float32(rng.next() % 2001) / np.float32(div) - np.float32(off) for _ in range(n * inp)]
    return np.array(v, np.float32).reshape(n, inp)
