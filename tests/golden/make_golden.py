"""Regenerate the committed golden vectors under tests/golden/ (run in a container that has the reference mounted).

Sources, all from lmaksym/voxrt 0.2.1:
  * crates/voxrt/tests/fixtures/*: the reference's own real-weight codec fixtures (first rows of three ternary
    modules: packed qweight bytes, f16 scales, expected trits, expected dequantised f32), made by the reference's
    reference-py/make_fixtures.py from the real model. Copied byte for byte.
  * reference-py/trits.py: the reference's Python codec, imported here (not copied) to produce pack/unpack/dequant
    vectors on seeded random trit matrices with ragged widths -> codec_vectors.npz.

Usage: python tests/golden/make_golden.py /path/to/reference
"""
import json
import os
import shutil
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref):
    fx = os.path.join(ref, "crates/voxrt/tests/fixtures")
    meta = json.load(open(os.path.join(fx, "ternary_fixtures.json")))
    for tag in meta:
        for suffix in ("qweight.bin", "scales.f16.bin", "trits.i8.bin", "weight.f32.bin"):
            shutil.copyfile(os.path.join(fx, f"{tag}.{suffix}"), os.path.join(HERE, f"{tag}.{suffix}"))
    shutil.copyfile(os.path.join(fx, "ternary_fixtures.json"), os.path.join(HERE, "ternary_fixtures.json"))

    sys.path.insert(0, os.path.join(ref, "reference-py"))
    import trits as ref_trits  # the reference's own codec (reference-py/trits.py)

    rng = np.random.default_rng(20261201)
    out = {}
    for n in (1, 4, 5, 6, 127, 128, 1024, 4096):
        t = rng.integers(-1, 2, size=(7, n), dtype=np.int8)
        q = ref_trits.pack(t)
        out[f"pack_in_{n}"] = t
        out[f"pack_out_{n}"] = q
        out[f"unpack_{n}"] = ref_trits.unpack(q, n)
    t = rng.integers(-1, 2, size=(5, 256), dtype=np.int8)
    q = ref_trits.pack(t)
    s = (rng.uniform(0.01, 0.05, size=(5, 2))).astype(np.float16)
    out["dequant_q"] = q
    out["dequant_s"] = s.view(np.uint16)
    out["dequant_w"] = ref_trits.dequant(q, s, 256, 128)
    np.savez_compressed(os.path.join(HERE, "codec_vectors.npz"), **out)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
