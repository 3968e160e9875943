#!/usr/bin/env python3
"""Re-serialise the reference project's kernel golden vectors into one .npz.

The reference stores each tensor of tests/kern_golden/ as
    [u32 rank][u32 dims x rank][little-endian data]   (.f32: float32, .f16: fp16 bits)
(format written by tools/export_kern_golden.py:26-36, read by
tests/test_kern.cpp:36-57).  The vectors come from torch on the reference
author's machine with seed 20250823 (export_kern_golden.py:23):
    gemv_a (128x96), gemv_b (33x131): y = w.float() @ x
    rms_*, ln_*, sm_*, act_*, rope_*: the support primitives.

Run once on a machine that has the reference tree; the .npz it writes
(kern_golden.npz next to this script) is the committed fixture, so nothing
at test time reads the reference tree.

    python tests/golden/make_golden.py path/to/reference
"""
import os
import struct
import sys

import numpy as np

NAMES = [
    ("gemv_a_w", "f16"), ("gemv_a_x", "f32"), ("gemv_a_y", "f32"),
    ("gemv_b_w", "f16"), ("gemv_b_x", "f32"), ("gemv_b_y", "f32"),
    ("rms_x", "f32"), ("rms_g", "f32"), ("rms_y", "f32"),
    ("ln_x", "f32"), ("ln_g", "f32"), ("ln_b", "f32"), ("ln_y", "f32"),
    ("sm_x", "f32"), ("sm_y", "f32"),
    ("act_v", "f32"), ("act_silu", "f32"), ("act_relu", "f32"),
    ("rope_in", "f32"), ("rope_gptj_out", "f32"), ("rope_neox_out", "f32"),
]


def load(path: str, ext: str) -> np.ndarray:
    with open(path, "rb") as f:
        raw = f.read()
    (rank,) = struct.unpack_from("<I", raw, 0)
    dims = struct.unpack_from(f"<{rank}I", raw, 4)
    off = 4 + 4 * rank
    dt = np.dtype("<u2") if ext == "f16" else np.dtype("<f4")
    n = int(np.prod(dims)) if rank else 1
    arr = np.frombuffer(raw, dtype=dt, count=n, offset=off).reshape(dims)
    return arr.astype(np.uint16 if ext == "f16" else np.float32)


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py path/to/reference")
    ref = sys.argv[1]
    src = os.path.join(ref, "tests", "kern_golden")
    out = {}
    for name, ext in NAMES:
        out[name] = load(os.path.join(src, f"{name}.{ext}"), ext)
        print(f"  {name}.{ext} {list(out[name].shape)}")
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kern_golden.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst)


if __name__ == "__main__":
    main()
