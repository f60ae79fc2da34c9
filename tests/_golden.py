"""Helpers to read the fixtures written by tests/golden/make_golden.py."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def cases(name):
    z = load(name)
    n = int(z["n"])
    out = []
    for i in range(n):
        pre = f"c{i}_"
        out.append({k[len(pre):]: z[k] for k in z.files if k.startswith(pre)})
    return out


def bf16_from_i16(a):
    """int16 bit patterns of bf16 values -> float32 array."""
    return (np.asarray(a).astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
