"""Reader for the reference's golden tensors (raw float32, numpy .tofile()).

The format is the one tests/golden_io.mojo:1-25 of the reference reads: a flat
little-endian float32 array per file; the shapes live in the family's .txt.
"""

import os

import numpy as np

REF = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref")


def read_f32(name, shape=None):
    path = os.path.join(REF, name if name.endswith(".bin") else name + ".bin")
    raw = np.fromfile(path, dtype="<f4")
    if shape is not None:
        raw = raw.reshape(shape)
    return raw


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def max_rel_of_max(got, want):
    """Largest |got - want| relative to max |want| (the reference's gradient metric,
    tests/test_actor_backward.mojo:59-71)."""
    want = np.asarray(want, np.float64)
    den = max(float(np.max(np.abs(want))), 1e-30)
    return max_abs(got, want) / den
