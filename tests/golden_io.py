"""Loader for the committed golden vectors (produced by tests/golden/make_golden.py)."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def rel_rowsign(a, b):
    """Relative Frobenius distance after matching the sign of each row of a to b."""
    a = np.asarray(a, np.float64).copy()
    b = np.asarray(b, np.float64)
    s = np.sign(np.sum(a * b, axis=1))
    s[s == 0] = 1
    return rel(a * s[:, None], b)
