"""Loader for the golden vectors in tests/golden (extracted from the reference fixtures by make_golden.py)."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
EPS = float(np.finfo(np.float32).eps)


def load(group):
    with open(os.path.join(GOLDEN, group + ".json")) as f:
        meta = json.load(f)
    arrs = np.load(os.path.join(GOLDEN, group + ".npz"))
    return meta, arrs


def budget(k, width, max_abs):
    """k * sqrt(n) * eps * max|term| (crates/core/tests/kernels.rs:49-51)."""
    return k * np.sqrt(width) * EPS * max_abs


def kquant_terms_budget(t, wrow, w_deq, x_deq, k, f16):
    """k * eps * sum_j (|w_j + min_j| + |min_j|) |x_j| (crates/core/tests/common/mod.rs:112-131)."""
    width = w_deq.size
    nsb = width // 256
    bb = wrow.size // nsb
    mags = 0.0
    for sb in range(nsb):
        wb = wrow[sb * bb:(sb + 1) * bb]
        if t == 14:
            dmin = 0.0
        else:
            dmin = float(f16(int(wb[2]) | (int(wb[3]) << 8)))
        for s in range(8):
            if t == 14:
                m = 0
            else:
                q = wb[4:16]
                m = (q[s + 4] & 63) if s < 4 else ((q[s + 4] >> 4) | ((q[s] >> 6) << 4))
            mp = dmin * float(m)
            sl = slice(sb * 256 + s * 32, sb * 256 + (s + 1) * 32)
            mags += float(np.sum((np.abs(w_deq[sl].astype(np.float64) + mp) + abs(mp)) * np.abs(x_deq[sl].astype(np.float64))))
    return k * EPS * mags
