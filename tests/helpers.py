"""Test helpers: seeded random ggml blocks and device transfer helpers."""
import numpy as np

LAYOUT = {0: (1, 4), 2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210)}
SCALE_OFFSETS = {12: (0, 2), 13: (0, 2), 14: (208,), 8: (0,), 2: (0,)}


def row_bytes(t, cols):
    be, bb = LAYOUT[t]
    return cols // be * bb


def random_blocks(t, rows, cols, seed, exp_lo=12, exp_hi=19):
    """Random block bytes whose f16 scale fields are finite, exponent forced into [2^(lo-15), 2^(hi-15))
    (the device of crates/core/tests/q8k.rs finite_weights; random bytes alone include inf/NaN scales)."""
    rng = np.random.default_rng(seed)
    if t == 0:
        return rng.standard_normal((rows, cols), dtype=np.float32).view(np.uint8).reshape(-1)
    be, bb = LAYOUT[t]
    data = rng.integers(0, 256, size=rows * (cols // be) * bb, dtype=np.uint8).reshape(-1, bb)
    for off in SCALE_OFFSETS[t]:
        bits = data[:, off].astype(np.uint16) | (data[:, off + 1].astype(np.uint16) << 8)
        exp = exp_lo + (bits >> 10) % (exp_hi - exp_lo)
        fixed = (bits & 0x83FF) | (exp << 10)
        data[:, off] = (fixed & 0xFF).astype(np.uint8)
        data[:, off + 1] = (fixed >> 8).astype(np.uint8)
    return data.reshape(-1)


def hostile_rows(width, seed):
    """Activation rows of the reference's hostile set (crates/core/tests/q8k.rs hostile_acts)."""
    rng = np.random.default_rng(seed)
    r = lambda s: (rng.standard_normal(width) * s).astype(np.float32)
    rows = [r(1.0), r(1e30), r(1e-30), np.full(width, 3.0, np.float32), np.full(width, -0.0, np.float32),
            np.array([5.0 if i % 2 == 0 else -5.0 for i in range(width)], np.float32)]
    ties = np.array([(i % 9) - 4 + 0.5 for i in range(width)], np.float32)
    ties[0] = -127.0
    ties[300 % width] = 127.0
    rows.append(ties)
    pm = r(0.5)
    pm[7], pm[9] = 4.0, -4.0
    rows.append(pm.copy())
    pm[7], pm[9] = -4.0, 4.0
    rows.append(pm)
    z = r(1.0)
    z[256:min(512, width)] = 0.0
    rows.append(z)
    return np.stack(rows)


def to_dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits_equal(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))
