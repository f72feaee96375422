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


def gguf_tensors(path):
    """The tensor index of a GGUF v3 file: [(name, ggml type, dims (innermost first), bytes)] -- the header layout
    of crates/core/src/gguf.rs:483, read independently of the library."""
    import struct

    with open(path, "rb") as f:
        buf = f.read(64 << 20)
    o = 0

    def take(fmt):
        nonlocal o
        v = struct.unpack_from("<" + fmt, buf, o)
        o += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string():
        nonlocal o
        n = take("Q")
        s = buf[o:o + n].decode()
        o += n
        return s

    scalar = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}

    def value(t):
        if t == 8:
            return string()
        if t == 9:
            et, n = take("I"), take("Q")
            return [value(et) for _ in range(n)]
        return take(scalar[t])

    assert buf[:4] == b"GGUF" and take("4sI")[1] == 3
    n_t, n_kv = take("Q"), take("Q")
    for _ in range(n_kv):
        string()
        value(take("I"))
    out = []
    for _ in range(n_t):
        name = string()
        dims = [take("Q") for _ in range(take("I"))]
        t = take("I")
        take("Q")
        n = int(np.prod(dims))
        be, bb = {0: (1, 4), 1: (1, 2), **LAYOUT}[t]
        out.append((name, t, dims, n // be * bb))
    return out
