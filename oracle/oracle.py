"""ctypes binding of the CPU oracle (test infrastructure).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import this module; the product
(the `qdec` library) never does.  The library is built from oracle/*.c by oracle/Makefile into
oracle/_build/liboracle.so.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

F32, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 2, 8, 12, 13, 14
TYPE_IDS = {"F32": F32, "Q4_0": Q4_0, "Q8_0": Q8_0, "Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K}
LAYOUT = {F32: (1, 4), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}
LIBM_CR, LIBM_GLIBC = 0, 1

_lib = None


def build():
    """Compile the oracle (make -C oracle); a no-op when it is up to date."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I, F, S, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_uint32
        sig = {
            "oracle_set_libm": (None, [I]),
            "oracle_get_libm": (I, []),
            "oracle_set_threads": (None, [I]),
            "oracle_f16_to_f32": (F, [ctypes.c_uint16]),
            "oracle_f32_to_f16": (ctypes.c_uint16, [F]),
            "oracle_expf": (F, [F]),
            "oracle_dequantize": (I, [I, P, S, P, S]),
            "oracle_quantize_q8k": (None, [P, I, P]),
            "oracle_quantize_q8_0": (None, [P, I, P]),
            "oracle_dot": (F, [I, P, P, I]),
            "oracle_matmul_f32in": (None, [I, P, I, I, P, I, P]),
            "oracle_matmul_act": (None, [I, P, I, I, P, S, I, P]),
            "oracle_rmsnorm": (None, [P, P, I, F, P]),
            "oracle_rmsnorm_gated": (None, [P, P, P, I, F, P]),
            "oracle_swiglu": (None, [P, P, I, P]),
            "oracle_softmax": (None, [P, I, P]),
            "oracle_inv_freq": (None, [I, F, P]),
            "oracle_cos_sin": (None, [U, P, I, P, P]),
            "oracle_apply_rope": (None, [P, I, I, I, P, P]),
            "oracle_conv1d_step": (None, [P, P, I, P, I, P, I]),
            "oracle_l2norm": (None, [P, I, F]),
            "oracle_gate_g": (F, [F, F, F]),
            "oracle_gate_beta": (F, [F]),
            "oracle_deltanet_step": (None, [P, P, P, I, I, F, F, P, P]),
            "oracle_argmax": (U, [P, I]),
            "oracle_crc32": (U, [P, S]),
            "oracle_silu": (F, [F]),
        }
        U32P = ctypes.POINTER(ctypes.c_uint32)
        sig.update({
            "oracle_model_open": (P, [ctypes.c_char_p, ctypes.c_char_p, I]),
            "oracle_model_close": (None, [P]),
            "oracle_model_dims": (I, [P, ctypes.POINTER(ctypes.c_int)]),
            "oracle_state_new": (P, [P, I]),
            "oracle_state_free": (None, [P]),
            "oracle_state_pos": (I, [P]),
            "oracle_last_round_seconds": (ctypes.c_double, []),
            "oracle_forward_token": (I, [P, ctypes.c_uint32, P, P, P]),
            "oracle_generate": (I, [P, U32P, I, I, I, U32P]),
            "oracle_spec_generate": (I, [P, U32P, I, I, I, I, U32P, I, U32P, ctypes.POINTER(ctypes.c_uint64), U32P]),
            "oracle_generate_s": (I, [P, U32P, I, I, I, P, U32P]),
            "oracle_spec_generate_s": (I, [P, U32P, I, I, I, I, U32P, I, P, U32P, ctypes.POINTER(ctypes.c_uint64), U32P]),
            "oracle_sampler_new": (P, [ctypes.POINTER(SamplerCfg), I]),
            "oracle_sampler_free": (None, [P]),
            "oracle_sampler_process": (I, [P, P, U32P, P]),
            "oracle_sampler_draw": (ctypes.c_uint32, [P]),
            "oracle_sampler_sample": (ctypes.c_uint32, [P, P]),
            "oracle_sampler_accept": (I, [P, P, P, ctypes.c_uint32, U32P]),
            "oracle_rng_seed": (None, [ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint64]),
            "oracle_rng_next": (ctypes.c_uint64, [ctypes.POINTER(ctypes.c_uint64)]),
            "oracle_state_get": (ctypes.c_long, [P, I, I, P]),
            "oracle_set_simd": (None, [I]),
            "oracle_layer_f32": (I, [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float),
                                     ctypes.POINTER(ctypes.c_void_p), I, P, I, I, P, P, P, P, P]),
        })
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class SamplerCfg(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int), ("top_p", ctypes.c_float),
                ("min_p", ctypes.c_float), ("seed", ctypes.c_uint64)]


class OracleSampler:
    """The reference's Sampler (crates/core/src/sample.rs) on the CPU: process / draw / sample / accept."""

    def __init__(self, vocab, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, seed=0):
        self.vocab = vocab
        self.cfg = SamplerCfg(temperature, top_k, top_p, min_p, seed)
        self._h = lib().oracle_sampler_new(ctypes.byref(self.cfg), vocab)

    def __del__(self):
        try:
            lib().oracle_sampler_free(self._h)
        except Exception:
            pass

    def process(self, logits):
        lg = np.ascontiguousarray(logits, np.float32)
        ids = (ctypes.c_uint32 * self.vocab)()
        ps = np.empty(self.vocab, np.float32)
        n = lib().oracle_sampler_process(self._h, _p(lg), ids, _p(ps))
        return list(ids[:n]), ps[:n].copy()

    def draw(self):
        return lib().oracle_sampler_draw(self._h)

    def sample(self, logits):
        return lib().oracle_sampler_sample(self._h, _p(np.ascontiguousarray(logits, np.float32)))

    def accept(self, target_logits, q_dense, d):
        tok = ctypes.c_uint32()
        ok = lib().oracle_sampler_accept(self._h, _p(np.ascontiguousarray(target_logits, np.float32)),
                                         _p(np.ascontiguousarray(q_dense, np.float32)), d, ctypes.byref(tok))
        return bool(ok), tok.value


def rng_u64(seed, n):
    """The first n outputs of the sampler's xoshiro256** seeded through splitmix64."""
    st = (ctypes.c_uint64 * 4)()
    lib().oracle_rng_seed(st, seed)
    return [lib().oracle_rng_next(st) for _ in range(n)]


def set_libm(mode):
    lib().oracle_set_libm(mode)


def set_threads(n):
    lib().oracle_set_threads(n)


def set_simd(on):
    """1: the AVX2 matmul kernels (bit-identical to the scalar ones), 0: the scalar kernels, -1: by CPU detection."""
    lib().oracle_set_simd(on)


def row_bytes(t, cols):
    be, bb = LAYOUT[t]
    return cols // be * bb


def act_bytes(t, cols):
    if t in (Q4_K, Q5_K, Q6_K):
        return cols // 256 * 292
    if t in (Q8_0, Q4_0):
        return cols // 32 * 34
    return cols * 4


def dequantize(t, raw, n):
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    rc = lib().oracle_dequantize(t, _p(raw), raw.size, _p(out), n)
    if rc != 0:
        raise ValueError(f"dequantize: size mismatch for type {t}: {raw.size} bytes, {n} elements")
    return out


def quantize_q8k(x):
    """Rows of f32 (last dim a multiple of 256) -> uint8 array of block_q8_K bytes, one row per input row."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.reshape(-1, x.shape[-1])
    n = rows.shape[1]
    out = np.empty((rows.shape[0], n // 256 * 292), dtype=np.uint8)
    for r in range(rows.shape[0]):
        lib().oracle_quantize_q8k(_p(rows[r]), n, _p(out[r]))
    return out


def quantize_q8_0(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.reshape(-1, x.shape[-1])
    n = rows.shape[1]
    out = np.empty((rows.shape[0], n // 32 * 34), dtype=np.uint8)
    for r in range(rows.shape[0]):
        lib().oracle_quantize_q8_0(_p(rows[r]), n, _p(out[r]))
    return out


def dot(t, wrow, act, cols):
    wrow = np.ascontiguousarray(wrow, dtype=np.uint8)
    act = np.ascontiguousarray(act)
    return lib().oracle_dot(t, _p(wrow), _p(act), cols)


def matmul(t, w, rows, cols, x):
    """y[c, r] = w[r] . x[c] with x quantised into the form `t` consumes (matvec.rs:147-160)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
    y = np.empty((x.shape[0], rows), dtype=np.float32)
    lib().oracle_matmul_f32in(t, _p(w), rows, cols, _p(x), x.shape[0], _p(y))
    return y


def matmul_act(t, w, rows, cols, act):
    """As `matmul` on pre-quantised activation rows (uint8 blocks, or f32 for F32 weights)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    act = np.ascontiguousarray(act)
    ncols = act.shape[0]
    stride = act.strides[0]
    y = np.empty((ncols, rows), dtype=np.float32)
    lib().oracle_matmul_act(t, _p(w), rows, cols, _p(act), stride, ncols, _p(y))
    return y


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    rows = x.reshape(-1, x.shape[-1])
    yr = y.reshape(-1, x.shape[-1])
    for r in range(rows.shape[0]):
        lib().oracle_rmsnorm(_p(rows[r]), _p(w), rows.shape[1], eps, _p(yr[r]))
    return y


def rmsnorm_gated(x, gate, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    gate = np.ascontiguousarray(gate, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    xr, gr, yr = x.reshape(-1, x.shape[-1]), gate.reshape(-1, x.shape[-1]), y.reshape(-1, x.shape[-1])
    for r in range(xr.shape[0]):
        lib().oracle_rmsnorm_gated(_p(xr[r]), _p(gr[r]), _p(w), xr.shape[1], eps, _p(yr[r]))
    return y


def softmax(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().oracle_softmax(_p(x), x.size, _p(y))
    return y


def silu(x):
    return np.array([lib().oracle_silu(float(v)) for v in np.asarray(x, dtype=np.float32).ravel()], dtype=np.float32)


def swiglu(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    y = np.empty_like(g)
    lib().oracle_swiglu(_p(g), _p(u), g.size, _p(y))
    return y


def inv_freq(rope_dim, theta):
    out = np.empty(rope_dim // 2, dtype=np.float32)
    lib().oracle_inv_freq(rope_dim, theta, _p(out))
    return out


def cos_sin(pos, inv_f):
    inv_f = np.ascontiguousarray(inv_f, dtype=np.float32)
    half = inv_f.size
    c = np.empty(2 * half, dtype=np.float32)
    s = np.empty(2 * half, dtype=np.float32)
    lib().oracle_cos_sin(pos, _p(inv_f), half, _p(c), _p(s))
    return c, s


def apply_rope(x, head_dim, rope_dim, cos, sin):
    x = np.array(x, dtype=np.float32, copy=True)
    cos = np.ascontiguousarray(cos, dtype=np.float32)
    sin = np.ascontiguousarray(sin, dtype=np.float32)
    lib().oracle_apply_rope(_p(x), x.size, head_dim, rope_dim, _p(cos), _p(sin))
    return x


def conv1d_step(state, w, kernel, x_new):
    state = np.array(state, dtype=np.float32, copy=True)
    w = np.ascontiguousarray(w, dtype=np.float32)
    x_new = np.ascontiguousarray(x_new, dtype=np.float32)
    out = np.empty(x_new.size, dtype=np.float32)
    lib().oracle_conv1d_step(_p(state), _p(w), kernel, _p(x_new), x_new.size, _p(out), 1)
    return out, state


def l2norm(x, eps=1e-6):
    x = np.array(x, dtype=np.float32, copy=True)
    lib().oracle_l2norm(_p(x), x.size, eps)
    return x


def gate_g(a, dt_bias, big_a):
    return lib().oracle_gate_g(a, dt_bias, big_a)


def gate_beta(b):
    return lib().oracle_gate_beta(b)


def deltanet_step(q, k, v, g, beta, s):
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    s = np.array(s, dtype=np.float32, copy=True)
    out = np.empty(v.size, dtype=np.float32)
    lib().oracle_deltanet_step(_p(q), _p(k), _p(v), q.size, v.size, g, beta, _p(s), _p(out))
    return out, s


def argmax(v):
    v = np.ascontiguousarray(v, dtype=np.float32)
    return lib().oracle_argmax(_p(v), v.size)


def crc32(b):
    b = np.ascontiguousarray(b, dtype=np.uint8)
    return lib().oracle_crc32(_p(b), b.size)


# weight slots of oracle_layer_f32 (oracle.h OW_*), by GGUF tensor name
LAYER_WEIGHTS = ("attn_norm.weight", "post_attention_norm.weight", "attn_qkv.weight", "attn_gate.weight",
                 "ssm_alpha.weight", "ssm_beta.weight", "ssm_a", "ssm_dt.bias", "ssm_conv1d.weight", "ssm_norm.weight",
                 "ssm_out.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                 "attn_q_norm.weight", "attn_k_norm.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight")
LAYER_KINDS = {"deltanet": 0, "attention": 1, "mlp": 2, "decoder_deltanet": 3, "decoder_attention": 4}


class LayerF32:
    """One layer of the oracle (the functions oracle_forward_token runs) on caller-held F32 weights, as the
    reference's crates/core/tests/layers.rs loads them (WeightMat::from_f32): `dims` = dict(hidden, ffn, n_head,
    n_kv, head_dim, rope_dim, conv_kernel, dk, n_k, n_v, dv, eps, theta); `weights` = GGUF name -> f32 array.
    The carried state (S, conv window, K and V rows) lives in this object across calls."""

    def __init__(self, kind, dims, weights, max_pos=64):
        self.kind = LAYER_KINDS[kind]
        self.d = dims
        self._w = [np.ascontiguousarray(weights[n], np.float32) if n in weights else None for n in LAYER_WEIGHTS]
        self._wp = (ctypes.c_void_p * len(LAYER_WEIGHTS))(*[(_p(a).value if a is not None else None) for a in self._w])
        self._dims = (ctypes.c_int * 11)(*[int(dims[k]) for k in ("hidden", "ffn", "n_head", "n_kv", "head_dim", "rope_dim",
                                                                  "conv_kernel", "dk", "n_k", "n_v", "dv")])
        self._f = (ctypes.c_float * 2)(dims["eps"], dims["theta"])
        conv_dim = 2 * dims["n_k"] * dims["dk"] + dims["n_v"] * dims["dv"]
        self.S = np.zeros((max(dims["n_v"], 1), max(dims["dk"], 1), max(dims["dv"], 1)), np.float32)
        self.conv = np.zeros((max(conv_dim, 1), max(dims["conv_kernel"] - 1, 1)), np.float32)
        kvd = max(dims["n_kv"] * dims["head_dim"], 1)
        self.K = np.zeros((max_pos, kvd), np.float32)
        self.V = np.zeros((max_pos, kvd), np.float32)
        self.pos = 0

    def __call__(self, x):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.d["hidden"])
        y = np.empty_like(x)
        rc = lib().oracle_layer_f32(self._dims, self._f, self._wp, self.kind, _p(x), x.shape[0], self.pos, _p(self.S),
                                    _p(self.conv), _p(self.K), _p(self.V), _p(y))
        if rc != 0:
            raise ValueError("oracle_layer_f32 failed")
        self.pos += x.shape[0]
        return y


class OracleModel:
    """The reference's model seam restated on the CPU (oracle/model.c): forward_token, the plain greedy loop and
    the greedy --spec k loop, over a GGUF read through mmap."""

    def __init__(self, path):
        err = ctypes.create_string_buffer(512)
        self._h = lib().oracle_model_open(str(path).encode(), err, 512)
        if not self._h:
            raise ValueError(f"oracle: {err.value.decode()}")
        dims = (ctypes.c_int * 8)()
        lib().oracle_model_dims(self._h, dims)
        self.n_layer, self.hidden, self.vocab, self.has_mtp, self.eos, self.ffn, self.n_head, self.head_dim = list(dims)

    def close(self):
        if self._h:
            lib().oracle_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def state(self, max_pos=4096):
        return OracleState(self, max_pos)


class OracleState:
    def __init__(self, model, max_pos):
        self.model = model
        self._h = lib().oracle_state_new(model._h, max_pos)

    def __del__(self):
        try:
            lib().oracle_state_free(self._h)
        except Exception:
            pass

    @property
    def pos(self):
        return lib().oracle_state_pos(self._h)

    def forward_token(self, tok, capture=False, logits=True):
        """Returns (logits or None, captured per-layer residual rows [n_layer + 1][hidden] or None); with
        logits=False the lm_head is skipped (a prompt row)."""
        m = self.model
        lg = np.empty(m.vocab, np.float32) if logits else None
        cap = np.empty((m.n_layer + 1, m.hidden), np.float32) if capture else None
        rc = lib().oracle_forward_token(self._h, tok, _p(lg) if logits else None, _p(cap) if capture else None, None)
        if rc != 0:
            raise ValueError("oracle: forward_token failed (id out of range or sequence full)")
        return lg, cap

    def carried(self, layer, what):
        """The carried state of `layer` (0 DeltaNet S, 1 conv window, 2 K rows, 3 V rows [0, pos)), or None."""
        n = lib().oracle_state_get(self._h, layer, what, None)
        if n <= 0:
            return None
        out = np.empty(n, np.float32)
        lib().oracle_state_get(self._h, layer, what, _p(out))
        return out

    def generate(self, prompt, n_out, stop=True, sampler=None):
        out = (ctypes.c_uint32 * n_out)()
        arr = (ctypes.c_uint32 * len(prompt))(*prompt)
        c = lib().oracle_generate_s(self._h, arr, len(prompt), n_out, 1 if stop else 0, sampler._h if sampler else None, out)
        if c < 0:
            raise ValueError("oracle: generate failed")
        return list(out[:c])

    def spec_generate(self, prompt, n_out, k, stop=True, forced=None, sampler=None):
        """Returns (ids, stats dict, drafts used per round)."""
        out = (ctypes.c_uint32 * n_out)()
        arr = (ctypes.c_uint32 * len(prompt))(*prompt)
        st = (ctypes.c_uint64 * 4)()
        n_forced = 0
        fz = None
        if forced is not None:
            flat = [int(v) for r in forced for v in r]
            n_forced = len(forced)
            fz = (ctypes.c_uint32 * len(flat))(*flat)
        log = (ctypes.c_uint32 * (k * (n_out + 2)))()
        c = lib().oracle_spec_generate_s(self._h, arr, len(prompt), n_out, k, 1 if stop else 0, fz, n_forced,
                                         sampler._h if sampler else None, out, st, log)
        if c < 0:
            raise ValueError("oracle: spec_generate failed")
        stats = dict(zip(("rounds", "drafted", "accepted", "emitted"), list(st)))
        stats["round_seconds"] = lib().oracle_last_round_seconds()
        drafts = [list(log[i * k:(i + 1) * k]) for i in range(stats["rounds"])]
        return list(out[:c]), stats, drafts
