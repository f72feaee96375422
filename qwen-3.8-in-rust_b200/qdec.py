"""Python binding of the qdec C ABI (include/qdec.h), over ctypes.

This mirrors the reference engine's crate API for the decode path (`aqueduct`, crates/core): the kernel
seam (`matvec`, `matmul_fn`, `Q8KRow::quantize_into`, `dequantize_into`) and, in `Model`, the model seam
(`Model::load_with`, `new_state_spec`, `prefill`, `forward_token`, `spec_prefill`, `spec_round`).  Errors
raise QdecError carrying the library's status code and message, the counterpart of the reference's
`ModelError` / assert! panics.  Device buffers are passed as integer device pointers (e.g. from
`torch.Tensor.data_ptr()`); PyTorch is only the caller's allocator here.

The library must be built (build.py); importing this module on a machine without it raises, there is no
fallback implementation.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqdec.so")

OK, EINVAL, ECUDA, ENOMEM, EIO, EFORMAT, ESTATE, ETIMEOUT = 0, -1, -2, -3, -4, -5, -6, -7
F32, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 2, 8, 12, 13, 14
Q6_K_SPLIT = 114
TYPE_NAMES = {F32: "F32", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
LAYOUT = {F32: (1, 4), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}


class Opts(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("max_pos", ctypes.c_int)]


class ModelInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in ("n_layer", "hidden", "ffn", "vocab", "n_head", "n_head_kv", "head_dim",
                                               "dn_n_k_heads", "dn_n_v_heads", "dn_head_dim_k", "dn_head_dim_v",
                                               "n_full_attention", "has_mtp")] + [
        ("weight_bytes", ctypes.c_uint64), ("decode_bytes", ctypes.c_uint64), ("lm_head_bytes", ctypes.c_uint64),
        ("mtp_bytes", ctypes.c_uint64), ("load_secs", ctypes.c_double)]


class QdecError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"qdec error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built: run python qwen-3.8-in-rust_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        P, I, S = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
        L.qdec_version.restype = ctypes.c_char_p
        L.qdec_last_error.restype = ctypes.c_char_p
        for name, args in {
            "qdec_quantize_q8k": [P, I, I, P, P],
            "qdec_quantize_q8_0": [P, I, I, P, P],
            "qdec_gemv": [I, P, I, I, P, I, P, P],
            "qdec_matvec": [I, P, I, I, P, I, P, P],
            "qdec_matvec_noalloc": [I, P, I, I, P, I, P, P],
            "qdec_dequant_rows": [I, P, I, I, P, I, P, P],
            "qdec_repack_q6k": [P, I, I, P, P],
            "qdec_repack_tiles": [I, P, I, I, P, P],
            "qdec_tune_gemv": [I, I],
            "qdec_quantize_image": [I, P, I, I, P, P],
            "qdec_gemv_image": [I, P, I, I, P, I, P, P],
            "qdec_selftest_wait": [I, I],
            "qdec_gemv_image_pair": [I, P, P, I, I, P, I, P, P, P],
        }.items():
            fn = getattr(L, name)
            fn.restype = I
            fn.argtypes = args
        L.qdec_act_row_bytes.restype = S
        L.qdec_image_row_bytes.restype = S
        L.qdec_image_row_bytes.argtypes = [I, I]
        L.qdec_act_row_bytes.argtypes = [I, I]
        L.qdec_matvec_noalloc_max_bytes.restype = S
        L.qdec_matvec_noalloc_max_bytes.argtypes = []
        L.qdec_matvec_scratch_bytes.restype = S
        L.qdec_matvec_scratch_bytes.argtypes = [I, P, I, I]
        PP = ctypes.POINTER(ctypes.c_void_p)
        U32P = ctypes.POINTER(ctypes.c_uint32)
        for name, args in {
            "qdec_open": [ctypes.c_char_p, ctypes.POINTER(Opts), PP],
            "qdec_open_tp": [ctypes.c_char_p, ctypes.POINTER(Opts), I, I, PP],
            "qdec_tp_plan": [ctypes.c_char_p, I, I, ctypes.POINTER(ctypes.c_int32)],
            "qdec_tp_plan_dims": [ctypes.POINTER(ctypes.c_uint32), I, I, ctypes.POINTER(ctypes.c_int32)],
            "qdec_tp_export": [P, P],
            "qdec_tp_connect": [P, P],
            "qdec_tp_stats": [P, ctypes.POINTER(ctypes.c_uint64)],
            "qdec_set_sampler": [P, ctypes.c_float, I, ctypes.c_float, ctypes.c_float, ctypes.c_uint64],
            "qdec_close": [P],
            "qdec_model_get_info": [P, ctypes.POINTER(ModelInfo)],
            "qdec_is_stop": [P, ctypes.c_uint32],
            "qdec_state_new": [P, I, I, I, PP],
            "qdec_state_free": [P],
            "qdec_state_pos": [P],
            "qdec_prefill": [P, U32P, I, U32P],
            "qdec_step": [P, ctypes.c_uint32, U32P, P],
            "qdec_model_loaded_direct": [P],
            "qdec_batch_step": [P, I, U32P, U32P],
            "qdec_spec_prefill": [P, U32P, I, U32P],
            "qdec_spec_round": [P, ctypes.c_uint32, U32P, ctypes.POINTER(I)],
            "qdec_set_drafts": [P, U32P, I],
            "qdec_get_drafts": [P, U32P, I],
            "qdec_spec_counters": [P, ctypes.POINTER(ctypes.c_uint64)],
            "qdec_set_capture": [P, I],
            "qdec_debug_hidden": [P, I, I, P],
            "qdec_debug_logits": [P, I, P],
            "qdec_debug_state": [P, I, I, P, ctypes.POINTER(S)],
            "qdec_synth_gguf": [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint64, I],
        }.items():
            fn = getattr(L, name)
            fn.restype = I
            fn.argtypes = args
        L.qdec_state_stream.restype = P
        L.qdec_state_stream.argtypes = [P]
        L.qdec_state_launches.restype = ctypes.c_uint64
        L.qdec_state_launches.argtypes = [P]
        _lib = L
    return _lib


def _check(rc):
    if rc != OK:
        raise QdecError(rc, lib().qdec_last_error().decode(errors="replace"))


def version():
    return lib().qdec_version().decode()


def row_bytes(t, cols):
    be, bb = LAYOUT[t]
    return cols // be * bb


def act_row_bytes(t, cols):
    return lib().qdec_act_row_bytes(t, cols)


def quantize_q8k(x_ptr, n, rows, out_ptr, stream=0):
    """Q8KRow::quantize_into (crates/core/src/kernels/q8k.rs:51) on `rows` device rows."""
    _check(lib().qdec_quantize_q8k(x_ptr, n, rows, out_ptr, stream))


def quantize_q8_0(x_ptr, n, rows, out_ptr, stream=0):
    """Q8Row::quantize_into (crates/core/src/kernels/q8.rs:65)."""
    _check(lib().qdec_quantize_q8_0(x_ptr, n, rows, out_ptr, stream))


def gemv(t, w_ptr, rows, cols, act_ptr, ncols, y_ptr, stream=0):
    """matmul_fn over pre-quantised activations (crates/core/src/kernels/matvec.rs:377): y[c*rows + r]."""
    _check(lib().qdec_gemv(t, w_ptr, rows, cols, act_ptr, ncols, y_ptr, stream))


def matvec(t, w_ptr, rows, cols, x_ptr, ncols, y_ptr, stream=0):
    """matvec_f32_in / matmul (crates/core/src/kernels/matvec.rs:541, :369) from f32 activation rows."""
    _check(lib().qdec_matvec(t, w_ptr, rows, cols, x_ptr, ncols, y_ptr, stream))


def matvec_noalloc(t, w_ptr, rows, cols, x_ptr, ncols, y_ptr, stream=0):
    """As `matvec`, allocating nothing: the quantised columns use a fixed array inside the library (for callers
    that cannot let a library allocate device memory)."""
    _check(lib().qdec_matvec_noalloc(t, w_ptr, rows, cols, x_ptr, ncols, y_ptr, stream))


def matvec_noalloc_max_bytes():
    return lib().qdec_matvec_noalloc_max_bytes()


def matvec_scratch_bytes(t, w_ptr, cols, ncols):
    """Scratch bytes a matvec of ncols columns needs on these weights (qdec_matvec_scratch_bytes); None if the type
    or width is not taken."""
    v = lib().qdec_matvec_scratch_bytes(t, w_ptr, cols, ncols)
    return None if v == (1 << 64) - 1 else v


def image_row_bytes(t, cols):
    return lib().qdec_image_row_bytes(t, cols)


def quantize_image(t, x_ptr, n, rows, img_ptr, stream=0):
    """f32 rows -> the activation image weights of type t read (Q8_K image or Q8_0 image)."""
    _check(lib().qdec_quantize_image(t, x_ptr, n, rows, img_ptr, stream))


def gemv_image(t, w_ptr, rows, cols, img_ptr, ncols, y_ptr, stream=0):
    _check(lib().qdec_gemv_image(t, w_ptr, rows, cols, img_ptr, ncols, y_ptr, stream))


def gemv_image_pair(t, w1_ptr, w2_ptr, rows, cols, img_ptr, ncols, y1_ptr, y2_ptr, stream=0):
    """matvec2 (crates/core/src/kernels/matvec.rs:349) over the image: two tile matrices, one launch."""
    _check(lib().qdec_gemv_image_pair(t, w1_ptr, w2_ptr, rows, cols, img_ptr, ncols, y1_ptr, y2_ptr, stream))


GEMV7_CONFIGS = 10


def tune_gemv(impl=0, config=0):
    """Select a GEMV kernel / configuration (qdec_tune_gemv): impl 0/6 the image kernel of ggml-layout Q4_K/Q5_K
    and split Q6_K weights (config 0..8), impl 2 the reference-layout activation kernel, impl 7 the decode GEMV of
    K-quant tile matrices (0 by shape, 1..8), impl 8 the Q8_0/Q4_0 tile kernel (0..3), impl 9 the smallest column
    count of the tensor-core prefill GEMM (default 16, 0 never), impl 10 the smallest column group of the warp-MMA
    Q4_K GEMV (1..4, default 4, 0 never). Results are identical for every value."""
    _check(lib().qdec_tune_gemv(impl, config))


PREFILL_GEMM_MIN_COLS = 16
GEMV_MMA_MIN_COLS = 4


def selftest_wait(which, wait_ms=200):
    """Run a bounded device wait into its limit on the current device, then the same work normally
    (0 = the tensor-parallel exchange poll, 1 = the decode GEMV's stage wait); raises QdecError when the wait
    did not give up and report as designed, or the normal run afterwards failed."""
    _check(lib().qdec_selftest_wait(which, wait_ms))


def repack_tiles(t, src_ptr, rows, cols, dst_ptr, stream=0):
    """ggml Q4_K/Q5_K/Q6_K rows -> the tile layout (type TILE[t])."""
    _check(lib().qdec_repack_tiles(t, src_ptr, rows, cols, dst_ptr, stream))


TILE = {12: 112, 13: 113, 14: 116, 8: 108, 2: 102}


def repack_q6k(src_ptr, rows, cols, dst_ptr, stream=0):
    """ggml Q6_K rows -> the engine's split device layout (QDEC_TYPE_Q6_K_SPLIT)."""
    _check(lib().qdec_repack_q6k(src_ptr, rows, cols, dst_ptr, stream))


def dequant_rows(t, w_ptr, rows, cols, ids_ptr, nids, out_ptr, stream=0):
    """Model::embed_token_into (crates/core/src/model.rs:364) for n device-resident ids."""
    _check(lib().qdec_dequant_rows(t, w_ptr, rows, cols, ids_ptr, nids, out_ptr, stream))


def _u32(seq):
    arr = (ctypes.c_uint32 * len(seq))(*[int(v) for v in seq])
    return arr


def synth_gguf(path, preset, seed, threads=0):
    """Write a synthetic checkpoint ("tiny", "27b", "27b-L<n>"); the stand-in for the real GGUF."""
    _check(lib().qdec_synth_gguf(str(path).encode(), preset.encode(), seed, threads))


TP_HANDLE_BYTES = 80
TP_PLAN_FIELDS = ("rank", "world", "kh_lo", "nk", "nv", "qh_lo", "nq", "kv_lo", "nkv", "ff_lo", "ff_rows", "h_lo", "h_rows",
                  "v_lo", "v_rows")


def tp_plan(path, rank, world):
    """The rows / heads rank `rank` of `world` keeps (from the GGUF header; no device needed)."""
    out = (ctypes.c_int32 * 16)()
    _check(lib().qdec_tp_plan(str(path).encode(), rank, world, out))
    return dict(zip(TP_PLAN_FIELDS, list(out)))


def tp_plan_dims(hidden, ffn, vocab, n_head, n_head_kv, dn_k_heads, dn_v_heads, rank, world):
    """tp_plan from the dimensions alone (a model with DeltaNet layers when dn_k_heads > 0)."""
    dims = _u32([hidden, ffn, vocab, n_head, n_head_kv, dn_k_heads, dn_v_heads, 1 if dn_k_heads else 0])
    out = (ctypes.c_int32 * 16)()
    _check(lib().qdec_tp_plan_dims(dims, rank, world, out))
    return dict(zip(TP_PLAN_FIELDS, list(out)))


def gather_handles(handle, group=None):
    """Every rank's exchange handle, in rank order, over a torch.distributed process group."""
    import torch.distributed as dist

    hs = [None] * dist.get_world_size(group)
    dist.all_gather_object(hs, handle, group=group)
    return hs


class Model:
    """Model::load_with (crates/core/src/model.rs:184): the GGUF's weights resident on `device`.

    tp=(rank, world) loads rank `rank`'s shard for tensor parallelism over `world` GPUs (one process each)."""

    def __init__(self, path, device=0, max_pos=4096, tp=None):
        self._h = ctypes.c_void_p()
        o = Opts(device, max_pos)
        self.tp = tuple(tp) if tp else (0, 1)
        if tp:
            _check(lib().qdec_open_tp(str(path).encode(), ctypes.byref(o), self.tp[0], self.tp[1], ctypes.byref(self._h)))
        else:
            _check(lib().qdec_open(str(path).encode(), ctypes.byref(o), ctypes.byref(self._h)))
        info = ModelInfo()
        _check(lib().qdec_model_get_info(self._h, ctypes.byref(info)))
        self.info = info
        self.max_pos = max_pos

    def close(self):
        if self._h:
            lib().qdec_close(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def is_stop(self, tok):
        return bool(lib().qdec_is_stop(self._h, tok))

    @property
    def loaded_direct(self):
        """True when the weights were read with O_DIRECT (QDEC_LOAD_DIRECT=1 and a file system that allows it)."""
        return bool(lib().qdec_model_loaded_direct(self._h))

    def new_state(self, spec_k=0, max_pos=None, max_rows=32):
        """Model::new_state / new_state_spec (model.rs:334, spec.rs:184)."""
        return State(self, spec_k, max_pos or self.max_pos, max_rows)


class State:
    def __init__(self, model, spec_k, max_pos, max_rows):
        self.model = model
        self.k = spec_k
        self._h = ctypes.c_void_p()
        _check(lib().qdec_state_new(model._h, spec_k, max_pos, max_rows, ctypes.byref(self._h)))

    def free(self):
        if self._h:
            lib().qdec_state_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def pos(self):
        return lib().qdec_state_pos(self._h)

    def tp_export(self):
        """This rank's exchange handle (bytes) for the other ranks."""
        buf = ctypes.create_string_buffer(TP_HANDLE_BYTES)
        _check(lib().qdec_tp_export(self._h, buf))
        return buf.raw

    def tp_connect(self, handles):
        """Open every rank's exchange block: `handles` = all ranks' tp_export() results in rank order."""
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        _check(lib().qdec_tp_connect(self._h, buf))

    def tp_stats(self):
        buf = (ctypes.c_uint64 * 4)()
        _check(lib().qdec_tp_stats(self._h, buf))
        return dict(zip(("exchanges", "ns_push", "ns_wait", "unused"), list(buf)))

    def tp_connect_group(self, group=None):
        """tp_export + all_gather over a torch.distributed process group + tp_connect."""
        self.tp_connect(gather_handles(self.tp_export(), group))

    @property
    def stream(self):
        """The cudaStream_t (as an int) all of this state's kernels run on."""
        return lib().qdec_state_stream(self._h) or 0

    @property
    def launches(self):
        return lib().qdec_state_launches(self._h)

    def prefill(self, ids):
        out = ctypes.c_uint32()
        _check(lib().qdec_prefill(self._h, _u32(ids), len(ids), ctypes.byref(out)))
        return out.value

    def step(self, tok, want_logits=False):
        out = ctypes.c_uint32()
        if want_logits:
            import numpy as np

            lg = np.empty(self.model.info.vocab, np.float32)
            _check(lib().qdec_step(self._h, tok, ctypes.byref(out), lg.ctypes.data_as(ctypes.c_void_p)))
            return out.value, lg
        _check(lib().qdec_step(self._h, tok, ctypes.byref(out), None))
        return out.value

    def spec_prefill(self, ids):
        out = ctypes.c_uint32()
        _check(lib().qdec_spec_prefill(self._h, _u32(ids), len(ids), ctypes.byref(out)))
        return out.value

    def spec_round(self, x_p):
        buf = (ctypes.c_uint32 * (self.k + 1))()
        n = ctypes.c_int()
        _check(lib().qdec_spec_round(self._h, x_p, buf, ctypes.byref(n)))
        return list(buf[: n.value])

    def set_sampler(self, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, seed=0):
        """Sampler::new(SamplerConfig{..}) for this state (temperature <= 0: greedy); the RNG restarts at seed."""
        _check(lib().qdec_set_sampler(self._h, temperature, top_k, top_p, min_p, seed))

    def set_drafts(self, drafts):
        _check(lib().qdec_set_drafts(self._h, _u32(drafts), len(drafts)))

    def drafts(self):
        buf = (ctypes.c_uint32 * self.k)()
        _check(lib().qdec_get_drafts(self._h, buf, self.k))
        return list(buf)

    def counters(self):
        buf = (ctypes.c_uint64 * 4)()
        _check(lib().qdec_spec_counters(self._h, buf))
        return dict(zip(("rounds", "drafted", "accepted", "emitted"), list(buf)))

    def set_capture(self, on=True):
        _check(lib().qdec_set_capture(self._h, 1 if on else 0))

    def hidden(self, layer, row=0):
        import numpy as np

        out = np.empty(self.model.info.hidden, np.float32)
        _check(lib().qdec_debug_hidden(self._h, layer, row, out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def carried(self, layer, what):
        """The carried state of `layer` after the last call (what: 0 DeltaNet state, 1 conv window, 2 K rows,
        3 V rows [0, pos)) as a float32 array, or None when the layer holds no such state."""
        import numpy as np

        n = ctypes.c_size_t(0)
        _check(lib().qdec_debug_state(self._h, layer, what, None, ctypes.byref(n)))
        if n.value == 0:
            return None
        out = np.empty(n.value, np.float32)
        _check(lib().qdec_debug_state(self._h, layer, what, out.ctypes.data_as(ctypes.c_void_p), ctypes.byref(n)))
        return out

    def logits(self, row=0):
        import numpy as np

        out = np.empty(self.model.info.vocab, np.float32)
        _check(lib().qdec_debug_logits(self._h, row, out.ctypes.data_as(ctypes.c_void_p)))
        return out


def generate(state, prompt, n_tokens, stop=True):
    """The reference's plain greedy loop (crates/cli/src/run.rs:329-350): prefill, then one token per step."""
    out = [state.prefill(prompt)]
    while len(out) < n_tokens and not (stop and state.model.is_stop(out[-1])):
        out.append(state.step(out[-1]))
    return out


def batch_step(states, ids):
    """One greedy step of several sequences in one forward (qdec_batch_step): ids[i] into states[i], their next
    tokens out, identical to states[i].step(ids[i]); states[0] needs max_rows >= len(states)."""
    n = len(states)
    if n != len(ids):
        raise ValueError("batch_step: one id per state")
    hs = (ctypes.c_void_p * n)(*[s._h.value for s in states])
    out = (ctypes.c_uint32 * n)()
    _check(lib().qdec_batch_step(ctypes.cast(hs, ctypes.c_void_p), n, _u32(ids), out))
    return list(out)


def generate_batch(states, prompts, n_tokens):
    """Plain greedy decoding of several sequences together: each state prefilled with its prompt, then
    batch_step for the rest (the tokens of every sequence equal generate(state, prompt, n_tokens, stop=False))."""
    outs = [[s.prefill(p)] for s, p in zip(states, prompts)]
    while len(outs[0]) < n_tokens:
        nxt = batch_step(states, [o[-1] for o in outs])
        for o, t in zip(outs, nxt):
            o.append(t)
    return outs


def generate_spec(state, prompt, n_tokens, stop=True):
    """The reference's --spec loop (crates/cli/src/run.rs:353-383): spec_prefill, then rounds."""
    out = [state.spec_prefill(prompt)]
    while len(out) < n_tokens and not (stop and state.model.is_stop(out[-1])):
        em = state.spec_round(out[-1])
        for t in em:
            out.append(t)
            if len(out) >= n_tokens or (stop and state.model.is_stop(t)):
                break
    return out[:n_tokens]
