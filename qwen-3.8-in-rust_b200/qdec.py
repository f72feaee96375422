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
TYPE_NAMES = {F32: "F32", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
LAYOUT = {F32: (1, 4), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}


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
            "qdec_dequant_rows": [I, P, I, I, P, I, P, P],
        }.items():
            fn = getattr(L, name)
            fn.restype = I
            fn.argtypes = args
        L.qdec_act_row_bytes.restype = S
        L.qdec_act_row_bytes.argtypes = [I, I]
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


def dequant_rows(t, w_ptr, rows, cols, ids_ptr, nids, out_ptr, stream=0):
    """Model::embed_token_into (crates/core/src/model.rs:364) for n device-resident ids."""
    _check(lib().qdec_dequant_rows(t, w_ptr, rows, cols, ids_ptr, nids, out_ptr, stream))
