"""qdec_matvec_noalloc: the matvec entry point for callers that cannot let the library allocate device memory
(an application whose GPU memory belongs to another allocator, or a decode loop that must not allocate while it
runs).  It must give exactly what qdec_matvec gives, call after call, from its fixed in-library scratch array,
and allocate nothing doing so.

This file is collected last on purpose (pytest orders files by name), so a run that stops at its first failure
has run every other test before this one."""
import os
import subprocess
import sys

import numpy as np
import pytest

from helpers import random_blocks, to_dev

HERE = os.path.dirname(os.path.abspath(__file__))

# (weight type, weight pointer, bytes one column of `cols` values takes in the scratch, per 256 / 32 values):
# the image path (16-byte aligned ggml Q4_K), block_q8_K rows (unaligned Q4_K), the Q8_0 tile image, block_q8_0
SIZING = [(12, 256, 320 / 256), (12, 1, 292 / 256), (108, 256, 40 / 32), (8, 256, 34 / 32)]


@pytest.mark.parametrize("t,w_ptr,per_value", SIZING)
def test_oversize_request_is_rejected_before_any_device_work(t, w_ptr, per_value):
    """One column more than the scratch holds, for each path's column size, is refused without touching the
    device (the pointers are not device memory; a call that reached a kernel would fail differently)."""
    import qdec

    cap = qdec.matvec_noalloc_max_bytes()
    cols = 17408
    per_col = int(per_value * cols)
    n = cap // per_col + 1
    with pytest.raises(qdec.QdecError) as e:
        qdec.matvec_noalloc(t, w_ptr, 16, cols, 1, n, 1)
    assert e.value.code == qdec.EINVAL and "scratch" in str(e.value)
    assert f"need {n * per_col} bytes" in str(e.value)
    # the query gives the same sizes (no device work), so a caller can check before calling
    assert qdec.matvec_scratch_bytes(t, w_ptr, cols, n) == n * per_col
    assert qdec.matvec_scratch_bytes(t, w_ptr, cols, n - 1) <= cap


def test_scratch_query_rejects_what_the_kernels_do_not_take():
    import qdec

    assert qdec.matvec_scratch_bytes(12, 256, 100, 1) is None  # not a multiple of 256
    assert qdec.matvec_scratch_bytes(7, 256, 256, 1) is None   # not a kernel type
    assert qdec.matvec_scratch_bytes(0, 256, 256, 4) == 0       # F32 takes the columns as they are


def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _two_calls(torch, qdec, t, w, rows, cols, ncols):
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # the scratch keeps the previous call's bytes: the second call must not see them
        x = to_dev(np.random.default_rng(call * 10 + t).standard_normal((ncols, cols)).astype(np.float32) * (1 + call))
        y_ref = torch.empty(ncols * rows, dtype=torch.float32, device="cuda")
        y_new = torch.empty(ncols * rows, dtype=torch.float32, device="cuda")
        qdec.matvec(t, w.data_ptr(), rows, cols, x.data_ptr(), ncols, y_ref.data_ptr(), stream)
        qdec.matvec_noalloc(t, w.data_ptr(), rows, cols, x.data_ptr(), ncols, y_new.data_ptr(), stream)
        torch.cuda.synchronize()
        a, b = y_ref.cpu().numpy(), y_new.cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"type {t}, call {call}"


@pytest.mark.gpu
@pytest.mark.parametrize("t", [12, 13, 14, 8, 2])
def test_noalloc_matches_matvec_on_two_calls(t):
    torch = _cuda()
    import qdec

    rows, cols = 300, 5120
    _two_calls(torch, qdec, t, to_dev(random_blocks(t, rows, cols, seed=77 + t)), rows, cols, 4)


@pytest.mark.gpu
@pytest.mark.parametrize("t", [12, 14])
def test_noalloc_tile_matrices_gemv_and_tensor_core_routes(t):
    """Tile-layout K-quant weights: 4 columns take the decode GEMV, 16 the tensor-core GEMM; both equal
    qdec_matvec on two calls."""
    torch = _cuda()
    import qdec

    rows, cols = 256, 5120
    src = to_dev(random_blocks(t, rows, cols, seed=91 + t))
    tile = torch.empty_like(src)
    qdec.repack_tiles(t, src.data_ptr(), rows, cols, tile.data_ptr(), torch.cuda.current_stream().cuda_stream)
    tt = qdec.TILE[t]
    for ncols in (4, 16):
        _two_calls(torch, qdec, tt, tile, rows, cols, ncols)


_FRESH = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[2])
import qdec
qdec.lib()  # the library is loaded before the CUDA context exists, so eager module loading places its device code
import torch
from helpers import random_blocks, to_dev
rows, cols, t = 512, 5120, 12
w = to_dev(random_blocks(t, rows, cols, seed=5))
x = to_dev(np.random.default_rng(6).standard_normal((4, cols)).astype(np.float32))
y0 = torch.empty(4 * rows, dtype=torch.float32, device="cuda")
y1 = torch.empty(4 * rows, dtype=torch.float32, device="cuda")
stream = torch.cuda.current_stream().cuda_stream  # first use of torch's stream before the readings
torch.cuda.synchronize()
def free_now():
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0]
f0 = free_now()
for _ in range(3):
    qdec.matvec_noalloc(t, w.data_ptr(), rows, cols, x.data_ptr(), 4, y1.data_ptr(), stream)
f1 = free_now()
qdec.matvec(t, w.data_ptr(), rows, cols, x.data_ptr(), 4, y0.data_ptr(), stream)
torch.cuda.synchronize()
same = np.array_equal(y0.cpu().numpy().view(np.uint32), y1.cpu().numpy().view(np.uint32))
print("FREE", f0, f1, "SAME", int(same))
"""


@pytest.mark.gpu
def test_noalloc_allocates_nothing_in_a_fresh_process():
    """In a fresh process whose first compute call is qdec_matvec_noalloc, the device's free memory is the same
    before and after three calls, and the result equals qdec_matvec's, run afterwards.  The library is loaded
    before the CUDA context is created and modules load eagerly, so its device code and fixed arrays are in place
    before the first reading; torch's stream is taken before it too."""
    _cuda()
    pkg = os.path.join(os.path.dirname(HERE), "qwen-3.8-in-rust_b200")
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    r = subprocess.run([sys.executable, "-c", _FRESH, HERE, pkg], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("FREE")][-1].split()
    f0, f1, same = int(line[1]), int(line[2]), int(line[4])
    assert same == 1
    assert f0 == f1, f"free device memory changed by {f0 - f1} bytes across qdec_matvec_noalloc calls"
