"""The tensor-core prefill GEMM (K-quant tile matrices against >= 8 activation columns) gives the oracle's bits:
random blocks over ragged row tiles and column groups, worst-case magnitudes (every scale, code and activation
at its extreme, so every lane sum reaches its largest value), and the same bits as the CUDA-core GEMV it
replaces for prompt rows."""
import numpy as np
import pytest

from helpers import bits_equal, random_blocks, to_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TILE_TYPES = [12, 13, 14]


@pytest.fixture(scope="module")
def q():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qdec

    qdec.lib()
    return qdec


def tiles(q, t, w, rows, cols):
    src = to_dev(w)
    dst = torch.empty_like(src)
    q.repack_tiles(t, src.data_ptr(), rows, cols, dst.data_ptr())
    torch.cuda.synchronize()
    return dst


def matvec(q, tt, wd, rows, cols, x, min_cols=None):
    """qdec_matvec on the device; min_cols selects the prefill GEMM's threshold for this call (0 = GEMV only)."""
    xd = to_dev(np.ascontiguousarray(x, np.float32))
    n = x.shape[0]
    y = torch.empty(n * rows, dtype=torch.float32, device="cuda")
    if min_cols is not None:
        q.tune_gemv(9, min_cols)
    try:
        q.matvec(tt, wd.data_ptr(), rows, cols, xd.data_ptr(), n, y.data_ptr())
        torch.cuda.synchronize()
    finally:
        q.tune_gemv(9, q.PREFILL_GEMM_MIN_COLS)
    return y.cpu().numpy().reshape(n, rows)


@pytest.mark.parametrize("t", TILE_TYPES)
@pytest.mark.parametrize("ncols", [8, 16, 21, 40])
def test_prefill_gemm_random_bit_exact(q, orc, t, ncols):
    """296 rows (two full 128-row tiles and a ragged one), 21 super-blocks, 8..40 columns (full and ragged
    16-column groups); one column scaled by 1e20, one with a zero block."""
    rows, cols = 8 * 37, 5376
    w = random_blocks(t, rows, cols, seed=300 + t)
    x = np.random.default_rng(ncols).standard_normal((ncols, cols)).astype(np.float32)
    x[1] *= 1e20
    x[min(5, ncols - 1), 512:768] = 0.0
    want = orc.matmul(t, w, rows, cols, x)
    got = matvec(q, q.TILE[t], tiles(q, t, w, rows, cols), rows, cols, x, min_cols=8)  # the GEMM from 8 columns
    assert bits_equal(got, want), f"type {t} ncols {ncols}: max diff {np.abs(got - want).max()}"


def extreme_blocks(t, rows, cols, seed):
    """Blocks whose codes and scales sit at their extremes (Q4_K/Q5_K: scales and mins 63, codes 15 / 31;
    Q6_K: codes 63, scales -128 or 127), f16 super-block scales finite."""
    from helpers import LAYOUT

    rng = np.random.default_rng(seed)
    _, bb = LAYOUT[t]
    nblk = rows * (cols // 256)
    data = np.full((nblk, bb), 0xFF, np.uint8)
    one = np.array([0x00, 0x3C], np.uint8)  # f16 1.0
    if t in (12, 13):
        data[:, 0:2] = one
        data[:, 2:4] = one
    else:
        data[:, 192:208] = np.where(rng.integers(0, 2, (nblk, 16)) == 0, 0x80, 0x7F).astype(np.uint8)
        data[:, 208:210] = one
    return data.reshape(-1)


@pytest.mark.parametrize("t", TILE_TYPES)
def test_prefill_gemm_extreme_magnitudes_bit_exact(q, orc, t):
    """Every lane sum at its largest magnitude (activation codes all +-127): the integer sums on the tensor
    cores stay exact and the f32 steps match the oracle bit for bit."""
    rows, cols, n = 256, 1024, 16
    w = extreme_blocks(t, rows, cols, seed=7)
    x = np.ones((n, cols), np.float32)
    x[1] = -1.0
    x[2, ::2] = -1.0
    x[3] = np.where(np.arange(cols) % 7 == 0, -1.0, 1.0)
    x[4:] = np.random.default_rng(9).standard_normal((n - 4, cols)).astype(np.float32)
    want = orc.matmul(t, w, rows, cols, x)
    got = matvec(q, q.TILE[t], tiles(q, t, w, rows, cols), rows, cols, x)
    assert bits_equal(got, want), f"type {t}: max diff {np.abs(got - want).max()}"


@pytest.mark.parametrize("t", TILE_TYPES)
def test_prefill_gemm_equals_gemv(q, t):
    """The 27B FFN width (5120 -> 1024 rows of it) at 32 columns: the tensor-core GEMM and the CUDA-core GEMV
    (forced) give identical bits."""
    rows, cols, n = 1024, 5120, 32
    w = random_blocks(t, rows, cols, seed=400 + t)
    x = np.random.default_rng(401).standard_normal((n, cols)).astype(np.float32)
    wd = tiles(q, t, w, rows, cols)
    tc = matvec(q, q.TILE[t], wd, rows, cols, x)
    gv = matvec(q, q.TILE[t], wd, rows, cols, x, min_cols=0)
    assert bits_equal(tc, gv)


def test_prefill_gemm_threshold_knob(q):
    with pytest.raises(q.QdecError):
        q.tune_gemv(9, -1)
    q.tune_gemv(9, q.PREFILL_GEMM_MIN_COLS)
