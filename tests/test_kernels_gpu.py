"""GPU parity of the kernel-level C ABI against the CPU oracle and the reference's golden vectors.

Bit-exact everywhere: the quantisers, the dequantiser and every GEMV path compute the reference's exact
arithmetic (integer lanes, then f32 in the reference's order), so the expected result is the oracle's,
bit for bit, not a tolerance band.
"""
import numpy as np
import pytest

import golden_io as G
from helpers import bits_equal, hostile_rows, random_blocks, row_bytes, to_dev

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TYPES = [12, 13, 14, 8, 2, 0]


@pytest.fixture(scope="module")
def q():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qdec

    qdec.lib()
    return qdec


def gpu_q8k(q, x):
    x = np.ascontiguousarray(x, np.float32).reshape(-1, x.shape[-1])
    xd = to_dev(x)
    out = torch.empty(x.shape[0] * (x.shape[1] // 256) * 292, dtype=torch.uint8, device="cuda")
    q.quantize_q8k(xd.data_ptr(), x.shape[1], x.shape[0], out.data_ptr())
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(x.shape[0], -1)


def gpu_q8_0(q, x):
    x = np.ascontiguousarray(x, np.float32).reshape(-1, x.shape[-1])
    xd = to_dev(x)
    out = torch.empty(x.shape[0] * (x.shape[1] // 32) * 34, dtype=torch.uint8, device="cuda")
    q.quantize_q8_0(xd.data_ptr(), x.shape[1], x.shape[0], out.data_ptr())
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(x.shape[0], -1)


def test_q8k_quantiser_golden(q):
    meta, a = G.load("q8k_quantize")
    for c in meta["cases"]:
        x = a[c["case"] + "__x"]
        raw = a[c["case"] + "__raw"].reshape(x.shape[0], -1)
        got = gpu_q8k(q, x)
        for r in range(x.shape[0]):
            assert np.array_equal(got[r], raw[r]), f"{c['case']} row {r} ({c['rows'][r]})"


def test_q8k_quantiser_hostile_and_random(q, orc):
    for width in (256, 5120, 17408):
        x = np.concatenate([hostile_rows(width, 7), np.random.default_rng(3).standard_normal((5, width)).astype(np.float32)])
        assert np.array_equal(gpu_q8k(q, x), orc.quantize_q8k(x)), width


def test_q8_0_quantiser_golden_and_random(q, orc):
    meta, a = G.load("q8_quantize")
    for c in meta["cases"]:
        x = a[c["case"] + "__x"]
        raw = a[c["case"] + "__raw"].reshape(x.shape[0], -1)
        assert np.array_equal(gpu_q8_0(q, x), raw), c["case"]
    x = np.random.default_rng(5).standard_normal((7, 6144)).astype(np.float32) * 3
    assert np.array_equal(gpu_q8_0(q, x), orc.quantize_q8_0(x))


def run_gemv(q, t, w, rows, cols, x):
    """qdec_matvec from f32 columns: quantise on the device, then the GEMV."""
    wd = to_dev(w)
    xd = to_dev(np.ascontiguousarray(x, np.float32))
    n = x.shape[0]
    y = torch.empty(n * rows, dtype=torch.float32, device="cuda")
    q.matvec(t, wd.data_ptr(), rows, cols, xd.data_ptr(), n, y.data_ptr())
    torch.cuda.synchronize()
    return y.cpu().numpy().reshape(n, rows)


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("ncols", [1, 2, 3, 4, 5])
def test_gemv_random_bit_exact(q, orc, t, ncols):
    rows, cols = 261, 5120  # ragged row count: not a multiple of any tile
    w = random_blocks(t, rows, cols, seed=100 + t)
    x = np.random.default_rng(ncols).standard_normal((ncols, cols)).astype(np.float32)
    got = run_gemv(q, t, w, rows, cols, x)
    want = orc.matmul(t, w, rows, cols, x)
    assert bits_equal(got, want), f"type {t} ncols {ncols}: max diff {np.abs(got - want).max()}"


@pytest.mark.parametrize("name,t", [("Q4_K", 12), ("Q5_K", 13), ("Q6_K", 14), ("Q4_0", 2)])
def test_gemv_real_weights_bit_exact(q, orc, name, t):
    """64 rows of the real model's weights (reference fixtures/dequant) against hostile + random columns."""
    meta, a = G.load("dequant")
    info = meta["types"][name]["rows64"]
    w = a[name + "__rows64_raw"]
    cols = info["cols"]
    x = hostile_rows(cols, 11)[:4] if t != 2 else np.random.default_rng(1).standard_normal((4, cols)).astype(np.float32)
    x = np.nan_to_num(x, posinf=0, neginf=0)
    got = run_gemv(q, t, w, 64, cols, x)
    want = orc.matmul(t, w, 64, cols, x)
    assert bits_equal(got, want), name


@pytest.mark.parametrize("rows,cols", [(17408, 5120), (5120, 17408)])
def test_gemv_config2_full_size_bit_exact(q, orc, rows, cols):
    """The GEMV microbench shapes (17408 x 5120 and 5120 x 17408), Q4_K, N = 4: every output bit-identical to the
    oracle."""
    t = 12
    w = random_blocks(t, rows, cols, seed=rows)
    x = np.random.default_rng(9).standard_normal((4, cols)).astype(np.float32)
    got = run_gemv(q, t, w, rows, cols, x)
    want = orc.matmul(t, w, rows, cols, x)
    assert bits_equal(got, want)
    # column independence: column c of the batched call == the single-column call (matmul_t.rs property)
    got1 = run_gemv(q, t, w, rows, cols, x[2:3])
    assert bits_equal(got1[0], got[2])


def test_gemv_matches_golden_matvec(q):
    """The reference's matvec fixtures: within the f64 budget, like crates/core/tests/kernels.rs."""
    meta, a = G.load("matvec")
    for c in meta["cases"]:
        t, cols, rows = c["ggml_type_id"], c["width"], c["n_rows"]
        if t in (2, 8) and cols % 64:
            continue
        w = a[c["case"] + "__w_raw"]
        x = a[c["case"] + "__x_deq"][None, :]
        y = run_gemv(q, t, w, rows, cols, x)[0]
        if t in (12, 13, 14):
            continue  # K-quant budgets are checked on the oracle; bit-equality with it is checked above
        for r in range(rows):
            assert abs(y[r] - c["ref_f64"][r]) <= G.budget(meta["budget_k"], cols, c["max_abs_term"][r]), c["case"]


@pytest.mark.parametrize("t", TYPES)
def test_dequant_rows_bit_exact(q, orc, t):
    rows, cols = 50, 5120
    w = random_blocks(t, rows, cols, seed=t + 1)
    ids = np.array([3, 0, 49, 3, 17], np.int32)
    wd, idd = to_dev(w), to_dev(ids)
    out = torch.empty(len(ids) * cols, dtype=torch.float32, device="cuda")
    q.dequant_rows(t, wd.data_ptr(), rows, cols, idd.data_ptr(), len(ids), out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(len(ids), cols)
    rb = row_bytes(t, cols)
    for i, r in enumerate(ids):
        want = orc.dequantize(t, w[r * rb:(r + 1) * rb], cols)
        assert bits_equal(got[i], want), (t, r)


def test_dequant_golden_hostile(q):
    meta, a = G.load("dequant")
    for h in meta["hostile"]["hostile"]:
        tid = {"Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "F32": 0}[h["ggml_type"]]
        base = h["raw_bin"][:-4]
        raw, want, n = a[base + "__raw"], a[base + "__deq"], h["n_elements"]
        ids = np.zeros(1, np.int32)
        wd, idd = to_dev(raw), to_dev(ids)
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        q.dequant_rows(tid, wd.data_ptr(), 1, n, idd.data_ptr(), 1, out.data_ptr())
        torch.cuda.synchronize()
        assert bits_equal(out.cpu().numpy(), want), base


def run_gemv_raw(q, t, wd, rows, cols, x):
    xd = to_dev(np.ascontiguousarray(x, np.float32))
    n = x.shape[0]
    y = torch.empty(n * rows, dtype=torch.float32, device="cuda")
    q.matvec(t, wd.data_ptr(), rows, cols, xd.data_ptr(), n, y.data_ptr())
    torch.cuda.synchronize()
    return y.cpu().numpy().reshape(n, rows)


@pytest.mark.parametrize("cfg", [0, 1, 2, 3, 4])
def test_gemv_q6k_split_layout_bit_exact(q, orc, cfg):
    """Q6_K repacked into the split device layout (208-byte blocks + f16 scales) gives the ggml-layout bits."""
    rows, cols = 515, 5120
    w = random_blocks(14, rows, cols, seed=99)
    src = to_dev(w)
    dst = torch.empty_like(src)
    q.repack_q6k(src.data_ptr(), rows, cols, dst.data_ptr())
    torch.cuda.synchronize()
    x = np.random.default_rng(3).standard_normal((4, cols)).astype(np.float32)
    want = orc.matmul(14, w, rows, cols, x)
    q.tune_gemv(6, cfg)
    try:
        for n in (1, 2, 4):
            got = run_gemv_raw(q, q.Q6_K_SPLIT, dst, rows, cols, x[:n])
            assert bits_equal(got, want[:n]), (cfg, n)
    finally:
        q.tune_gemv(0, 0)


@pytest.mark.parametrize("t", [12, 13, 114])
@pytest.mark.parametrize("cfg", range(1, 9))
def test_gemv_image_kernel_every_config_bit_exact(q, orc, t, cfg):
    """The image-reading GEMV in each configuration (lanes per thread, rows per thread, depth, integer or FP32
    scale multiply): the oracle's bits for 1..5 columns, on a ragged row count and a width whose super-block
    count is not a multiple of any depth, through both entry points (f32 columns and block_q8_K columns)."""
    rows, cols = 389, 5376  # 21 super-blocks
    base = 14 if t == 114 else t
    w = random_blocks(base, rows, cols, seed=7 + t)
    x = np.random.default_rng(cfg).standard_normal((5, cols)).astype(np.float32)
    x[1] *= 1e-30  # tiny and hostile scales
    x[2, ::7] = 0.0
    want = orc.matmul(base, w, rows, cols, x)
    wd = to_dev(w)
    if t == 114:
        dst = torch.empty_like(wd)
        q.repack_q6k(wd.data_ptr(), rows, cols, dst.data_ptr())
        wd = dst
    q.tune_gemv(6, cfg)
    try:
        for n in (1, 2, 3, 4, 5):
            got = run_gemv_raw(q, t, wd, rows, cols, x[:n])
            assert bits_equal(got, want[:n]), (t, cfg, n)
        act = gpu_q8k(q, x[:4])  # reference-layout block_q8_K columns through qdec_gemv
        ad = to_dev(np.ascontiguousarray(act).reshape(-1))
        y = torch.empty(4 * rows, dtype=torch.float32, device="cuda")
        q.gemv(t, wd.data_ptr(), rows, cols, ad.data_ptr(), 4, y.data_ptr())
        torch.cuda.synchronize()
        assert bits_equal(y.cpu().numpy().reshape(4, rows), want[:4]), (t, cfg, "gemv")
    finally:
        q.tune_gemv(0, 0)


@pytest.mark.parametrize("rows,cols", [(1, 256), (5, 17408), (4099, 256)])
def test_gemv_image_kernel_edge_shapes(q, orc, rows, cols):
    """One row, one super-block per row, and the widest activation rows of the model."""
    w = random_blocks(12, rows, cols, seed=rows)
    x = np.random.default_rng(2).standard_normal((4, cols)).astype(np.float32)
    want = orc.matmul(12, w, rows, cols, x)
    got = run_gemv_raw(q, 12, to_dev(w), rows, cols, x)
    assert bits_equal(got, want)


@pytest.mark.parametrize("t", [12, 13, 14])
def test_gemv_reference_layout_kernel_bit_exact(q, orc, t):
    """The kernel that reads block_q8_K columns in the reference layout (forced for Q4_K/Q5_K; the ggml Q6_K
    layout always takes it)."""
    rows, cols = 261, 5120
    w = random_blocks(t, rows, cols, seed=3 + t)
    x = np.random.default_rng(t).standard_normal((4, cols)).astype(np.float32)
    want = orc.matmul(t, w, rows, cols, x)
    q.tune_gemv(2, 0)
    try:
        got = run_gemv_raw(q, t, to_dev(w), rows, cols, x)
    finally:
        q.tune_gemv(0, 0)
    assert bits_equal(got, want)


def test_tile_repack_rejects_ragged_rows(q):
    src = torch.zeros(12 * 144, dtype=torch.uint8, device="cuda")
    dst = torch.empty_like(src)
    with pytest.raises(q.QdecError):
        q.repack_tiles(12, src.data_ptr(), 12, 256, dst.data_ptr())


@pytest.mark.parametrize("split", [1, 2, 3])
@pytest.mark.parametrize("t", [8, 2])
def test_gemv_q80_tile_layout_bit_exact(q, orc, t, split):
    """Q8_0 / Q4_0 weights in the tile layout (8 rows x 8 blocks per tile block) against the Q8_0 activation
    image: the oracle's bits for 1..5 columns, from f32 columns and from block_q8_0 columns."""
    rows, cols = 8 * 29, 6144
    w = random_blocks(t, rows, cols, seed=57 + t)
    x = np.random.default_rng(t).standard_normal((5, cols)).astype(np.float32)
    x[2] *= 1e-25
    x[4, :40] = 0.0
    want = orc.matmul(t, w, rows, cols, x)
    src = to_dev(w)
    dst = torch.empty_like(src)
    q.repack_tiles(t, src.data_ptr(), rows, cols, dst.data_ptr())
    torch.cuda.synchronize()
    q.tune_gemv(8, split)
    try:
        for n in (1, 2, 3, 4, 5):
            got = run_gemv_raw(q, q.TILE[t], dst, rows, cols, x[:n])
            assert bits_equal(got, want[:n]), (t, n)
        act = to_dev(np.ascontiguousarray(gpu_q8_0(q, x[:4])).reshape(-1))
        y = torch.empty(4 * rows, dtype=torch.float32, device="cuda")
        q.gemv(q.TILE[t], dst.data_ptr(), rows, cols, act.data_ptr(), 4, y.data_ptr())
        torch.cuda.synchronize()
        assert bits_equal(y.cpu().numpy().reshape(4, rows), want[:4])
    finally:
        q.tune_gemv(8, 0)


@pytest.mark.parametrize("t,base", [(112, 12), (116, 14), (108, 8), (102, 2)])
def test_gemv_image_entry_points(q, orc, t, base):
    """qdec_quantize_image + qdec_gemv_image (activations already in the library's image) give the oracle's bits."""
    rows, cols = 64, 5120
    w = random_blocks(base, rows, cols, seed=t)
    x = np.random.default_rng(t).standard_normal((3, cols)).astype(np.float32)
    want = orc.matmul(base, w, rows, cols, x)
    src = to_dev(w)
    dst = torch.empty_like(src)
    q.repack_tiles(base, src.data_ptr(), rows, cols, dst.data_ptr())
    xd = to_dev(x)
    img = torch.empty(3 * q.image_row_bytes(t, cols), dtype=torch.uint8, device="cuda")
    q.quantize_image(t, xd.data_ptr(), cols, 3, img.data_ptr())
    y = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
    q.gemv_image(t, dst.data_ptr(), rows, cols, img.data_ptr(), 3, y.data_ptr())
    torch.cuda.synchronize()
    assert bits_equal(y.cpu().numpy().reshape(3, rows), want)


def _repack(q, t, w, rows, cols):
    src = to_dev(w)
    dst = torch.empty_like(src)
    q.repack_tiles(t, src.data_ptr(), rows, cols, dst.data_ptr())
    torch.cuda.synchronize()
    return dst


@pytest.mark.parametrize("t", [12, 13, 14])
@pytest.mark.parametrize("cfg", range(0, 9))
def test_gemv7_every_config_bit_exact(q, orc, t, cfg):
    """The decode GEMV of tile matrices (gemv7.cu) in each configuration (tiles per warp, warps splitting the
    super-blocks, depth, register cap): the oracle's bits for 1..5 columns on a tile count that is not a multiple
    of any split and 21 super-blocks (not a multiple of any depth or split), with tiny, huge and zero columns."""
    rows, cols = 8 * 37, 5376
    w = random_blocks(t, rows, cols, seed=71 + t)
    x = np.random.default_rng(200 + cfg).standard_normal((5, cols)).astype(np.float32)
    x[1] *= 1e-30
    x[3] *= 1e20
    x[4, ::3] = 0.0
    want = orc.matmul(t, w, rows, cols, x)
    dst = _repack(q, t, w, rows, cols)
    q.tune_gemv(7, cfg)
    try:
        for n in (1, 2, 3, 4, 5):
            got = run_gemv_raw(q, q.TILE[t], dst, rows, cols, x[:n])
            assert bits_equal(got, want[:n]), (t, cfg, n)
    finally:
        q.tune_gemv(0, 0)


@pytest.mark.parametrize("t", [12, 14])
def test_gemv_image_pair_bit_exact(q, orc, t):
    """qdec_gemv_image_pair (matvec2, matvec.rs:349): two tile matrices against the same image columns in one
    launch give, matrix by matrix, the oracle's bits for 1..5 columns."""
    rows, cols = 8 * 45, 5120
    w1 = random_blocks(t, rows, cols, seed=81 + t)
    w2 = random_blocks(t, rows, cols, seed=91 + t)
    x = np.random.default_rng(t).standard_normal((5, cols)).astype(np.float32)
    x[2] *= 1e-20
    want1 = orc.matmul(t, w1, rows, cols, x)
    want2 = orc.matmul(t, w2, rows, cols, x)
    d1, d2 = _repack(q, t, w1, rows, cols), _repack(q, t, w2, rows, cols)
    tt = q.TILE[t]
    for n in (1, 2, 3, 4, 5):
        xd = to_dev(x[:n])
        img = torch.empty(n * q.image_row_bytes(tt, cols), dtype=torch.uint8, device="cuda")
        q.quantize_image(tt, xd.data_ptr(), cols, n, img.data_ptr())
        y1 = torch.empty(n * rows, dtype=torch.float32, device="cuda")
        y2 = torch.empty(n * rows, dtype=torch.float32, device="cuda")
        q.gemv_image_pair(tt, d1.data_ptr(), d2.data_ptr(), rows, cols, img.data_ptr(), n, y1.data_ptr(), y2.data_ptr())
        torch.cuda.synchronize()
        assert bits_equal(y1.cpu().numpy().reshape(n, rows), want1[:n]), (t, n, 1)
        assert bits_equal(y2.cpu().numpy().reshape(n, rows), want2[:n]), (t, n, 2)


def _extreme_blocks(t, rows, cols, seed, neg_scales=False):
    """Blocks at the integer extremes of the dot: every code at its maximum (Q4_K 15, Q5_K 31, Q6_K 63), every
    6-bit scale and min 63 (Q6_K int8 scales -128 or +127), finite random f16 d / dmin."""
    w = random_blocks(t, rows, cols, seed).reshape(-1, {12: 144, 13: 176, 14: 210}[t]).copy()
    if t in (12, 13):
        w[:, 4:] = 0xFF
    else:
        w[:, :192] = 0xFF
        w[:, 192:208] = 0x80 if neg_scales else 0x7F
    return w.reshape(-1)


@pytest.mark.parametrize("t,neg", [(12, False), (13, False), (14, False), (14, True)])
@pytest.mark.parametrize("cfg", [0, 1, 4, 7])
def test_gemv7_integer_extremes_bit_exact(q, orc, t, neg, cfg):
    """The largest lane sums the formats allow (the packed 16-bit chunk sums and the biased lane conversion at
    their limits): activation codes all -127, all +127 and alternating, against maximal codes and scales."""
    rows, cols = 64, 2048
    w = _extreme_blocks(t, rows, cols, seed=t, neg_scales=neg)
    x = np.stack([np.full(cols, 3.0, np.float32), np.full(cols, -3.0, np.float32),
                  np.where(np.arange(cols) % 2 == 0, 2.0, -2.0).astype(np.float32),
                  np.random.default_rng(t).standard_normal(cols).astype(np.float32)])
    want = orc.matmul(t, w, rows, cols, x)
    dst = _repack(q, t, w, rows, cols)
    q.tune_gemv(7, cfg)
    try:
        got = run_gemv_raw(q, q.TILE[t], dst, rows, cols, x)
    finally:
        q.tune_gemv(0, 0)
    assert bits_equal(got, want), (t, neg, cfg)


@pytest.mark.parametrize("cfg", [0, 3, 4, 5, 7])
def test_gemv7_warp_mma_bit_exact(q, orc, cfg):
    """The warp-MMA forms of the Q4_K tile GEMV (integer lanes on mma.sync m16n8k32, gemv7.cu): streaming (configs
    3-5) and windowed (7; 0 picks by shape) with every column count 1..5 routed there, against the oracle's bits:
    an odd tile count (the last warp's second tile is past the end), 21 super-blocks (not a multiple of any
    window or stage), tiny, huge and zero columns, and the integer extremes of the codes and scales."""
    rows, cols = 8 * 37, 5376
    w = random_blocks(12, rows, cols, seed=300 + cfg)
    x = np.random.default_rng(400 + cfg).standard_normal((5, cols)).astype(np.float32)
    x[1] *= 1e-30
    x[3] *= 1e20
    x[4, ::3] = 0.0
    want = orc.matmul(12, w, rows, cols, x)
    dst = _repack(q, 12, w, rows, cols)
    we = _extreme_blocks(12, 64, 2048, seed=5)
    xe = np.stack([np.full(2048, 3.0, np.float32), np.full(2048, -3.0, np.float32),
                   np.where(np.arange(2048) % 2 == 0, 2.0, -2.0).astype(np.float32),
                   np.random.default_rng(6).standard_normal(2048).astype(np.float32)])
    want_e = orc.matmul(12, we, 64, 2048, xe)
    dst_e = _repack(q, 12, we, 64, 2048)
    q.tune_gemv(7, cfg)
    q.tune_gemv(10, 1)
    try:
        for n in (1, 2, 3, 4, 5):
            got = run_gemv_raw(q, q.TILE[12], dst, rows, cols, x[:n])
            assert bits_equal(got, want[:n]), (cfg, n)
        got_e = run_gemv_raw(q, q.TILE[12], dst_e, 64, 2048, xe)
        assert bits_equal(got_e, want_e), (cfg, "extremes")
    finally:
        q.tune_gemv(10, q.GEMV_MMA_MIN_COLS)
        q.tune_gemv(0, 0)
