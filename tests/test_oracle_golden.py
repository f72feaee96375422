"""Pin the CPU oracle against the reference's own golden vectors (tests/golden, from the reference's
tests/fixtures).  Exact where the reference's tests are exact (quantisers, dequant), within the reference's
derived budgets elsewhere (crates/core/tests/{q8k,kernels,dequant}.rs)."""
import numpy as np
import pytest

import golden_io as G

K_TYPES = (12, 13, 14)


def test_q8k_quantiser_bit_exact(orc):
    """crates/core/tests/q8k.rs (a): every byte of every fixture row."""
    meta, a = G.load("q8k_quantize")
    n = 0
    for c in meta["cases"]:
        x = a[c["case"] + "__x"]
        raw = a[c["case"] + "__raw"].reshape(x.shape[0], -1)
        got = orc.quantize_q8k(x)
        for r in range(x.shape[0]):
            assert np.array_equal(got[r], raw[r]), f"{c['case']} row {r} ({c['rows'][r]})"
            n += 1
    assert n == 36


def test_q8_0_quantiser_bit_exact(orc):
    meta, a = G.load("q8_quantize")
    for c in meta["cases"]:
        x = a[c["case"] + "__x"]
        raw = a[c["case"] + "__raw"].reshape(x.shape[0], -1)
        got = orc.quantize_q8_0(x)
        assert np.array_equal(got, raw), c["case"]


def test_dequant_bit_exact(orc):
    """crates/core/tests/dequant.rs: prefixes, heads of full tensors and the hostile blocks, bit for bit."""
    meta, a = G.load("dequant")
    for name, t in meta["types"].items():
        tid = t["ggml_type_id"]
        got = orc.dequantize(tid, a[name + "__prefix_raw"], t["prefix"]["n_elements"])
        assert np.array_equal(got.view(np.uint32), a[name + "__prefix"].view(np.uint32)), name
        if name + "__full_head_raw" in a:
            head = a[name + "__full_head"]
            got = orc.dequantize(tid, a[name + "__full_head_raw"], head.size)
            assert np.array_equal(got.view(np.uint32), head.view(np.uint32)), name + " head"
    for h in meta["hostile"]["hostile"]:
        tid = {"Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "F32": 0}[h["ggml_type"]]
        base = h["raw_bin"][:-4]
        want = a[base + "__deq"]
        got = orc.dequantize(tid, a[base + "__raw"], h["n_elements"])
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), base


def test_dequant_size_errors(orc):
    """quant.rs length checks (quant.rs tests length_errors_are_reported)."""
    with pytest.raises(ValueError):
        orc.dequantize(2, np.zeros(17, np.uint8), 32)
    with pytest.raises(ValueError):
        orc.dequantize(8, np.zeros(34, np.uint8), 33)


def test_f16_known_values(orc):
    """quant.rs tests f16_roundtrip_exact."""
    L = orc.lib()
    assert L.oracle_f16_to_f32(0x3C00) == 1.0
    assert L.oracle_f16_to_f32(0xC000) == -2.0
    assert L.oracle_f16_to_f32(0x0001) == np.float32(5.9604645e-8)
    assert L.oracle_f16_to_f32(0x7BFF) == 65504.0


def test_f32_to_f16_round_trip_all_halves(orc):
    """f32 -> f16 (RNE) inverts f16 -> f32 on every finite half, and rounds midpoints to even."""
    L = orc.lib()
    for h in range(0, 0x7C00, 7):
        f = L.oracle_f16_to_f32(h)
        assert L.oracle_f32_to_f16(f) == h
        assert L.oracle_f32_to_f16(-f) == (h | 0x8000) or h == 0
    # 1 + 2^-11 is the midpoint between 1 and the next half: ties to even (1.0)
    assert L.oracle_f32_to_f16(np.float32(1.0 + 2.0 ** -11)) == 0x3C00
    assert L.oracle_f32_to_f16(np.float32(1.0 + 3 * 2.0 ** -11)) == 0x3C02


def test_crc32_known_vector(orc):
    assert orc.crc32(np.frombuffer(b"123456789", np.uint8)) == 0xCBF43926


def test_kquant_dots_within_terms_budget(orc):
    """crates/core/tests/q8k.rs (b): K-quant x Q8_K dots against the f64 reference of the dequantised rows."""
    meta, a = G.load("dot")
    k = meta["budget_k"]
    checked = 0
    for c in meta["cases"]:
        t = c["ggml_type_id"]
        if t not in K_TYPES:
            continue
        width, n_rows = c["width"], c["n_rows"]
        rb = orc.row_bytes(t, width)
        w = a[c["case"] + "__w_raw"]
        x = a[c["case"] + "__x_deq"].reshape(n_rows, width)
        for r in range(n_rows):
            wrow = w[r * rb:(r + 1) * rb]
            xq = orc.quantize_q8k(x[r])[0]
            wd = orc.dequantize(t, wrow, width)
            xd = np.concatenate([np.frombuffer(xq[b * 292:b * 292 + 4].tobytes(), np.float32)[0]
                                 * xq[b * 292 + 4:b * 292 + 260].view(np.int8).astype(np.float32)
                                 for b in range(width // 256)])
            ref = float(np.sum(wd.astype(np.float64) * xd.astype(np.float64)))
            bud = G.kquant_terms_budget(t, wrow, wd, xd, k, orc.lib().oracle_f16_to_f32)
            got = orc.dot(t, wrow, xq, width)
            assert abs(got - ref) <= bud, f"{c['case']} row {r}: {got} vs {ref} budget {bud}"
            checked += 1
    assert checked >= 20


def test_q8_0_q4_0_f32_dots_within_budget(orc):
    """crates/core/tests/kernels.rs dot_kernels_within_budget for the Q8_0-activation and F32 paths."""
    meta, a = G.load("dot")
    k = meta["budget_k"]
    for c in meta["cases"]:
        t = c["ggml_type_id"]
        if t in K_TYPES:
            continue
        width, n_rows = c["width"], c["n_rows"]
        rb = orc.row_bytes(t, width)
        w = a[c["case"] + "__w_raw"]
        for r in range(n_rows):
            wrow = w[r * rb:(r + 1) * rb]
            if t == 0:
                act = a[c["case"] + "__x_deq"].reshape(n_rows, width)[r]
            else:
                act = a[c["case"] + "__x_raw"].reshape(n_rows, -1)[r]
            got = orc.dot(t, wrow, act, width)
            bud = G.budget(k, width, c["max_abs_term"][r])
            assert abs(got - c["ref_f64"][r]) <= bud, f"{c['case']} row {r}"


def test_matvec_within_budget(orc):
    """crates/core/tests/kernels.rs matvec_within_budget_and_thread_invariant (default Q8_K path)."""
    meta, a = G.load("matvec")
    k = meta["budget_k"]
    for c in meta["cases"]:
        t = c["ggml_type_id"]
        width, rows = c["width"], c["n_rows"]
        w = a[c["case"] + "__w_raw"]
        x = a[c["case"] + "__x_deq"]
        y = orc.matmul(t, w, rows, width, x)[0]
        rb = orc.row_bytes(t, width)
        if t in K_TYPES:
            xq = orc.quantize_q8k(x)[0]
            xd = np.concatenate([np.frombuffer(xq[b * 292:b * 292 + 4].tobytes(), np.float32)[0]
                                 * xq[b * 292 + 4:b * 292 + 260].view(np.int8).astype(np.float32)
                                 for b in range(width // 256)])
        for r in range(rows):
            if t in K_TYPES:
                wd = orc.dequantize(t, w[r * rb:(r + 1) * rb], width)
                ref = float(np.sum(wd.astype(np.float64) * xd.astype(np.float64)))
                bud = G.kquant_terms_budget(t, w[r * rb:(r + 1) * rb], wd, xd, k, orc.lib().oracle_f16_to_f32)
            else:
                ref = c["ref_f64"][r]
                bud = G.budget(k, width, c["max_abs_term"][r])
            assert abs(y[r] - ref) <= bud, f"{c['case']} row {r}: {y[r]} vs {ref}"
        # thread invariance: every row is computed by one participant with the same kernel
        orc.set_threads(1)
        y1 = orc.matmul(t, w, rows, width, x)[0]
        orc.set_threads(0)
        assert np.array_equal(y.view(np.uint32), y1.view(np.uint32))


def _rowwise(got, want, k, width, label):
    got = got.reshape(-1, width)
    want = want.reshape(-1, width)
    for r in range(got.shape[0]):
        fin = np.isfinite(want[r])
        max_abs = float(np.max(np.abs(want[r][fin]))) if fin.any() else 0.0
        bud = G.budget(k, width, max_abs)
        d = np.abs(got[r].astype(np.float64) - want[r].astype(np.float64))
        assert np.all(d[fin] <= bud), f"{label} row {r}: {d[fin].max()} > {bud}"


@pytest.mark.parametrize("libm", [0, 1])
def test_rmsnorm_within_budget(orc, libm):
    orc.set_libm(libm)
    try:
        meta, a = G.load("rmsnorm")
        for c in meta["cases"]:
            x, w, y = a[c["case"] + "__x"], a[c["case"] + "__w_gguf"], a[c["case"] + "__y"]
            if c["kind"] == "rmsnorm":
                got = orc.rmsnorm(x, w, c["eps"])
            else:
                got = orc.rmsnorm_gated(x, a[c["case"] + "__gate"], w, c["eps"])
            _rowwise(got, y, meta["budget_k"], c["width"], c["case"])
    finally:
        orc.set_libm(0)


@pytest.mark.parametrize("libm", [0, 1])
def test_softmax_within_budget(orc, libm):
    orc.set_libm(libm)
    try:
        meta, a = G.load("softmax")
        k = meta["budget_k"]
        for c in meta["cases"]:
            if c["kind"] == "softmax":
                x, y = a[c["case"] + "__x"], a[c["case"] + "__y"]
                got = np.stack([orc.softmax(row) for row in x])
                _rowwise(got, y, k, c["width"], c["case"])
            else:
                s, y = a[c["case"] + "__scores"], a[c["case"] + "__y"]
                t = c["t"]
                for i in range(t):
                    got = np.zeros(t, np.float32)
                    got[:i + 1] = orc.softmax(s[i, :i + 1])
                    assert np.all(got[i + 1:] == 0.0)
                    assert np.all(np.abs(got - y[i]) <= G.budget(k, t, 1.0)), c["case"]
    finally:
        orc.set_libm(0)


def test_rope_within_budget(orc):
    meta, a = G.load("rope")
    k = meta["budget_k"]
    for c in meta["cases"]:
        hd, rd = c["head_dim"], c["rope_dim"]
        inv = orc.inv_freq(rd, c["theta"])
        assert np.all(np.abs(inv - a[c["case"] + "__inv_freq"]) <= G.budget(k, 1, 1.0) * np.abs(a[c["case"] + "__inv_freq"]) + 1e-30)
        for name in ("q", "k"):
            x = a[c["case"] + "__" + name]  # [heads, positions, head_dim]
            want = a[c["case"] + "__" + name + "_out"]
            for pi, pos in enumerate(c["positions"]):
                cos, sin = orc.cos_sin(pos, inv)
                assert np.all(np.abs(cos - a[c["case"] + "__cos"][pi]) <= G.budget(k, 1, 1.0))
                got = orc.apply_rope(x[:, pi, :].reshape(-1), hd, rd, cos, sin).reshape(-1, hd)
                bud = G.budget(k, 2, c["max_abs"])
                assert np.all(np.abs(got - want[:, pi, :]) <= bud), (c["case"], name, pos)


def test_act_within_budget(orc):
    meta, a = G.load("act")
    for c in meta["cases"]:
        if c["kind"] == "silu":
            x, y = a["silu__x"], a["silu__y"]
            got = orc.silu(x)
        else:
            got = orc.swiglu(a["swiglu__gate"], a["swiglu__up"])
            y = a["swiglu__y"]
        fin = np.isfinite(y)
        bud = meta["budget_k"] * G.EPS * np.maximum(np.abs(y[fin].astype(np.float64)), np.finfo(np.float32).tiny)
        assert np.all(np.abs(got[fin].astype(np.float64) - y[fin]) <= bud), c["case"]


def test_conv1d_within_budget(orc):
    meta, a = G.load("conv1d")
    k = meta["budget_k"]
    for c in meta["cases"]:
        kern = c["kernel"]
        w = a[c["case"] + "__w"]
        bud = G.budget(k, kern, c["max_abs"])
        if c["kind"] == "conv_step":
            out, st = orc.conv1d_step(a[c["case"] + "__state"], w, kern, a[c["case"] + "__x_new"])
            assert np.all(np.abs(out - a[c["case"] + "__out"]) <= bud), c["case"]
            assert np.array_equal(st, a[c["case"] + "__new_state"]), c["case"]
        else:
            ch, t = c["channels"], c["t"]
            st = np.zeros((ch, kern - 1), np.float32)
            x = a[c["case"] + "__x"]
            want = a[c["case"] + "__out"]
            for i in range(t):
                out, st = orc.conv1d_step(st, w, kern, x[:, i].copy())
                assert np.all(np.abs(out - want[:, i]) <= bud), (c["case"], i)


def test_deltanet_step_within_budget(orc):
    meta, a = G.load("deltanet")
    k = meta["budget_k"]
    for c in meta["cases"]:
        h, dk, dv = c["heads"], c["dk"], c["dv"]
        g = lambda n: a[c["case"] + "__" + n]
        for p in range(h):
            gg = orc.gate_g(float(g("a")[p]), float(g("dt_bias")[p]), float(g("ssm_a")[p]))
            beta = orc.gate_beta(float(g("b")[p]))
            assert abs(gg - g("g")[p]) <= G.budget(k, 1, abs(float(g("g")[p])))
            assert abs(beta - g("beta")[p]) <= G.budget(k, 1, 1.0)
            q = orc.l2norm(g("q")[p])
            kk = orc.l2norm(g("k")[p])
            q = (q * np.float32(1.0 / np.sqrt(np.float32(dk)))).astype(np.float32)
            out, s = orc.deltanet_step(q, kk, g("v")[p], gg, beta, g("state")[p].reshape(-1))
            ma = c["max_abs"]
            assert np.all(np.abs(out - g("out")[p]) <= G.budget(k, dk, ma)), (c["case"], p)
            assert np.all(np.abs(s - g("new_state")[p].reshape(-1)) <= G.budget(k, dk, ma)), (c["case"], p)


def test_argmax_first_on_ties(orc):
    v = np.array([1.0, 3.0, 2.0, 3.0], np.float32)
    assert orc.argmax(v) == 1


# --------------------------------------------------------------------- the sampler (crates/core/src/sample.rs)

def _xoshiro_py(seed, n):
    """splitmix64 seeding + xoshiro256** (Blackman & Vigna), restated independently in Python."""
    M = (1 << 64) - 1
    x, s = seed, []
    for _ in range(4):
        x = (x + 0x9E3779B97F4A7C15) & M
        z = x
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        s.append(z ^ (z >> 31))
    rotl = lambda v, k: ((v << k) | (v >> (64 - k))) & M
    out = []
    for _ in range(n):
        out.append((rotl((s[1] * 5) & M, 7) * 9) & M)
        t = (s[1] << 17) & M
        s[2] ^= s[0]; s[3] ^= s[1]; s[1] ^= s[2]; s[0] ^= s[3]; s[2] ^= t
        s[3] = rotl(s[3], 45)
    return out


def test_sampler_rng_is_xoshiro256starstar_seeded_by_splitmix64(orc):
    for seed in (0, 1, 42, 2**63 + 5):
        assert orc.rng_u64(seed, 64) == _xoshiro_py(seed, 64)


def test_sampler_keeps_the_reference_sets(orc):
    """sample.rs:492-517: top-k, top-p (the crossing token stays), min-p and greedy on six logits."""
    logits = np.array([1.0, 2.0, 3.0, 0.0, -1.0, 4.0], np.float32)
    ids, ps = orc.OracleSampler(6, 1.0, top_k=3, seed=1).process(logits)
    assert ids == [5, 2, 1] and abs(float(ps.sum()) - 1.0) < 1e-6
    assert orc.OracleSampler(6, 1.0, top_p=0.5, seed=1).process(logits)[0] == [5]
    assert orc.OracleSampler(6, 1.0, top_p=0.9, seed=1).process(logits)[0] == [5, 2, 1]
    assert orc.OracleSampler(6, 1.0, top_p=0.85, seed=1).process(logits)[0] == [5, 2]
    assert orc.OracleSampler(6, 1.0, min_p=0.2, seed=1).process(logits)[0] == [5, 2]
    g = orc.OracleSampler(6, 0.0)
    assert g.process(logits)[0] == [5] and g.sample(logits) == 5


def test_sampler_seeded_draws_are_reproducible(orc):
    """sample.rs:518-529: the same seed gives the same 200 draws, another seed others."""
    logits = np.array([((i * 7919) % 101) / 10.0 for i in range(1000)], np.float32)
    mk = lambda seed: orc.OracleSampler(1000, 1.0, top_k=20, top_p=0.95, seed=seed)
    a, b, c = mk(42), mk(42), mk(43)
    xa = [a.sample(logits) for _ in range(200)]
    assert xa == [b.sample(logits) for _ in range(200)]
    assert xa != [c.sample(logits) for _ in range(200)]
    ids, _ = mk(1).process(logits)
    assert set(xa) <= set(ids)


def test_sampler_accept_rule(orc):
    """accept_or_resample (sample.rs:279-313): a draft drawn from q = p is always accepted; with q putting all
    its mass on a token p does not keep, the draft is rejected and the resample comes from p's kept set."""
    logits = np.array([((i * 31) % 17) / 4.0 for i in range(64)], np.float32)
    s = orc.OracleSampler(64, 0.8, top_k=10, top_p=0.9, seed=7)
    ids, ps = s.process(logits)
    q = np.zeros(64, np.float32)
    q[ids] = ps
    for d in ids:
        assert s.accept(logits, q, d) == (True, d)
    outside = next(i for i in range(64) if i not in ids)
    q2 = np.zeros(64, np.float32)
    q2[outside] = 1.0
    ok, tok = s.accept(logits, q2, outside)
    assert not ok and tok in ids


@pytest.mark.parametrize("t", [12, 13, 14, 8, 2])
def test_simd_matmul_bit_identical_to_scalar(orc, t):
    """The timed baseline's AVX2 kernels (blocked over up to 16 columns) give the scalar restatement's bits --
    the reference asks the same of its own AVX2 path (tests/avx2.rs): random blocks, blocks at the integer
    extremes, hostile activation rows, 1..17 columns."""
    from helpers import hostile_rows, random_blocks

    rows, cols = 37, 2048
    w = random_blocks(t, rows, cols, seed=5 + t)
    bb = {12: 144, 13: 176, 14: 210, 8: 34, 2: 18}[t]
    wx = w.reshape(-1, bb).copy()
    if t in (12, 13):
        wx[::3, 4:] = 0xFF  # every third block: maximal codes, scales and mins
    elif t == 14:
        wx[::3, :192] = 0xFF
        wx[::3, 192:208] = 0x80
    elif t == 8:
        wx[::3, 2:] = 0x80  # -128 codes
    w = wx.reshape(-1)
    x = np.concatenate([hostile_rows(cols, 3), np.random.default_rng(t).standard_normal((7, cols)).astype(np.float32)])
    x = np.nan_to_num(x, posinf=0, neginf=0)
    try:
        orc.set_simd(0)
        want = orc.matmul(t, w, rows, cols, x)
        orc.set_simd(1)
        got = orc.matmul(t, w, rows, cols, x)
        for n in (1, 3, 16):
            got_n = orc.matmul(t, w, rows, cols, x[:n])
            assert np.array_equal(got_n.view(np.uint32), want[:n].view(np.uint32)), (t, n)
    finally:
        orc.set_simd(-1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
