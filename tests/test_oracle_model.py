"""The oracle's model-level forms against each other on the tiny synthetic checkpoint (CPU only): the batched
prefill / verify / MTP re-feed (the reference's forward_batch_in, matmul_t and rows_in) give the token form's bits,
the speculative loop with the reference's rollback (snapshot restore + replay of the kept rows' recurrence from
the verify's saved projections, spec.rs:395-415) gives plain decoding's ids for k = 1..4 and under forced drafts
that reach every acceptance count (crates/core/tests/spec_identity.rs), and the AVX2 kernels change no id."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SEED = 20261201


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    sys.path.insert(0, os.path.join(ROOT, "qwen-3.8-in-rust_b200"))
    try:
        import qdec

        qdec.lib()
    except (ImportError, OSError) as e:
        pytest.skip(f"the library that writes the synthetic checkpoint is not built: {e}")
    path = tmp_path_factory.mktemp("tiny") / "tiny.gguf"
    qdec.synth_gguf(path, "tiny", SEED)
    return path


@pytest.fixture(scope="module")
def om(tiny, orc):
    m = orc.OracleModel(tiny)
    yield m
    m.close()


def prompt(n, seed=SEED + 1):
    return [int(v) for v in np.random.default_rng(seed).integers(0, 4096, n)]


def token_form_generate(om, p, n):
    st = om.state(512)
    lg = None
    for tok in p:
        lg, _ = st.forward_token(tok)
    out = [int(np.argmax(lg))]
    while len(out) < n:
        lg, _ = st.forward_token(out[-1])
        out.append(int(np.argmax(lg)))
    return out, lg


def test_batched_prefill_equals_token_form(om):
    p = prompt(40)  # three batches of 16, 16 and 8 rows
    want, _ = token_form_generate(om, p, 12)
    assert om.state(512).generate(p, 12, stop=False) == want


@pytest.mark.parametrize("k", [1, 2, 3, 4])
def test_spec_ids_equal_plain(om, k):
    p = prompt(16)
    plain = om.state(512).generate(p, 32, stop=False)
    got, stats, _ = om.state(512).spec_generate(p, 32, k, stop=False)
    assert got == plain
    assert stats["rounds"] > 0


def test_forced_drafts_every_acceptance_count(om):
    k = 3
    p = prompt(16)
    plain = om.state(512).generate(p, 48, stop=False)
    forced, pos = [], 1
    for r in range(12):
        miss = r % (k + 1)
        d = list(plain[pos:pos + k])
        if miss < k:
            d[miss] = (d[miss] + 1) % 4096
        forced.append(d)
        pos += miss + 1 if miss < k else k + 1
    got, stats, _ = om.state(512).spec_generate(p, pos, k, stop=False, forced=forced)
    assert got == plain[:pos]
    assert stats["accepted"] == sum(min(r % (k + 1), k) for r in range(12))


def test_simd_and_scalar_give_the_same_ids(om, orc):
    p = prompt(16, SEED + 5)
    try:
        orc.set_simd(0)
        want = om.state(512).spec_generate(p, 16, 3, stop=False)[0]
        orc.set_simd(1)
        got = om.state(512).spec_generate(p, 16, 3, stop=False)[0]
    finally:
        orc.set_simd(-1)
    assert got == want
