"""GPU parity of the whole decode path (the tiny synthetic Qwen3.8-style checkpoint, the reference's CPU-runnable
toy) against the CPU oracle: greedy ids, per-layer hidden states and logits, the --spec 3 loop (ids identical to plain decoding
and to the oracle, MTP drafts identical), and forced drafts that exercise every acceptance count
(the device of crates/core/tests/spec_identity.rs)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SEED = 20261201
N_TOKENS = 32


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qdec

    path = tmp_path_factory.mktemp("tiny") / "tiny.gguf"
    qdec.synth_gguf(path, "tiny", SEED)
    return path


@pytest.fixture(scope="module")
def model(tiny):
    import qdec

    return qdec.Model(tiny, max_pos=512)


@pytest.fixture(scope="module")
def omodel(tiny, orc):
    return orc.OracleModel(tiny)


def prompt16():
    return [int(v) for v in np.random.default_rng(SEED + 1).integers(0, 4096, 16)]


def test_config_from_synthetic_gguf(model):
    i = model.info
    assert (i.n_layer, i.hidden, i.ffn, i.vocab, i.n_head, i.n_head_kv, i.head_dim) == (4, 256, 768, 4096, 4, 2, 64)
    assert (i.dn_n_k_heads, i.dn_n_v_heads, i.dn_head_dim_k, i.dn_head_dim_v, i.n_full_attention, i.has_mtp) == (2, 4, 64, 64, 1, 1)


def test_greedy_ids_match_oracle(model, omodel):
    import qdec

    p = prompt16()
    want = omodel.state(512).generate(p, N_TOKENS, stop=False)
    got = qdec.generate(model.new_state(), p, N_TOKENS, stop=False)
    assert got == want


@pytest.mark.parametrize("mma_min", [4, 1])
def test_hidden_states_and_logits_bit_exact(model, omodel, mma_min):
    """Every layer's residual row and the logits of every prompt position, bit for bit; with mma_min = 1 the
    one-column steps take the warp-MMA Q4_K GEMV (the gate/up pair with its SwiGLU epilogue included)."""
    import qdec

    p = prompt16()
    st = model.new_state(max_rows=1)
    st.set_capture(True)
    os_ = omodel.state(512)
    qdec.tune_gemv(10, mma_min)
    try:
        for tok in p[:6]:
            st.step(tok)
            lg, cap = os_.forward_token(tok, capture=True)
            for layer in range(model.info.n_layer + 1):
                h = st.hidden(layer)
                assert np.array_equal(h.view(np.uint32), cap[layer].view(np.uint32)), f"layer {layer} at position {os_.pos - 1}"
            assert np.array_equal(st.logits(0).view(np.uint32), lg.view(np.uint32))
    finally:
        qdec.tune_gemv(10, qdec.GEMV_MMA_MIN_COLS)


def test_batched_prefill_equals_token_steps(model):
    """Row i of a batched forward == forward_token on row i (crates/core/tests/matmul_t.rs, spec.md:31-34)."""
    p = prompt16()
    a = model.new_state(max_rows=32)
    b = model.new_state(max_rows=1)
    first_a = a.prefill(p)
    first_b = None
    for tok in p:
        first_b = b.step(tok)
    assert first_a == first_b
    ga = [first_a] + [a.step(0) for _ in range(3)]
    gb = [first_b] + [b.step(0) for _ in range(3)]
    assert ga == gb


@pytest.mark.parametrize("k", [1, 2, 3, 4])
def test_spec_ids_equal_plain_and_oracle(model, omodel, k):
    import qdec

    p = prompt16()
    plain = qdec.generate(model.new_state(), p, N_TOKENS, stop=False)
    st = model.new_state(spec_k=k)
    got = qdec.generate_spec(st, p, N_TOKENS, stop=False)
    assert got == plain
    want, stats, _ = omodel.state(512).spec_generate(p, N_TOKENS, k, stop=False)
    assert want == plain
    c = st.counters()
    assert c["rounds"] == stats["rounds"] and c["accepted"] == stats["accepted"]


def test_mtp_drafts_match_oracle(model, omodel):
    """The drafts the MTP head proposes each round, compared with the oracle's."""
    k = 3
    p = prompt16()
    st = model.new_state(spec_k=k)
    x = st.spec_prefill(p)
    drafts = [st.drafts()]
    seq = [x]
    for _ in range(6):
        em = st.spec_round(seq[-1])
        seq += em
        drafts.append(st.drafts())
    _, stats, odrafts = omodel.state(512).spec_generate(p, len(seq), k, stop=False)
    assert drafts[: len(odrafts)] == odrafts[: len(drafts)]


def test_forced_drafts_every_acceptance_count(model, omodel):
    """Drafts forced to the plain run's own next tokens with a deliberate miss at position j accept exactly j
    drafts; ids stay identical to plain decoding and to the oracle under the same forced drafts."""
    import qdec

    k = 3
    p = prompt16()
    plain = qdec.generate(model.new_state(), p, N_TOKENS + 8, stop=False)
    st = model.new_state(spec_k=k)
    seq = [st.spec_prefill(p)]
    forced = []
    hist = [0] * (k + 1)
    r = 0
    while len(seq) < N_TOKENS:
        pos = len(seq)  # the next plain token index the verify's row 0 predicts
        want = plain[pos:pos + k]
        miss = r % (k + 1)  # accept exactly `miss` drafts (k = all)
        d = list(want)
        if miss < k:
            d[miss] = (d[miss] + 1) % 4096
        forced.append(d)
        st.set_drafts(d)
        em = st.spec_round(seq[-1])
        hist[len(em) - 1] += 1
        seq += em
        r += 1
    assert seq[:N_TOKENS] == plain[:N_TOKENS]
    assert all(h > 0 for h in hist), hist
    want, stats, _ = omodel.state(512).spec_generate(p, len(seq), k, stop=False, forced=forced)
    assert want[: len(seq)] == seq


@pytest.mark.parametrize("max_pos", [1024, 4096])
def test_long_context_ids_and_logits_match_oracle(tiny, omodel, max_pos):
    """A 700-token prompt: the attention runs over several 256-position score chunks and wraps the value
    stream's stage ring; greedy ids, the last prompt row's logits and --spec 3 ids match the oracle.  With caches
    longer than 2048 positions the attention takes its long-cache form (8 pairs per scores CTA)."""
    import qdec

    m = qdec.Model(tiny, max_pos=max_pos)
    p = [int(v) for v in np.random.default_rng(SEED + 7).integers(0, 4096, 700)]
    want = omodel.state(1024).generate(p, 12, stop=False)
    st = m.new_state(max_rows=32)
    got = qdec.generate(st, p, 12, stop=False)
    assert got == want
    os_ = omodel.state(1024)
    lg = None
    for tok in p[:300]:
        lg, _ = os_.forward_token(tok)
    s1 = m.new_state(max_rows=32)
    s1.prefill(p[:299])
    _, glg = s1.step(p[299], want_logits=True)
    assert np.array_equal(glg.view(np.uint32), lg.view(np.uint32))
    sp = m.new_state(spec_k=3, max_rows=32)
    assert qdec.generate_spec(sp, p, 12, stop=False) == want
    m.close()


SAMPLERS = [dict(temperature=0.8, top_k=20, top_p=0.95, seed=3), dict(temperature=1.0, top_k=0, top_p=1.0, seed=11),
            dict(temperature=0.6, top_k=50, top_p=0.9, min_p=0.05, seed=42)]


@pytest.mark.parametrize("cfg", SAMPLERS)
def test_sampled_ids_match_oracle(model, omodel, orc, cfg):
    """Sampled decoding (crates/core/src/sample.rs, run.rs:313-348): the device's candidate sort, softmax, top-k /
    top-p / min-p, xoshiro256** draws give the oracle's ids, plain and --spec 3 (exact acceptance rule)."""
    import qdec

    p = prompt16()
    st = model.new_state(max_rows=32)
    st.set_sampler(**cfg)
    got = qdec.generate(st, p, N_TOKENS, stop=False)
    want = omodel.state(512).generate(p, N_TOKENS, stop=False, sampler=orc.OracleSampler(4096, **cfg))
    assert got == want
    sp = model.new_state(spec_k=3, max_rows=32)
    sp.set_sampler(**cfg)
    got_s = qdec.generate_spec(sp, p, N_TOKENS, stop=False)
    want_s, stats, _ = omodel.state(512).spec_generate(p, N_TOKENS, 3, stop=False, sampler=orc.OracleSampler(4096, **cfg))
    assert got_s == want_s
    c = sp.counters()
    assert c["rounds"] == stats["rounds"] and c["accepted"] == stats["accepted"]


def test_sampler_switch_to_greedy_mid_sequence(model):
    """temperature 0 after sampled rounds: the captured round is rebuilt greedy, and the continuation equals
    plain greedy decoding from the same history."""
    import qdec

    p = prompt16()
    a = model.new_state(spec_k=3, max_rows=32)
    a.set_sampler(temperature=0.9, top_k=10, seed=1)
    x = a.spec_prefill(p)  # x_T, then sampled rounds (the first captures the sampled round)
    hist = [x]
    for _ in range(4):
        em = a.spec_round(x)
        hist += em
        x = em[-1]
    a.set_sampler(temperature=0.0)
    x = hist[-1]
    cont = []
    while len(cont) < 12:
        em = a.spec_round(x)
        cont += em
        x = em[-1]
    b2 = model.new_state(max_rows=32)  # prefill the same history, then greedy steps
    plain = [b2.prefill(p + hist)]
    while len(plain) < 12:
        plain.append(b2.step(plain[-1]))
    assert cont[:12] == plain


def _carried_all(st, n_layer):
    out = {}
    for layer in range(n_layer):
        for what in range(4):
            v = st.carried(layer, what)
            if v is not None:
                out[(layer, what)] = v
    return out


def test_batch_step_equals_single_sequences(model, omodel):
    """Multi-sequence batching: three sequences of different prompt lengths decoded together (every weight
    read once per step for the three rows) give each sequence's own greedy ids -- the oracle's -- and leave
    every state's carried state (DeltaNet states, conv windows, K/V rows) bit for bit as single stepping does."""
    import qdec

    rng = np.random.default_rng(SEED + 7)
    prompts = [[int(v) for v in rng.integers(0, 4096, n)] for n in (16, 9, 5)]
    n = 12
    batched = [model.new_state(max_rows=4) for _ in prompts]
    got = qdec.generate_batch(batched, prompts, n)
    singles = [model.new_state(max_rows=4) for _ in prompts]
    for st, p, g in zip(singles, prompts, got):
        assert qdec.generate(st, p, n, stop=False) == g
        assert omodel.state(512).generate(p, n, stop=False) == g
    for a, b in zip(batched, singles):
        assert a.pos == b.pos
        ca, cb = _carried_all(a, model.info.n_layer), _carried_all(b, model.info.n_layer)
        assert ca.keys() == cb.keys()
        for key in ca:
            assert np.array_equal(ca[key].view(np.uint32), cb[key].view(np.uint32)), key
    # a batched state continues on its own, and a single state joins a batch
    assert batched[1].step(got[1][-1]) == singles[1].step(got[1][-1])


def test_batch_step_rejects_bad_batches(model):
    import qdec

    a, b = model.new_state(max_rows=1), model.new_state(max_rows=4)
    a.prefill([1, 2, 3])
    b.prefill([4, 5])
    with pytest.raises(qdec.QdecError):
        qdec.batch_step([a, b], [7, 8])  # the first state's rows hold one sequence
    with pytest.raises(qdec.QdecError):
        qdec.batch_step([b, b], [7, 8])  # a state twice
    c = model.new_state(max_rows=4)
    c.set_sampler(temperature=0.8, seed=1)
    with pytest.raises(qdec.QdecError):
        qdec.batch_step([b, c], [7, 8])  # batching is greedy
    assert (a.pos, b.pos) == (3, 2)  # nothing advanced
    qdec.batch_step([b, a], [7, 8])  # the second state needs no spare rows
    assert (a.pos, b.pos) == (4, 3)


def test_model_close_waits_for_its_states(tiny):
    """qdec_close with a state still alive defers the release to the state's qdec_state_free: the state keeps
    decoding after the close, and freeing it afterwards releases the model."""
    import qdec

    m = qdec.Model(tiny, max_pos=64)
    st = m.new_state(max_rows=4)
    a = st.prefill([5, 6, 7])
    m.close()
    assert isinstance(st.step(a), int)
    st.free()


def _takes_odirect(path):
    import os

    try:
        os.close(os.open(path, os.O_RDONLY | os.O_DIRECT))
        return True
    except OSError:
        return False


def test_direct_io_load_equals_buffered(tiny, tmp_path, monkeypatch):
    """QDEC_LOAD_DIRECT=1 (O_DIRECT reads from the block boundary before the data section, the head bytes skipped
    on upload, the last block cut by the end of the file) loads the same weights: greedy ids equal the buffered
    load's; where the file system takes O_DIRECT the direct path was the one used."""
    import shutil

    import qdec

    path = tmp_path / "tiny_direct.gguf"
    shutil.copy(tiny, path)
    p = prompt16()
    monkeypatch.setenv("QDEC_LOAD_DIRECT", "1")
    m = qdec.Model(path, max_pos=64)
    direct = m.loaded_direct
    got = qdec.generate(m.new_state(max_rows=4), p, 8, stop=False)
    m.close()
    monkeypatch.delenv("QDEC_LOAD_DIRECT")
    mb = qdec.Model(path, max_pos=64)
    assert not mb.loaded_direct
    want = qdec.generate(mb.new_state(max_rows=4), p, 8, stop=False)
    mb.close()
    assert got == want
    assert direct == _takes_odirect(str(path))
