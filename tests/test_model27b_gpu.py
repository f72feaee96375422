"""GPU parity at the 27B dimensions against the CPU oracle, on the `27b-L4` synthetic checkpoint: the full 27B
widths (hidden 5120, DeltaNet 16 K / 48 V heads of 128, GQA 24 q / 4 kv heads of 256 with rope_dim 64 in sections
{11, 11, 10}, FFN 17408, vocabulary 248320, the Q4_K_M type recipe, the MTP block) with 4 layers (3 DeltaNet + 1
attention).  This runs the kernels the headline runs -- deltanet_halves<128>, head_dim-256 attention, the
248320-row lm_head and argmax -- against the oracle:

  - every layer's residual row, the post-final-norm row and the logits, bit for bit, over 6 positions;
  - greedy ids after a batched prompt (the prefill's multi-row path);
  - --spec 3 ids (equal to plain decoding and to the oracle's spec loop, with the same round / accept counts);
  - forced drafts reaching every acceptance count 0..3, and after every round the whole carried state (DeltaNet
    states, conv windows, KV rows [0, pos), position) bit-identical to a plain state that stepped through the
    same tokens -- the reference's crates/core/tests/spec_identity.rs:1-9 -- and, at the end, to the oracle's.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PRESET = "27b-L4"
SEED = 20261201
K = 3
MAX_POS = 512


def _prompt(n, seed):
    return [int(v) for v in np.random.default_rng(seed).integers(0, 248044, n)]


@pytest.fixture(scope="module")
def ck27(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qdec

    base = "/dev/shm" if os.path.isdir("/dev/shm") else str(tmp_path_factory.mktemp("ck27"))
    path = os.path.join(base, f"qdec_test_{PRESET}_{SEED}_{os.getpid()}.gguf")
    qdec.synth_gguf(path, PRESET, SEED)
    yield path
    os.remove(path)


@pytest.fixture(scope="module")
def m27(ck27):
    import qdec

    m = qdec.Model(ck27, max_pos=MAX_POS)
    yield m
    m.close()


@pytest.fixture(scope="module")
def o27(ck27, orc):
    orc.set_threads(os.cpu_count() or 1)
    om = orc.OracleModel(ck27)
    yield om
    om.close()


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_27b_dimensions(m27):
    i = m27.info
    assert (i.hidden, i.ffn, i.vocab, i.n_head, i.n_head_kv, i.head_dim) == (5120, 17408, 248320, 24, 4, 256)
    assert (i.dn_n_k_heads, i.dn_n_v_heads, i.dn_head_dim_k, i.dn_head_dim_v, i.n_layer, i.has_mtp) == (16, 48, 128, 128, 4, 1)


def test_hidden_states_and_logits_bit_exact_27b(m27, o27):
    """Every layer's residual row, the post-final-norm row and the logits at 6 positions, bit for bit."""
    st = m27.new_state(max_rows=1)
    st.set_capture(True)
    os_ = o27.state(MAX_POS)
    for pos, tok in enumerate(_prompt(6, SEED + 11)):
        st.step(tok)
        lg, cap = os_.forward_token(tok, capture=True)
        for layer in range(m27.info.n_layer + 1):
            h = st.hidden(layer)
            bad = np.flatnonzero(_bits(h) != _bits(cap[layer]))
            assert bad.size == 0, f"layer {layer} at position {pos}: {bad.size} of 5120 differ (first {bad[:4]})"
        g = st.logits(0)
        bad = np.flatnonzero(_bits(g) != _bits(lg))
        assert bad.size == 0, f"logits at position {pos}: {bad.size} differ"
    st.free()


def test_greedy_ids_27b(m27, o27):
    """An 8-token prompt prefilled as one batch, then 8 greedy tokens: the oracle's ids."""
    import qdec

    p = _prompt(8, SEED + 1)
    want = o27.state(MAX_POS).generate(p, 8, stop=False)
    got = qdec.generate(m27.new_state(max_rows=32), p, 8, stop=False)
    assert got == want


def test_spec3_ids_27b(m27, o27):
    """--spec 3: ids equal plain decoding and the oracle's spec loop, with its round and acceptance counts."""
    import qdec

    p = _prompt(6, SEED + 2)
    n = 6
    plain = qdec.generate(m27.new_state(max_rows=32), p, n, stop=False)
    st = m27.new_state(spec_k=K, max_rows=32)
    got = qdec.generate_spec(st, p, n, stop=False)
    assert got == plain
    want, stats, _ = o27.state(MAX_POS).spec_generate(p, n, K, stop=False)
    assert want == plain
    c = st.counters()
    assert c["rounds"] == stats["rounds"] and c["accepted"] == stats["accepted"]


def _carried(st, n_layer):
    out = {}
    for layer in range(n_layer):
        for what in range(4):
            v = st.carried(layer, what)
            if v is not None:
                out[(layer, what)] = v
    return out


def test_forced_drafts_every_acceptance_count_and_carried_state_27b(m27, o27):
    """Forced drafts (the plain run's next tokens, one wrong at position j, so exactly j are accepted) reach every
    acceptance count; after every round the spec state's whole carried state equals, bit for bit, that of a plain
    state stepped through the same tokens (spec_identity.rs:5-9), and the ids equal plain decoding and the
    oracle's spec loop under the same forced drafts; the final carried state equals the oracle's."""
    import qdec

    n_layer = m27.info.n_layer
    p = _prompt(5, SEED + 3)
    n_tokens = 12
    plain_ids = qdec.generate(m27.new_state(max_rows=32), p, n_tokens + K + 2, stop=False)
    st = m27.new_state(spec_k=K, max_rows=32)
    ref = m27.new_state(max_rows=32)  # the plain state, stepped through the tokens the spec state consumes
    seq = [st.spec_prefill(p)]
    assert ref.prefill(p) == seq[0]
    consumed = list(p)
    forced, hist, r = [], [0] * (K + 1), 0
    while len(seq) < n_tokens:
        want = plain_ids[len(seq):len(seq) + K]
        miss = r % (K + 1)
        d = list(want)
        if miss < K:
            d[miss] = (d[miss] + 1) % 248044
        forced.append(d)
        st.set_drafts(d)
        x_p = seq[-1]
        em = st.spec_round(x_p)
        assert len(em) == miss + 1 if miss < K else len(em) == K + 1
        hist[len(em) - 1] += 1
        fed = [x_p] + em[:-1]  # the rows the round kept: x_p and the accepted drafts
        for tok in fed:
            ref.step(tok)
        consumed += fed
        seq += em
        r += 1
        assert st.pos == ref.pos == len(consumed)
        a, b = _carried(st, n_layer), _carried(ref, n_layer)
        assert a.keys() == b.keys() and len(a) == 3 * 2 + 2
        for key in a:
            bad = np.flatnonzero(_bits(a[key]) != _bits(b[key]))
            assert bad.size == 0, f"round {r}: carried state {key} differs from the plain state's in {bad.size} places"
    assert seq[:n_tokens] == plain_ids[:n_tokens]
    assert all(h > 0 for h in hist), hist
    want, stats, _ = o27.state(MAX_POS).spec_generate(p, len(seq), K, stop=False, forced=forced)
    assert want[: len(seq)] == seq
    # the final carried state against the oracle's after the same tokens
    ost = o27.state(MAX_POS)
    for tok in consumed:
        ost.forward_token(tok, logits=False)
    for (layer, what), v in _carried(st, n_layer).items():
        o = ost.carried(layer, what)
        assert o is not None and o.size == v.size, (layer, what)
        bad = np.flatnonzero(_bits(v) != _bits(o))
        assert bad.size == 0, f"carried state {(layer, what)} differs from the oracle's in {bad.size} places"


# tensors a tensor-parallel rank slices by rows (each row on exactly one rank at these dimensions); every other
# tensor is held whole by every rank, and the three per-head DeltaNet vectors are also sliced from that copy
SLICED = ("attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight", "attn_qkv.weight", "attn_gate.weight",
          "ssm_alpha.weight", "ssm_beta.weight", "ssm_out.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight",
          "nextn.eh_proj.weight")
VEC_SLICED = ("ssm_a", "ssm_dt.bias", "ssm_conv1d.weight")


def test_tp_rank_holds_its_share_not_the_whole_model(ck27):
    """A tensor-parallel rank allocates the replicated tensors plus its slices, not the whole data section: over
    the two ranks of world 2 the weight bytes add up to 2 x replicated + every sliced byte once, each rank's device
    memory grows by its weight bytes (plus the RoPE tables and allocation rounding), well under the whole model."""
    import qdec
    from helpers import gguf_tensors

    ts = gguf_tensors(ck27)
    total = sum(b for _, _, _, b in ts)
    names = {n for n, _, _, _ in ts}
    tied = "output.weight" not in names
    sliced = sum(b for n, _, _, b in ts if n.endswith(SLICED) or n == "output.weight")
    replicated = total - sliced
    vec_sliced = sum(b for n, _, _, b in ts if n.endswith(VEC_SLICED))
    lm_from_embd = sum(b for n, _, _, b in ts if n == "token_embd.weight") if tied else 0
    got = []
    for rank in range(2):
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        m = qdec.Model(ck27, max_pos=64, tp=(rank, 2))
        torch.cuda.synchronize()
        grew = free0 - torch.cuda.mem_get_info()[0]
        wb = m.info.weight_bytes
        m.close()
        got.append(wb)
        assert wb < 0.75 * total, f"rank {rank} holds {wb} of {total} bytes"
        assert wb <= grew <= wb + (512 << 20), f"rank {rank}: device memory grew by {grew}, weight bytes {wb}"
    assert sum(got) == 2 * replicated + sliced + vec_sliced + lm_from_embd


def test_batch_step_27b(m27, o27):
    """Four sequences decoded together at the 27B dimensions (the 4-column GEMVs and the fused gate/up/SwiGLU
    over four sequences' rows; DeltaNet<128>, head_dim 256 attention and rope per sequence): each sequence's
    greedy ids equal its own decoding and the oracle's."""
    import qdec

    prompts = [_prompt(n, SEED + 20 + n) for n in (5, 3, 2, 1)]
    n = 4
    got = qdec.generate_batch([m27.new_state(max_rows=8) for _ in prompts], prompts, n)
    for p, g in zip(prompts, got):
        assert qdec.generate(m27.new_state(max_rows=8), p, n, stop=False) == g
        assert o27.state(MAX_POS).generate(p, n, stop=False) == g


def test_direct_io_load_27b_dims(ck27, m27, tmp_path, monkeypatch):
    """The O_DIRECT load over many 256 MiB staging chunks (the 4-layer 27B-dimension checkpoint copied to a disk
    path): the same greedy ids as the buffered load."""
    import shutil

    import qdec

    path = tmp_path / "ck27_direct.gguf"
    shutil.copy(ck27, path)
    try:
        if not _odirect_ok(str(path)):
            pytest.skip("the temporary directory's file system refuses O_DIRECT")
        monkeypatch.setenv("QDEC_LOAD_DIRECT", "1")
        m = qdec.Model(path, max_pos=MAX_POS)
        try:
            assert m.loaded_direct
            p = _prompt(4, SEED + 31)
            got = qdec.generate(m.new_state(max_rows=8), p, 3, stop=False)
        finally:
            m.close()
        assert got == qdec.generate(m27.new_state(max_rows=8), p, 3, stop=False)
    finally:
        os.remove(path)


def _odirect_ok(path):
    try:
        os.close(os.open(path, os.O_RDONLY | os.O_DIRECT))
        return True
    except OSError:
        return False
