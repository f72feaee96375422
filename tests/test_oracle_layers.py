"""Pin the oracle's layer code -- the DeltaNet mixer, the gated GQA mixer, the MLP and both decoder layers, i.e.
the functions its forward_token runs -- against the reference's HF-derived layer fixtures (tests/golden/layers,
from the reference's tests/fixtures/layers/layers), exactly as the reference's own crates/core/tests/layers.rs
checks its layers: F32 weights, a prefill of t rows, then one step on the carried state / KV cache, each output
within k * sqrt(width) * eps * max|reference| (k from the fixture manifest, width the layer's largest reduction
length).  The carried DeltaNet state, conv window and KV caches are checked the same way.  CPU only."""
import numpy as np
import pytest

import golden_io as G


def _fx():
    meta, a = G.load("layers")
    cases = {c["case"]: c for c in meta["cases"]}
    return meta, a, cases


def _dims(meta):
    c = meta["config"]
    hd = c["head_dim"]
    return dict(hidden=c["hidden_size"], ffn=c["intermediate_size"], n_head=c["num_attention_heads"],
                n_kv=c["num_key_value_heads"], head_dim=hd, rope_dim=int(hd * c["rope_parameters"]["partial_rotary_factor"]),
                conv_kernel=c["linear_conv_kernel_dim"], dk=c["linear_key_head_dim"], n_k=c["linear_num_key_heads"],
                n_v=c["linear_num_value_heads"], dv=c["linear_value_head_dim"], eps=c["rms_norm_eps"],
                theta=c["rope_parameters"]["rope_theta"])


def _weights(a, case):
    pre = case["case"] + "__w__"
    return {n: a[pre + n] for n in case["weights"]}


def _check(label, got, want, width, k):
    """crates/core/tests/layers.rs check(): max |got - want| <= k sqrt(width) eps max|want|."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    assert got.shape == want.shape, label
    bud = G.budget(k, width, float(np.max(np.abs(want))))
    d = float(np.max(np.abs(got - want)))
    assert d <= bud, f"{label}: max |diff| {d:.3e} exceeds the budget {bud:.3e}"
    return d / bud if bud > 0 else 0.0


def _hf_conv_window(a, name, kernel):
    """HF keeps `kernel` samples per channel ([conv_dim, kernel]); the last kernel - 1 feed the next step
    (layers.rs hf_conv_window)."""
    w = a[name]
    return w[:, w.shape[1] - (kernel - 1):]


def test_deltanet_layer_prefill_and_step(orc):
    meta, a, cases = _fx()
    c = cases["deltanet_layer"]
    d = _dims(meta)
    k = meta["budget_k"]
    lay = orc.LayerF32("deltanet", d, _weights(a, c))
    width = max(d["hidden"], d["dk"] * d["dv"])
    x = a["deltanet_layer__prefill__x"]
    y = lay(x)
    _check("deltanet prefill vs HF chunk kernel", y, a["deltanet_layer__prefill__y"], width, k)
    _check("deltanet prefill vs HF sequential recurrence", y, a["deltanet_layer__prefill__y_seq"], width, k)
    _check("deltanet prefill recurrent state", lay.S, a["deltanet_layer__prefill__rec_state"], width, k)
    _check("deltanet prefill conv window", lay.conv,
           _hf_conv_window(a, "deltanet_layer__prefill__conv_state", d["conv_kernel"]), d["hidden"], k)
    y1 = lay(a["deltanet_layer__step__x"])
    _check("deltanet step with carried state", y1, a["deltanet_layer__step__y"], width, k)
    _check("deltanet step recurrent state", lay.S, a["deltanet_layer__step__rec_state"], width, k)
    _check("deltanet step conv window", lay.conv,
           _hf_conv_window(a, "deltanet_layer__step__conv_state", d["conv_kernel"]), d["hidden"], k)


def test_attention_layer_prefill_and_step(orc):
    meta, a, cases = _fx()
    c = cases["attention_layer"]
    d = _dims(meta)
    assert d["rope_dim"] == c["rope_dim"] and d["head_dim"] == c["head_dim"]
    k = meta["budget_k"]
    lay = orc.LayerF32("attention", d, _weights(a, c))
    t = c["t"]
    width = max(d["hidden"], d["head_dim"], t)
    y = lay(a["attention_layer__prefill__x"])
    _check("attention prefill", y, a["attention_layer__prefill__y"], width, k)
    # KV cache: HF stores (n_kv, T, head_dim) post-RoPE keys; here [T][n_kv * head_dim]
    nkv, hd = d["n_kv"], d["head_dim"]
    k_ours = lay.K[:t].reshape(t, nkv, hd).transpose(1, 0, 2)
    v_ours = lay.V[:t].reshape(t, nkv, hd).transpose(1, 0, 2)
    _check("attention K cache (post-RoPE)", k_ours, a["attention_layer__prefill__k_cache"], d["hidden"], k)
    _check("attention V cache", v_ours, a["attention_layer__prefill__v_cache"], d["hidden"], k)
    assert lay.pos == c["step"]["position"]
    y1 = lay(a["attention_layer__step__x"])
    _check("attention step with KV cache", y1, a["attention_layer__step__y"], width, k)


def test_rope_tables_match_the_fixture_cos_sin(orc):
    """The attention fixture's cos/sin rows (positions 0..t) against the oracle's tables (rope.rs:10-29)."""
    meta, a, cases = _fx()
    c = cases["attention_layer"]
    d = _dims(meta)
    inv = orc.inv_freq(d["rope_dim"], d["theta"])
    for pos in range(c["t"]):
        co, si = orc.cos_sin(pos, inv)
        _check(f"cos at {pos}", co, a["attention_layer__prefill__cos"][pos], d["rope_dim"], meta["budget_k"])
        _check(f"sin at {pos}", si, a["attention_layer__prefill__sin"][pos], d["rope_dim"], meta["budget_k"])


def test_mlp_layer(orc):
    meta, a, cases = _fx()
    c = cases["mlp_layer"]
    d = _dims(meta)
    lay = orc.LayerF32("mlp", d, _weights(a, c))
    y = lay(a["mlp_layer__prefill__x"])
    _check("mlp", y, a["mlp_layer__prefill__y"], d["ffn"], meta["budget_k"])


@pytest.mark.parametrize("kind", ["linear_attention", "full_attention"])
def test_decoder_layer_prefill_and_step(orc, kind):
    """layers.rs decoder_layers_prefill_and_step: t token steps, then one more on the carried state."""
    meta, a, cases = _fx()
    name = f"decoder_{kind}"
    c = cases[name]
    d = _dims(meta)
    k = meta["budget_k"]
    lay = orc.LayerF32("decoder_deltanet" if kind == "linear_attention" else "decoder_attention", d, _weights(a, c))
    width = max(d["hidden"], d["ffn"])
    y = lay(a[name + "__prefill__x"])
    _check(f"decoder {kind} prefill", y, a[name + "__prefill__y"], width, k)
    assert lay.pos == c["step"]["position"]
    y1 = lay(a[name + "__step__x"])
    _check(f"decoder {kind} step", y1, a[name + "__step__y"], width, k)


def test_layer_outputs_are_deterministic(orc):
    """Repeated runs give the same bits (the reference's thread-invariance checks; the oracle is single-order)."""
    meta, a, cases = _fx()
    c = cases["decoder_linear_attention"]
    d = _dims(meta)
    ys = []
    for _ in range(2):
        lay = orc.LayerF32("decoder_deltanet", d, _weights(a, c))
        ys.append(lay(a["decoder_linear_attention__prefill__x"]))
    assert np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32))
