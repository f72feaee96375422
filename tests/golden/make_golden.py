"""Extract the golden vectors that pin the CPU oracle from the reference's own test fixtures.

The reference (`aqueduct`, ManeeshJupalle/Qwen-3.8-in-Rust) ships known-answer fixtures under
`tests/fixtures/` that its Rust tests (`crates/core/tests/{q8k,kernels,dequant}.rs`) check its kernels
against.  This script copies a compact subset of them into `tests/golden/*.npz` (+ a JSON manifest per
group) so the parity tests run without the reference tree.  Run it where the reference is mounted:

    python tests/golden/make_golden.py /path/to/reference

Nothing else in this repository reads the reference tree at run time.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_manifest(d):
    with open(os.path.join(d, "manifest.json")) as f:
        return json.load(f)


def npy(d, field):
    return np.load(os.path.join(d, field["file"]))


def raw(d, field):
    with open(os.path.join(d, field["file"]), "rb") as f:
        return np.frombuffer(f.read(), dtype=np.uint8)


def strip(c, keep):
    return {k: v for k, v in c.items() if k in keep}


def save(group, arrays, manifest):
    np.savez_compressed(os.path.join(HERE, group + ".npz"), **arrays)
    with open(os.path.join(HERE, group + ".json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    size = os.path.getsize(os.path.join(HERE, group + ".npz"))
    print(f"{group}: {len(arrays)} arrays, {size / 1024:.0f} KiB")


def main(ref):
    fx = os.path.join(ref, "tests", "fixtures")
    kd = os.path.join(fx, "kernels")

    # --- Q8_K quantiser: bit-exact (tests/fixtures/kernels/q8k_quantize, checked by crates/core/tests/q8k.rs)
    d = os.path.join(kd, "q8k_quantize")
    m = load_manifest(d)
    arrs, cases = {}, []
    for c in m["cases"]:
        arrs[c["case"] + "__x"] = npy(d, c["x"]).astype(np.float32)
        arrs[c["case"] + "__raw"] = raw(d, c["raw"])
        cases.append(strip(c, {"case", "width", "rows"}))
    save("q8k_quantize", arrs, {"source": m["source"], "exact": True, "cases": cases})

    # --- Q8_0 quantiser: bit-exact
    d = os.path.join(kd, "q8_quantize")
    m = load_manifest(d)
    arrs, cases = {}, []
    for c in m["cases"]:
        arrs[c["case"] + "__x"] = npy(d, c["x"]).astype(np.float32)
        arrs[c["case"] + "__raw"] = raw(d, c["raw"])
        cases.append(strip(c, {"case", "width", "rows"}))
    save("q8_quantize", arrs, {"source": m["source"], "exact": True, "cases": cases})

    # --- dot: f64 reference within k*sqrt(n)*eps*max|term| (widths 256 and 5120/6144 kept)
    d = os.path.join(kd, "dot")
    m = load_manifest(d)
    arrs, cases = {}, []
    for c in m["cases"]:
        if c["width"] > 6144:
            continue
        arrs[c["case"] + "__w_raw"] = raw(d, c["w_raw"])
        arrs[c["case"] + "__x_deq"] = npy(d, c["x_deq"]).astype(np.float32)
        arrs[c["case"] + "__x_raw"] = raw(d, c["x_raw"])
        cases.append(strip(c, {"case", "ggml_type", "ggml_type_id", "width", "n_rows", "rows", "ref_f64", "max_abs_term"}))
    save("dot", arrs, {"source": m["source"], "budget_k": m["budget_k"], "cases": cases})

    # --- matvec: f64 reference per row
    d = os.path.join(kd, "matvec")
    m = load_manifest(d)
    arrs, cases = {}, []
    for c in m["cases"]:
        arrs[c["case"] + "__w_raw"] = raw(d, c["w_raw"])
        arrs[c["case"] + "__x_deq"] = npy(d, c["x_deq"]).astype(np.float32)
        cases.append(strip(c, {"case", "ggml_type", "ggml_type_id", "width", "n_rows", "ref_f64", "max_abs_term"}))
    save("matvec", arrs, {"source": m["source"], "budget_k": m["budget_k"], "cases": cases})

    # --- elementwise groups (HF-derived, budgeted): copied whole
    for g in ("rmsnorm", "softmax", "rope", "act", "deltanet"):
        d = os.path.join(kd, g)
        m = load_manifest(d)
        arrs, cases = {}, []
        for c in m["cases"]:
            cc = {}
            for k, v in c.items():
                if isinstance(v, dict) and "file" in v and v["file"].endswith(".npy"):
                    arrs[c["case"] + "__" + k] = npy(d, v)
                else:
                    cc[k] = v
            cases.append(cc)
        meta = {k: v for k, v in m.items() if k != "cases"}
        meta["cases"] = cases
        save(g, arrs, meta)

    # conv1d: the step cases and the short prefill (the 10240-channel prefill is 0.6 MB and adds nothing)
    d = os.path.join(kd, "conv1d")
    m = load_manifest(d)
    arrs, cases = {}, []
    for c in m["cases"]:
        if c["case"] == "conv_prefill_c10240":
            continue
        cc = {}
        for k, v in c.items():
            if isinstance(v, dict) and "file" in v:
                arrs[c["case"] + "__" + k] = npy(d, v)
            else:
                cc[k] = v
        cases.append(cc)
    meta = {k: v for k, v in m.items() if k != "cases"}
    meta["cases"] = cases
    save("conv1d", arrs, meta)

    # --- dequant: gguf-py output, bit-exact (tests/fixtures/dequant, checked by crates/core/tests/dequant.rs).
    # Prefix and hostile blocks whole; for the full tensors the bytes of the first 4096 values (the head the
    # fixture stores) plus, for the K-quant / Q4_0 tensors, the first 64 rows of real weights, which the GPU
    # GEMV parity tests use as realistic blocks.
    d = os.path.join(fx, "dequant")
    m = load_manifest(d)
    arrs, types = {}, {}
    for name, t in m["types"].items():
        tt = {k: t[k] for k in ("ggml_type", "ggml_type_id", "block_size", "type_size")}
        p = t["prefix"]
        arrs[name + "__prefix_raw"] = np.fromfile(os.path.join(d, p["raw_bin"]), dtype=np.uint8)
        arrs[name + "__prefix"] = np.load(os.path.join(d, p["npy"])).astype(np.float32)
        tt["prefix"] = {k: p[k] for k in ("tensor", "n_blocks", "n_elements")}
        f = t["full"]
        head = np.load(os.path.join(d, f["head_npy"])).astype(np.float32)
        arrs[name + "__full_head"] = head
        tt["full"] = {k: f[k] for k in ("tensor", "shape_numpy", "n_elements", "byte_size", "digest")}
        if f.get("raw_bin") and os.path.exists(os.path.join(d, f["raw_bin"])):
            full = np.fromfile(os.path.join(d, f["raw_bin"]), dtype=np.uint8)
            nhead = head.size // t["block_size"] * t["type_size"]
            arrs[name + "__full_head_raw"] = full[:nhead]
            shape = f["shape_numpy"]
            if len(shape) == 2 and name in ("Q4_K", "Q5_K", "Q6_K", "Q4_0", "Q8_0"):
                row_bytes = shape[1] // t["block_size"] * t["type_size"]
                arrs[name + "__rows64_raw"] = full[: 64 * row_bytes]
                tt["rows64"] = {"rows": 64, "cols": shape[1], "row_bytes": row_bytes}
        types[name] = tt
    hostile = {}
    for k, v in m.items():
        if k.startswith("hostile") or k == "hostile":
            hostile[k] = v
    for fn in sorted(os.listdir(d)):
        if fn.startswith("hostile_") and fn.endswith(".bin"):
            base = fn[:-4]
            arrs[base + "__raw"] = np.fromfile(os.path.join(d, fn), dtype=np.uint8)
            arrs[base + "__deq"] = np.load(os.path.join(d, base + ".npy")).astype(np.float32)
    save("dequant", arrs, {"spec": m["spec"], "types": types, "hostile": hostile})

    # --- layers: HF module outputs on F32 weights (tests/fixtures/layers/layers, checked by
    # crates/core/tests/layers.rs): every case's weights, prefill and step arrays, copied whole
    d = os.path.join(fx, "layers", "layers")
    m = load_manifest(d)
    arrs, cases = {}, []
    for c in m["cases"]:
        cc = {}
        for k, v in c.items():
            if k == "weights":
                cc[k] = {}
                for wn, wf in v.items():
                    arrs[c["case"] + "__w__" + wn] = npy(d, wf).astype(np.float32)
                    cc[k][wn] = {"shape": wf["shape"]}
            elif k in ("prefill", "step"):
                cc[k] = {}
                for fk, fv in v.items():
                    if isinstance(fv, dict) and "file" in fv:
                        arrs[c["case"] + "__" + k + "__" + fk] = npy(d, fv).astype(np.float32)
                        cc[k][fk] = {"shape": fv["shape"]}
                    else:
                        cc[k][fk] = fv
            else:
                cc[k] = v
        cases.append(cc)
    meta = {k: v for k, v in m.items() if k != "cases"}
    meta["cases"] = cases
    save("layers", arrs, meta)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the reference project root>")
    main(sys.argv[1])
