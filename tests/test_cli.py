"""`qdec run` (qwen-3.8-in-rust_b200/csrc/cli_run.cpp, the reference's `aqueduct run`, crates/cli/src/run.rs):
argument handling on the CPU, and on a GPU the ids it prints against the oracle's on the tiny checkpoint, plain
and --spec 3, with the --stats JSON."""
import json
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "qwen-3.8-in-rust_b200", "qdec")
SEED = 20261201


def run(args, timeout=300):
    return subprocess.run([CLI] + args, capture_output=True, text=True, timeout=timeout)


def test_cli_rejects_bad_arguments():
    if not os.path.exists(CLI):
        pytest.skip("the CLI is not built")
    r = run([])
    assert r.returncode == 2 and "usage" in r.stderr
    r = run(["run", "--ids", "1,2"])
    assert r.returncode == 2 and "--model is required" in r.stderr
    r = run(["run", "--model", "x.gguf"])
    assert r.returncode == 2 and "--ids is required" in r.stderr
    r = run(["run", "--model", "x.gguf", "--ids", "1,a"])
    assert r.returncode == 2 and "bad id" in r.stderr
    r = run(["run", "--model", "x.gguf", "--ids", "1", "--mode", "ring"])
    assert r.returncode == 2
    r = run(["run", "--model", "x.gguf", "--ids", "1", "--frobnicate"])
    assert r.returncode == 2 and "unknown argument" in r.stderr


@pytest.mark.gpu
def test_cli_ids_match_oracle(tmp_path, orc):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qdec

    path = tmp_path / "tiny.gguf"
    qdec.synth_gguf(path, "tiny", SEED)
    prompt = [int(v) for v in np.random.default_rng(SEED + 1).integers(0, 4096, 16)]
    om = orc.OracleModel(path)
    want = om.state(512).generate(prompt, 24, stop=False)
    ids = ",".join(map(str, prompt))
    r = run(["run", "--model", str(path), "--ids", ids, "--max-tokens", "24", "--ids-only"])
    assert r.returncode == 0, r.stderr
    got = [int(v) for v in r.stdout.strip().split(",")]
    # the CLI stops at a stop id like the reference's loop; the oracle ran without stopping
    assert got == want[: len(got)] and len(got) >= 1
    stats = tmp_path / "stats.json"
    r = run(["run", "--model", str(path), "--ids", ids, "--max-tokens", "24", "--spec", "3", "--stats", str(stats)])
    assert r.returncode == 0, r.stderr
    line = [l for l in r.stdout.splitlines() if l.startswith("generated ids:")][0]
    got_s = [int(v) for v in line.split(":")[1].strip().split(",")]
    assert got_s == got
    js = json.loads(stats.read_text())
    assert js["ids"] == got_s and js["spec_k"] == 3 and js["spec_rounds"] >= 1 and js["prompt_len"] == 16
    want_s, st, _ = om.state(512).spec_generate(prompt, len(got_s), 3, stop=False)
    assert want_s == got_s
    assert "s/round" in r.stderr and "spec:" in r.stderr
