"""Tensor parallelism over the GPUs of one node (one process per GPU, torchrun): greedy ids identical to one GPU's,
plain and --spec 3 (free-running and with forced drafts, every draft accepted).  Every matrix is split by output
rows and the sharded activations are all-gathered, so each row is computed whole and the ids are bit-identical
by construction; these tests check it end to end.  Skipped with fewer GPUs than ranks."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TP = os.path.join(ROOT, "qwen-3.8-in-rust_b200", "tp.py")
SEED = 20261201


def need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_tp(world, path, ids, tokens, tmp_path, spec=0, forced=None, max_pos=512):
    out = tmp_path / f"tp{world}_{spec}_{'f' if forced else 'x'}.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}", "--master-addr",
           "127.0.0.1", f"--master-port={free_port()}", TP, "--model", str(path), "--ids", ",".join(map(str, ids)),
           "--tokens", str(tokens), "--spec", str(spec), "--max-pos", str(max_pos), "--out", str(out)]
    if forced:
        cmd += ["--forced", ",".join(map(str, forced))]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "900"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    with open(out) as f:
        res = json.load(f)
    assert res["world"] == world and res["ranks_agree"]
    return res


def one_gpu(path, ids, tokens, spec=0, forced=None, max_pos=512):
    import qdec
    from tp import spec_generate

    m = qdec.Model(path, device=0, max_pos=max_pos)
    st = m.new_state(spec_k=spec, max_rows=32)
    got = spec_generate(st, ids, tokens, forced) if spec else qdec.generate(st, ids, tokens, stop=False)
    st.free()
    m.close()
    return got


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    need(2)
    import qdec

    path = tmp_path_factory.mktemp("tp_tiny") / "tiny.gguf"
    qdec.synth_gguf(path, "tiny", SEED)
    return path


def prompt(vocab, n=16):
    return [int(v) for v in np.random.default_rng(SEED + 1).integers(0, vocab, n)]


def test_tp2_tiny_plain_ids_match_one_gpu(tiny, tmp_path):
    p = prompt(4096)
    want = one_gpu(tiny, p, 32)
    assert run_tp(2, tiny, p, 32, tmp_path)["ids"] == want


def test_tp2_tiny_spec3_ids_match_one_gpu_and_plain(tiny, tmp_path):
    p = prompt(4096)
    plain = one_gpu(tiny, p, 32)
    want = one_gpu(tiny, p, 32, spec=3)
    assert want == plain
    assert run_tp(2, tiny, p, 32, tmp_path, spec=3)["ids"] == want


def test_tp2_tiny_forced_drafts_accept_every_draft(tiny, tmp_path):
    """Drafts forced to the plain run's next ids: every round accepts k = 3 drafts (the m = k regime)."""
    p = prompt(4096)
    plain = one_gpu(tiny, p, 64)
    res = run_tp(2, tiny, p, 41, tmp_path, spec=3, forced=plain)
    assert res["ids"] == plain[:41]
    c = res["counters"]
    assert c["accepted"] == 3 * c["rounds"]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_27b_dims_ids_match_one_gpu(world, tmp_path_factory, tmp_path):
    """The 27B dimensions (16 K heads / 48 V heads, 24 q / 4 kv heads, FFN 17408 split on 256-row blocks, vocab
    248320) with 4 layers: plain and --spec 3 ids over 2, 4 and 8 ranks equal one GPU's."""
    need(world)
    import qdec

    path = tmp_path_factory.getbasetemp() / "tp_27b_L4.gguf"
    if not path.exists():
        qdec.synth_gguf(path, "27b-L4", SEED)
    p = prompt(248044, 12)
    want_plain = one_gpu(path, p, 8)
    want_spec = one_gpu(path, p, 12, spec=3)
    assert want_spec[:8] == want_plain
    assert run_tp(world, path, p, 8, tmp_path)["ids"] == want_plain
    assert run_tp(world, path, p, 12, tmp_path, spec=3)["ids"] == want_spec
