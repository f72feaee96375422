"""Tensor-parallel greedy decode over the GPUs of one node: one process per GPU, launched by torchrun.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 --master-port P \\
        qwen-3.8-in-rust_b200/tp.py --model M.gguf --ids 1,2,3 --tokens 32 [--spec 3] [--out ids.json]

Each rank opens its shard of the model (qdec.Model(..., tp=(rank, world))), the ranks exchange the handles of
their exchange blocks over the process group (gloo: only the 80-byte handles travel through it; the activations
move GPU to GPU), and every rank runs the same decode calls.  The ids are the same on every rank and the same as
one GPU's; rank 0 prints them (and writes them to --out).  This is the CLI's `run` (crates/cli/src/run.rs:272-383)
with --gpus N --mode tp.
"""
import argparse
import datetime
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

import qdec  # noqa: E402


def setup(backend="gloo", timeout_s=120):
    """(rank, world, local_rank) from the torchrun environment, with the process group initialised."""
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return rank, world, local


def open_state(path, rank, world, device, spec_k=0, max_pos=4096, max_rows=32):
    """This rank's model shard and a connected decode state."""
    model = qdec.Model(path, device=device, max_pos=max_pos, tp=(rank, world) if world > 1 else None)
    st = model.new_state(spec_k=spec_k, max_rows=max_rows)
    if world > 1:
        st.tp_connect_group()
    return model, st


def spec_generate(st, prompt, n_tokens, forced=None):
    """The greedy --spec k loop (run.rs:352-383): spec_prefill, then rounds until n_tokens ids; with `forced`
    (a reference id sequence whose first id is the prefill's) each round's drafts are forced to its next ids."""
    x = st.spec_prefill(prompt)
    out = [x]
    while len(out) < n_tokens:
        if forced is not None:
            st.set_drafts(forced[len(out):len(out) + st.k])
        em = st.spec_round(x)
        out.extend(em)
        x = em[-1]
    return out[:n_tokens]


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", required=True)
    ap.add_argument("--ids", required=True, help="comma-separated prompt ids")
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--spec", type=int, default=0, help="draft k tokens per round with the MTP head (0: plain)")
    ap.add_argument("--forced", default=None, help="comma-separated ids whose next tokens are forced as drafts")
    ap.add_argument("--max-pos", type=int, default=1024)
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    import torch
    import torch.distributed as dist

    rank, world, local = setup("gloo")
    torch.cuda.set_device(local)
    prompt = [int(v) for v in a.ids.split(",")]
    model, st = open_state(a.model, rank, world, local, spec_k=a.spec, max_pos=a.max_pos)
    if a.spec > 0:
        forced = [int(v) for v in a.forced.split(",")] if a.forced else None
        ids = spec_generate(st, prompt, a.tokens, forced)
        counters = st.counters()
    else:
        ids = qdec.generate(st, prompt, a.tokens, stop=False)
        counters = None
    if world > 1:
        every = [None] * world
        dist.all_gather_object(every, ids)
        same = all(e == ids for e in every)
        dist.barrier()  # every rank's last exchange is done before any rank frees its state
    else:
        same = True
    st.free()
    model.close()
    if rank == 0:
        res = {"ids": ids, "world": world, "ranks_agree": same, "counters": counters}
        print(json.dumps(res), flush=True)
        if a.out:
            with open(a.out, "w") as f:
                json.dump(res, f)
    if world > 1:
        dist.destroy_process_group()
    return 0 if same else 1


if __name__ == "__main__":
    sys.exit(main())
