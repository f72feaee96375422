"""Benchmark of the qdec hot path on B200 (one process per GPU; torchrun for N > 1).

Default workload (`--workload spec`): `--spec 3` decoding of the 27B architecture (64 layers: 48 Gated DeltaNet
+ 16 gated GQA, hidden 5120, FFN 17408, vocabulary 248320, the MTP block) with synthetic Q4_K_M weights (seeded,
the reference's type recipe), after a 128-token prompt prefilled as one batch.  One step = one speculative round
(k = 3 MTP drafts, one verify pass over 4 rows, rollback, the MTP re-feed) replayed as one CUDA graph.  Metric:
accepted tokens / second, whole job over all ranks (replicas, or one tensor-parallel model with --gpus N).  The
JSON line also carries the plain-decode rate, the multi-sequence batched decode rate (2, 4 and 8 sequences per
step through qdec_batch_step), the prefill rate, the K-quant GEMV table of the config-2 shapes
(Q4_K / Q5_K / Q6_K / Q8_0 / Q4_0 at N = 1, 2, 4), an 8K-position KV run, the roofline of the dominant GEMV,
parity against the CPU oracle and the CPU baseline (the AVX2 C restatement of the reference's decode on all host
cores, on the same 128-token prompt).

`--workload gemv`: the isolated K-quant GEMV microbench -- Q4_K W_up 17408 x 5120 and W_down 5120 x 17408 times
N = 1, 2, 4 quantised columns, three rotating weight sets (301 MB) so no step finds its weights in the 126 MB L2;
metric weight bytes streamed / second (crates/cli/src/bench.rs:65-91).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl qdec|reference] [--workload spec|gemv]

`--impl reference` times the reference's CPU path (its C restatement in oracle/, all host threads) on a bounded
sample of the same workload, without loading the product library.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen-3.8-in-rust_b200"))

UP = (17408, 5120)
DOWN = (5120, 17408)
NS = (1, 2, 4)
Q4K_BB = 144
N_SETS = 3


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def synth_q4k(rows, cols, seed):
    """Seeded Q4_K blocks with finite scales: d ~ U(1e-3, 4e-3), dmin ~ U(0, 1e-3), 6-bit scales/mins, 4-bit codes."""
    rng = np.random.default_rng(seed)
    nb = rows * (cols // 256)
    blk = np.empty((nb, Q4K_BB), np.uint8)
    d = rng.uniform(1e-3, 4e-3, nb).astype(np.float16).view(np.uint16)
    dm = rng.uniform(0.0, 1e-3, nb).astype(np.float16).view(np.uint16)
    blk[:, 0], blk[:, 1] = d & 0xFF, d >> 8
    blk[:, 2], blk[:, 3] = dm & 0xFF, dm >> 8
    sc = rng.integers(0, 64, (nb, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, (nb, 8), dtype=np.uint8)
    q = np.zeros((nb, 12), np.uint8)  # pack as ggml's quantize_row_q4_K_ref does (inverse of get_scale_min_k4)
    for j in range(8):
        if j < 4:
            q[:, j] = sc[:, j]
            q[:, j + 4] = mn[:, j]
        else:
            q[:, j + 4] = (sc[:, j] & 0xF) | ((mn[:, j] & 0xF) << 4)
            q[:, j - 4] |= (sc[:, j] >> 4) << 6
            q[:, j] |= (mn[:, j] >> 4) << 6
    blk[:, 4:16] = q
    blk[:, 16:] = rng.integers(0, 256, (nb, 128), dtype=np.uint8)
    return blk.reshape(-1)


def algorithmic_bytes(rows, cols, n):
    """Weights + Q8_K activations + f32 outputs of one GEMV launch."""
    return rows * (cols // 256) * Q4K_BB + n * (cols // 256) * 292 + 4 * n * rows


class ClockSampler:
    """NVML samples of SM clock and throttle reasons while the timed region runs (nvidia-smi's data)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join()
            if not self.samples:  # region shorter than one sample period: take one now
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup(backend):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        import torch

        torch.cuda.set_device(local)  # before the process group, so NCCL binds this rank's GPU
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def max_over_ranks(values, device):
    """The element-wise maximum over the ranks of a list of floats (the slowest rank's times); one rank: as is."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def oracle_spec_sample(path, k, prompt_len, rounds):
    """The reference's greedy --spec k loop on the host cores: the oracle (oracle/model.c) with its AVX2 kernels
    (bit-identical to the scalar restatement) and the reference's batching -- the prompt in 16-row chunks and the
    k + 1 verify rows through one blocked pass over the weights (matmul_t), the rollback by replaying the kept
    rows' recurrence -- OpenMP over all host threads.  The given prompt length, then `rounds` rounds; returns
    (tok/s over the rounds, s/round, stats with the prompt and ids, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    oracle.build()
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    om = oracle.OracleModel(path)
    st = om.state(max_pos=prompt_len + (k + 1) * (rounds + 2) + 8)
    prompt = spec_prompt(om.vocab, SPEC_SEED + 1)[:prompt_len]
    t0 = time.perf_counter()
    ids, stats, _ = st.spec_generate(prompt, 1 + rounds, k, stop=False)
    total = time.perf_counter() - t0
    secs = stats["round_seconds"]
    emitted = len(ids) - 1
    om.close()
    stats["prompt"], stats["ids"] = prompt, ids
    stats["prefill_seconds"] = total - secs
    return emitted / secs, secs / max(1, stats["rounds"]), stats, cores


CPU_KIND = "port"
CPU_VARIANT = ("the oracle's AVX2 kernels (bit-identical to its scalar restatement of kdot.rs), blocked over the verify "
               "rows like matmul_t, batched prefill, replay rollback; OpenMP over every host thread")


def gpu_spec_ids(model, k, prompt, n_ids):
    """The GPU's --spec k ids for `prompt` (spec_prefill, then rounds until n_ids ids): the ids the parity object
    compares with the CPU leg's."""
    import qdec

    st = model.new_state(spec_k=k, max_rows=32)
    ids = qdec.generate_spec(st, prompt, n_ids, stop=False)
    st.free()
    return ids


def run_reference_spec(args, world, rank):
    if rank != 0:
        return
    # the checkpoint is written by a child process, so this arm maps none of the product's libraries
    path = checkpoint_path(args.preset, SPEC_SEED)
    if not os.path.exists(path):
        import subprocess

        subprocess.run([sys.executable, "-c", "import sys; sys.path.insert(0, sys.argv[1]); import bench; "
                        "bench.ensure_checkpoint(sys.argv[2], int(sys.argv[3]))", ROOT, args.preset, str(SPEC_SEED)],
                       check=True, cwd=ROOT)
    k = SPEC_K
    # the same workload as the GPU arm -- the 128-token prompt, then --spec 3 rounds -- with a bounded number of
    # timed rounds (each a whole pass over the 17.8 GB of weights on the host cores)
    rounds = max(2, min(args.steps, 6))
    tok_s, s_round, stats, cores = oracle_spec_sample(path, k, PROMPT_LEN, rounds)
    sample = (f"{stats['rounds']} --spec {k} rounds after the {PROMPT_LEN}-token prompt on the {args.preset} checkpoint "
              f"(of {args.steps} requested steps; {s_round:.2f} s/round; prompt prefill {stats['prefill_seconds']:.1f} s)")
    line = {
        "metric": "decode tok/s (greedy, --spec 3) Qwen3.8-27B Q4_K_M", "value": round(tok_s, 5), "unit": "tok/s",
        "n_gpus": world, "steps": stats["rounds"], "warmup": 0, "ms_per_step": round(s_round * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "Q4_K_M weights x Q8_K activations, f32", "data": "synthetic",
        "config": {"workload": f"{args.preset} --spec 3, {PROMPT_LEN}-token prompt", "prompt": PROMPT_LEN, "k": k},
        "impl": "reference",
        "cpu_baseline": {"value": round(tok_s, 5), "unit": "tok/s", "cores": cores, "kind": CPU_KIND,
                         "variant": CPU_VARIANT, "sample": sample},
        "e2e": {"value": round(tok_s, 5), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference(args, world, rank):
    """The reference's CPU path (oracle restatement, all host threads) on a bounded row sample per step."""
    if rank != 0:
        return
    if args.workload == "spec":
        run_reference_spec(args, world, rank)
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    oracle.build()
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    # per step: the same 6 passes on a sample of rows, sized so the whole run stays within ~90 s of CPU time
    frac_rows = {}
    w = {}
    for name, (rows, cols) in (("up", UP), ("down", DOWN)):
        w[name] = synth_q4k(rows, cols, seed=1 + (name == "down"))
    x = {n: np.random.default_rng(n).standard_normal((n, UP[1])).astype(np.float32) for n in NS}
    xd = {n: np.random.default_rng(10 + n).standard_normal((n, DOWN[1])).astype(np.float32) for n in NS}

    def step(sample_rows):
        done = 0
        for n in NS:
            for name, (rows, cols), xx in (("up", UP, x[n]), ("down", DOWN, xd[n])):
                r = sample_rows[name]
                oracle.matmul(oracle.Q4_K, w[name][: r * (cols // 256) * Q4K_BB], r, cols, xx)
                done += r * (cols // 256) * Q4K_BB
        return done

    # calibrate on a small sample
    probe = {"up": 256, "down": 128}
    t0 = time.perf_counter()
    b = step(probe)
    dt = max(time.perf_counter() - t0, 1e-6)
    rate = b / dt
    budget_s = 60.0
    per_step_bytes = min(rate * budget_s / max(1, args.steps + args.warmup), float(sum(r * (c // 256) * Q4K_BB for r, c in (UP, DOWN)) * len(NS)))
    scale = per_step_bytes / (sum(r * (c // 256) * Q4K_BB for r, c in (UP, DOWN)) * len(NS))
    sample = {"up": max(8, int(UP[0] * scale) // 8 * 8), "down": max(8, int(DOWN[0] * scale) // 8 * 8)}
    for _ in range(args.warmup):
        step(sample)
    t0 = time.perf_counter()
    total = 0
    for _ in range(args.steps):
        total += step(sample)
    el = time.perf_counter() - t0
    gbs = total / el / 1e9
    sample_desc = f"{sample['up']} of {UP[0]} rows of W_up and {sample['down']} of {DOWN[0]} rows of W_down per step, N in {list(NS)}"
    line = {
        "metric": "Q4_K GEMV weight GB/s (config 2: 17408x5120 + 5120x17408, N=1,2,4)", "value": round(gbs, 3),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8 (Q4_K) x i8 (Q8_K), f32 accumulate", "data": "synthetic",
        "config": {"workload": "q4k_gemv_config2", "shapes": [list(UP), list(DOWN)], "n_cols": list(NS)},
        "impl": "reference",
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample_desc},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample():
    """The oracle (the reference's CPU arithmetic restated in C, OpenMP over the host cores) on a bounded
    sample: the 6 passes of one step over the first 2048 / 512 rows, repeated for ~10 s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    oracle.build()
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    rows_up, rows_down = 2048, 512
    wu = synth_q4k(rows_up, UP[1], seed=11)
    wd = synth_q4k(rows_down, DOWN[1], seed=12)
    xs = {n: (np.random.default_rng(n).standard_normal((n, UP[1])).astype(np.float32),
              np.random.default_rng(n + 7).standard_normal((n, DOWN[1])).astype(np.float32)) for n in NS}
    t0 = time.perf_counter()
    total, reps = 0, 0
    while time.perf_counter() - t0 < 10.0 or reps == 0:
        for n in NS:
            oracle.matmul(oracle.Q4_K, wu, rows_up, UP[1], xs[n][0])
            oracle.matmul(oracle.Q4_K, wd, rows_down, DOWN[1], xs[n][1])
            total += rows_up * (UP[1] // 256) * Q4K_BB + rows_down * (DOWN[1] // 256) * Q4K_BB
        reps += 1
    el = time.perf_counter() - t0
    return {"value": round(total / el / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{reps} x (6 passes: {rows_up} rows of W_up, {rows_down} rows of W_down, N=1,2,4), {el:.1f} s"}


def run_qdec(args, world, rank, local):
    import torch

    import qdec

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    L = qdec.lib()
    # weights: N_SETS rotating sets (more bytes than L2)
    sets = []
    for s in range(N_SETS):
        wu = torch.from_numpy(synth_q4k(*UP, seed=100 * (rank + 1) + 2 * s)).to(dev)
        wdn = torch.from_numpy(synth_q4k(*DOWN, seed=100 * (rank + 1) + 2 * s + 1)).to(dev)
        sets.append((wu, wdn))
    x_up = {n: torch.randn(n, UP[1], generator=torch.Generator().manual_seed(n), dtype=torch.float32).to(dev) for n in NS}
    x_dn = {n: torch.randn(n, DOWN[1], generator=torch.Generator().manual_seed(10 + n), dtype=torch.float32).to(dev) for n in NS}
    a_up = torch.empty(4 * qdec.act_row_bytes(qdec.Q4_K, UP[1]), dtype=torch.uint8, device=dev)
    a_dn = torch.empty(4 * qdec.act_row_bytes(qdec.Q4_K, DOWN[1]), dtype=torch.uint8, device=dev)
    y_up = torch.empty(4 * UP[0], dtype=torch.float32, device=dev)
    y_dn = torch.empty(4 * DOWN[0], dtype=torch.float32, device=dev)
    launches_per_step = 4 * len(NS)
    ev_pairs = []

    def step(i, record=False):
        wu, wdn = sets[i % N_SETS]
        for n in NS:
            qdec.quantize_q8k(x_up[n].data_ptr(), UP[1], n, a_up.data_ptr(), sp)
            if record and n == 4:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            qdec.gemv(qdec.Q4_K, wu.data_ptr(), UP[0], UP[1], a_up.data_ptr(), n, y_up.data_ptr(), sp)
            if record and n == 4:
                e1.record(stream)
                ev_pairs.append((e0, e1))
            qdec.quantize_q8k(x_dn[n].data_ptr(), DOWN[1], n, a_dn.data_ptr(), sp)
            qdec.gemv(qdec.Q4_K, wdn.data_ptr(), DOWN[0], DOWN[1], a_dn.data_ptr(), n, y_dn.data_ptr(), sp)

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            step(i)
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    barrier()
    torch.cuda.synchronize()
    # the dominant kernel timed alone per launch (N = 4 on W_up), on the launching stream
    for i in range(min(args.steps, 200)):
        step(i, record=True)
    torch.cuda.synchronize()
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in ev_pairs)
    # end to end through the C ABI from pinned host buffers: H2D of x, qdec_matvec, D2H of y, every step
    hx_up = {n: x_up[n].cpu().pin_memory() for n in NS}
    hx_dn = {n: x_dn[n].cpu().pin_memory() for n in NS}
    hy_up = torch.empty(4 * UP[0], dtype=torch.float32).pin_memory()
    hy_dn = torch.empty(4 * DOWN[0], dtype=torch.float32).pin_memory()
    dx_up = torch.empty(4 * UP[1], dtype=torch.float32, device=dev)
    dx_dn = torch.empty(4 * DOWN[1], dtype=torch.float32, device=dev)
    h2d = sum(4 * n * (UP[1] + DOWN[1]) for n in NS)
    d2h = sum(4 * n * (UP[0] + DOWN[0]) for n in NS)

    def e2e_step(i):
        wu, wdn = sets[i % N_SETS]
        for n in NS:
            dx_up[: n * UP[1]].copy_(hx_up[n].view(-1), non_blocking=True)
            qdec.matvec(qdec.Q4_K, wu.data_ptr(), UP[0], UP[1], dx_up.data_ptr(), n, y_up.data_ptr(), sp)
            hy_up[: n * UP[0]].copy_(y_up[: n * UP[0]], non_blocking=True)
            dx_dn[: n * DOWN[1]].copy_(hx_dn[n].view(-1), non_blocking=True)
            qdec.matvec(qdec.Q4_K, wdn.data_ptr(), DOWN[0], DOWN[1], dx_dn.data_ptr(), n, y_dn.data_ptr(), sp)
            hy_dn[: n * DOWN[0]].copy_(y_dn[: n * DOWN[0]], non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end)

    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms, e2e_ms, kern_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, kern_ms = t.tolist()
    bytes_per_step = sum(r * (c // 256) * Q4K_BB for r, c in (UP, DOWN)) * len(NS)
    value = world * bytes_per_step * args.steps / (ms / 1e3) / 1e9
    e2e_value = world * bytes_per_step * args.steps / (e2e_ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    alg = algorithmic_bytes(UP[0], UP[1], 4)
    achieved = alg / (kern_ms / 1e3) / 1e9
    if rank == 0:
        traffic = None
        tp = os.path.join(ROOT, "profiles", "q4k_gemv_traffic.json")
        if os.path.exists(tp):
            with open(tp) as f:
                traffic = json.load(f).get("dram_bytes_per_launch")
        line = {
            "metric": "Q4_K GEMV weight GB/s (config 2: 17408x5120 + 5120x17408, N=1,2,4)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8 (Q4_K) x i8 (Q8_K), f32 accumulate", "data": "synthetic",
            "config": {"workload": "q4k_gemv_config2", "shapes": [list(UP), list(DOWN)], "n_cols": list(NS),
                       "l2": f"{N_SETS} rotating weight sets ({N_SETS * bytes_per_step // len(NS) / 1e6:.0f} MB) > 126 MB L2",
                       "parallelism": f"replicas x{world}"},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "kernel": "kq_gemv_kernel<Q4_K, N=4> 17408x5120", "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "alg_bytes_per_launch": alg, "launch_us": round(kern_ms * 1e3, 3)},
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------------
# The --spec 3 decode workload: the full 27B architecture, synthetic Q4_K_M weights, a 128-token prompt.

SPEC_K = 3
PROMPT_LEN = 128
SPEC_SEED = 20261201


def checkpoint_path(preset, seed):
    d = os.environ.get("QDEC_BENCH_DIR") or ("/dev/shm" if os.path.isdir("/dev/shm") else "/tmp")
    return os.path.join(d, f"qdec_{preset}_{seed}.gguf")


def ensure_checkpoint(preset, seed):
    import qdec

    path = checkpoint_path(preset, seed)
    if not os.path.exists(path):
        tmp = path + f".part{os.getpid()}"
        qdec.synth_gguf(tmp, preset, seed)
        os.replace(tmp, path)
    return path


def spec_prompt(vocab, seed):
    return [int(v) for v in np.random.default_rng(seed).integers(0, min(vocab, 248044), PROMPT_LEN)]


def dominant_gemv_timing(dev, launches=200, n=4):
    """The verify's dominant kernel timed alone on the launching stream with CUDA events: the fused Q4_K GEMV of
    ffn_gate and ffn_up (two 17408 x 5120 tile matrices against the same N = 4 image columns, one launch, as the
    layer runs it), weight pairs rotating over 3 sets (300 MB > L2).  With n >= 16 columns the same call runs the
    prefill's tensor-core GEMM."""
    import torch

    import qdec

    rows, cols = UP[0], UP[1]
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    sets = []
    for s in range(N_SETS):
        pair = []
        for m in range(2):
            src = torch.from_numpy(synth_q4k(rows, cols, seed=500 + 2 * s + m)).to(dev)
            dst = torch.empty_like(src)
            qdec.repack_tiles(qdec.Q4_K, src.data_ptr(), rows, cols, dst.data_ptr(), sp)
            pair.append(dst)
        sets.append(pair)
    x = torch.randn(n, cols, generator=torch.Generator().manual_seed(7), dtype=torch.float32).to(dev)
    t = qdec.TILE[qdec.Q4_K]
    img = torch.empty(n * qdec.image_row_bytes(t, cols), dtype=torch.uint8, device=dev)
    y1 = torch.empty(n * rows, dtype=torch.float32, device=dev)
    y2 = torch.empty(n * rows, dtype=torch.float32, device=dev)
    qdec.quantize_image(t, x.data_ptr(), cols, n, img.data_ptr(), sp)

    def launch(i):
        w1, w2 = sets[i % N_SETS]
        qdec.gemv_image_pair(t, w1.data_ptr(), w2.data_ptr(), rows, cols, img.data_ptr(), n, y1.data_ptr(), y2.data_ptr(), sp)

    for i in range(min(10, launches)):
        launch(i)
    torch.cuda.synchronize()
    # back-to-back launches between two events on the launching stream (the weight sets rotate, 300 MB > L2):
    # the average launch duration, without per-launch event records in between; median of 5 batches
    batch = max(1, launches // 5)
    per = []
    for b in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(batch):
            launch(i)
        e1.record(stream)
        torch.cuda.synchronize()
        per.append(e0.elapsed_time(e1) / batch)
    ms = statistics.median(per)
    # algorithmic bytes of one launch: both weight matrices once, the image columns once, both outputs
    alg = 2 * rows * (cols // 256) * Q4K_BB + n * (cols // 256) * 320 + 2 * 4 * n * rows
    del sets
    return alg, ms


BLOCK = {12: (256, 144), 13: (256, 176), 14: (256, 210), 8: (32, 34), 2: (32, 18)}


def synth_blocks(t, rows, cols, seed):
    """Seeded random blocks of ggml type t whose f16 scales are finite (magnitudes 2^-3 .. 2^3): the config-2
    weights for the types other than Q4_K."""
    be, bb = BLOCK[t]
    rng = np.random.default_rng(seed)
    data = rng.integers(0, 256, size=(rows * (cols // be), bb), dtype=np.uint8)
    for off in ((0, 2) if t in (12, 13) else (208,) if t == 14 else (0,)):
        bits = data[:, off].astype(np.uint16) | (data[:, off + 1].astype(np.uint16) << 8)
        fixed = (bits & 0x83FF) | ((12 + (bits >> 10) % 7) << 10)
        data[:, off], data[:, off + 1] = (fixed & 0xFF).astype(np.uint8), (fixed >> 8).astype(np.uint8)
    return data.reshape(-1)


def gemv_table(dev):
    """Config 2: every weight type of the model (tile layout) on W_up 17408 x 5120 and W_down 5120 x 17408 at N = 1,
    2, 4 columns: CUDA-event time of back-to-back launches over rotating weight sets (> L2), the weight GB/s of the
    reference bench (crates/cli/src/bench.rs:65-91: rows * row bytes / s) and the algorithmic GB/s (weights +
    activation image + outputs)."""
    import torch

    import qdec

    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    out = {}
    names = {12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 8: "Q8_0", 2: "Q4_0"}
    for t in (12, 13, 14, 8, 2):
        for rows, cols in (UP, DOWN):
            be, bb = BLOCK[t]
            wbytes = rows * (cols // be) * bb
            sets = []
            for s in range(N_SETS):
                src = torch.from_numpy(synth_q4k(rows, cols, 300 + s) if t == 12 else synth_blocks(t, rows, cols, 300 + s)).to(dev)
                dst = torch.empty_like(src)
                qdec.repack_tiles(t, src.data_ptr(), rows, cols, dst.data_ptr(), sp)
                del src
                sets.append(dst)
            tt = qdec.TILE[t]
            x = torch.randn(4, cols, generator=torch.Generator().manual_seed(t), dtype=torch.float32).to(dev)
            img = torch.empty(4 * qdec.image_row_bytes(tt, cols), dtype=torch.uint8, device=dev)
            qdec.quantize_image(tt, x.data_ptr(), cols, 4, img.data_ptr(), sp)
            y = torch.empty(4 * rows, dtype=torch.float32, device=dev)
            for n in NS:
                for i in range(6):
                    qdec.gemv_image(tt, sets[i % N_SETS].data_ptr(), rows, cols, img.data_ptr(), n, y.data_ptr(), sp)
                per = []
                for b in range(5):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for i in range(12):
                        qdec.gemv_image(tt, sets[i % N_SETS].data_ptr(), rows, cols, img.data_ptr(), n, y.data_ptr(), sp)
                    e1.record(stream)
                    torch.cuda.synchronize()
                    per.append(e0.elapsed_time(e1) / 12)
                us = statistics.median(per) * 1e3
                img_b = n * qdec.image_row_bytes(tt, cols)
                out[f"{names[t]} {rows}x{cols} N={n}"] = {"us": round(us, 2), "weight_gb_s": round(wbytes / us / 1e3, 1),
                                                         "alg_gb_s": round((wbytes + img_b + 4 * n * rows) / us / 1e3, 1)}
            del sets
            torch.cuda.empty_cache()
    return out


def plain_decode_timing(model, prompt, steps):
    """Config 3: plain greedy decode (run.rs:329-350) after the prompt, `steps` tokens, CUDA-event time on the
    state's stream; tokens/s and the weight bytes one token streams (model.rs:274) per second."""
    import torch

    st = model.new_state(spec_k=0, max_rows=32)
    stream = torch.cuda.ExternalStream(st.stream)
    x = st.prefill(prompt)
    for _ in range(3):
        x = st.step(x)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        x = st.step(x)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    st.free()
    s_tok = ms / 1e3 / steps
    return {"tokens": steps, "tok_s": round(1.0 / s_tok, 2), "s_per_token": round(s_tok, 6),
            "weight_gb_s": round(model.info.decode_bytes / s_tok / 1e9, 1)}


def batch_decode_timing(model, prompt, steps, sizes=(2, 4, 8)):
    """Multi-sequence batching (qdec_batch_step): B sequences decoded together, one greedy token each per step,
    every weight read once per step for the B rows; aggregate tokens/s from CUDA events on the batch's stream
    (the first state's).  Each sequence starts from its own prompt (the headline prompt rotated)."""
    import torch

    import qdec

    res = {}
    for b in sizes:
        sts = [model.new_state(spec_k=0, max_rows=max(b, 4)) for _ in range(b)]
        xs = [st.prefill(prompt[i:] + prompt[:i]) for i, st in enumerate(sts)]
        stream = torch.cuda.ExternalStream(sts[0].stream)
        for _ in range(3):
            xs = qdec.batch_step(sts, xs)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            xs = qdec.batch_step(sts, xs)
        e1.record(stream)
        torch.cuda.synchronize()
        s_step = e0.elapsed_time(e1) / 1e3 / steps
        for st in sts:
            st.free()
        res[str(b)] = {"tok_s": round(b / s_step, 2), "s_per_step": round(s_step, 6)}
    return {"sequences": res, "api": "qdec_batch_step (greedy, one token per sequence per step)"}


def long_kv_timing(path, dev_index, k, rounds, prompt_len=8064):
    """Config 5 on one GPU: the KV cache grown to ~8.2K positions (an 8064-token prompt prefilled on the device),
    then --spec 3 rounds; s/round from CUDA events."""
    import torch

    import qdec

    max_pos = prompt_len + (rounds + 8) * (k + 1) * 2 + 64
    m = qdec.Model(path, device=dev_index, max_pos=max_pos)
    prompt = [int(v) for v in np.random.default_rng(SPEC_SEED + 9).integers(0, min(m.info.vocab, 248044), prompt_len)]
    st = m.new_state(spec_k=k, max_rows=128)
    stream = torch.cuda.ExternalStream(st.stream)
    t0 = time.perf_counter()
    x = st.spec_prefill(prompt)
    prefill_s = time.perf_counter() - t0
    for _ in range(3):
        x = st.spec_round(x)[-1]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    emitted = 0
    for _ in range(rounds):
        em = st.spec_round(x)
        emitted += len(em)
        x = em[-1]
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    pos = st.pos
    st.free()
    m.close()
    return {"kv_positions": pos, "rounds": rounds, "s_per_round": round(ms / 1e3 / rounds, 6),
            "tok_s": round(emitted / (ms / 1e3), 2), "prompt_prefill_s": round(prefill_s, 2)}


def tp_spec_timing(path, args, world, rank, local, k, prompt, max_pos):
    """--spec k rounds of ONE sequence tensor-parallel over the `world` ranks (every rank runs the same rounds on its
    shard; the sharded activations are exchanged GPU to GPU): device time of the timed rounds on each rank's
    stream, max over ranks, and the host wall time of the same calls (the C ABI per round: x_p in, ids out)."""
    import torch
    import torch.distributed as dist

    import qdec

    t_load = time.perf_counter()
    model = qdec.Model(path, device=local, max_pos=max_pos, tp=(rank, world))  # each rank reads its shard rows
    load_s = time.perf_counter() - t_load
    st = model.new_state(spec_k=k, max_rows=32)
    st.tp_connect_group()
    stream = torch.cuda.ExternalStream(st.stream)
    x = st.spec_prefill(prompt)
    for _ in range(args.warmup):
        x = st.spec_round(x)[-1]
    torch.cuda.synchronize()
    dist.barrier()
    l0 = st.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    emitted = 0
    t0 = time.perf_counter()
    e0.record(stream)
    for _ in range(args.steps):
        em = st.spec_round(x)
        emitted += len(em)
        x = em[-1]
    e1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms, wall_ms, load_s = max_over_ranks([e0.elapsed_time(e1), wall * 1e3, load_s], torch.device("cuda", local))
    launches = st.launches - l0
    info = model.info
    dist.barrier()  # every rank's last exchange is done before any rank frees its exchange block
    st.free()
    model.close()
    s_round = ms / 1e3 / args.steps
    return {"value": round(emitted / (ms / 1e3), 3), "unit": "tok/s", "ms_per_step": round(ms / args.steps, 4),
            "scaling": "strong", "parallelism": f"tp{world}", "gpu_launches_per_rank": launches,
            "e2e": {"value": round(emitted / (wall_ms / 1e3), 3), "unit": "tok/s", "h2d_bytes_per_step": 4 * world,
                    "d2h_bytes_per_step": 4 * (k + 2) * world},
            "per_rank_verify_bytes": info.decode_bytes,
            "load_seconds_max_over_ranks": round(load_s, 3),
            "round_frac_per_rank": None,
            "_s_round": s_round, "_bytes": info.decode_bytes + k * (info.mtp_bytes + info.lm_head_bytes)}


def prefill_timing(model, info, max_pos, seed, rows=128):
    """Prompt prefill (Model::prefill, model.rs:443) of a seeded prompt in chunks of `rows` rows, CUDA-event
    timed on the state's stream: with the tensor-core GEMM for the K-quant matrices (the default), and with the
    CUDA-core GEMV forced for comparison.  The second of two runs is the one reported."""
    import torch

    import qdec

    n = min(512, max_pos - 8)
    prompt = [int(v) for v in np.random.default_rng(seed).integers(0, min(info.vocab, 248044), n)]
    out = {"tokens": n, "rows_per_chunk": rows}
    for key, min_cols in (("tok_s", qdec.PREFILL_GEMM_MIN_COLS), ("tok_s_gemv_path", 0)):
        qdec.tune_gemv(9, min_cols)
        try:
            for _ in range(2):
                st = model.new_state(spec_k=0, max_rows=rows)
                stream = torch.cuda.ExternalStream(st.stream)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                a.record(stream)
                st.prefill(prompt)
                b.record(stream)
                torch.cuda.synchronize()
                st.free()
            out[key] = round(n / (a.elapsed_time(b) / 1e3), 1)
        finally:
            qdec.tune_gemv(9, qdec.PREFILL_GEMM_MIN_COLS)
    out["gemm"] = "K-quant matrices: tcgen05 GEMM, 128 rows x 16 columns per CTA (bit-exact); tok_s_gemv_path: 4-column GEMV passes"
    return out


def run_spec_qdec(args, world, rank, local):
    import torch

    import qdec

    torch.cuda.set_device(local)
    preset = args.preset
    if rank == 0:
        path = ensure_checkpoint(preset, SPEC_SEED)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    path = checkpoint_path(preset, SPEC_SEED)
    k = SPEC_K
    max_pos = PROMPT_LEN + (args.warmup + args.steps) * (k + 1) * 2 + 64
    tp_res = None
    if world > 1 and not args.no_tp:
        # one sequence over all the GPUs first (its prompt is the same on every rank), then the replicas
        vocab = qdec.tp_plan(path, 0, 1)["v_rows"]
        try:
            tp_res = tp_spec_timing(path, args, world, rank, local, k, spec_prompt(vocab, SPEC_SEED + 1), max_pos)
        except qdec.QdecError as e:  # e.g. a model whose heads do not split over this many GPUs: report, go on
            tp_res = {"error": str(e)[:300], "_s_round": None, "_bytes": None}
            import torch.distributed as dist

            dist.barrier()
    t_load = time.perf_counter()
    model = qdec.Model(path, device=local, max_pos=max_pos)
    load_s = time.perf_counter() - t_load
    info = model.info
    prompt = spec_prompt(info.vocab, SPEC_SEED + 1 + rank)
    st = model.new_state(spec_k=k, max_rows=32)
    stream = torch.cuda.ExternalStream(st.stream)
    x = st.spec_prefill(prompt)
    for _ in range(args.warmup):
        x = st.spec_round(x)[-1]

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()

    torch.cuda.synchronize()
    barrier()
    c0 = st.counters()
    l0 = st.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    emitted = 0
    with ClockSampler(local) as clk:
        torch.cuda.profiler.start()  # a profiler run with --profile-from-start off sees exactly the timed rounds
        t0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            em = st.spec_round(x)
            emitted += len(em)
            x = em[-1]
        e1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1)
    c1 = st.counters()
    launches = st.launches - l0
    # forced drafts (drafts = the plain run's own next tokens, every draft accepted): the m = k regime
    plain = model.new_state(spec_k=0, max_rows=32)
    n_forced = min(args.steps, 64)
    seq = qdec.generate(plain, prompt, 1 + n_forced * (k + 1) + k, stop=False)
    plain.free()
    fs = model.new_state(spec_k=k, max_rows=32)
    fx = fs.spec_prefill(prompt)
    fstream = torch.cuda.ExternalStream(fs.stream)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pos = 1
    f0.record(fstream)
    forced_tokens = 0
    for _ in range(n_forced):
        fs.set_drafts(seq[pos:pos + k])
        em = fs.spec_round(fx)
        forced_tokens += len(em)
        pos += len(em)
        fx = em[-1]
    f1.record(fstream)
    torch.cuda.synchronize()
    forced_ms = f0.elapsed_time(f1)
    fs.free()
    # sampled decoding (temperature 0.8, top-k 20, top-p 0.95): the exact acceptance rule instead of greedy
    ss = model.new_state(spec_k=k, max_rows=32)
    ss.set_sampler(temperature=0.8, top_k=20, top_p=0.95, seed=SPEC_SEED)
    sx = ss.spec_prefill(prompt)
    for _ in range(3):
        sx = ss.spec_round(sx)[-1]
    sstream = torch.cuda.ExternalStream(ss.stream)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sc0 = ss.counters()
    n_samp = min(args.steps, 64)
    s_tokens = 0
    s0.record(sstream)
    for _ in range(n_samp):
        em = ss.spec_round(sx)
        s_tokens += len(em)
        sx = em[-1]
    s1.record(sstream)
    torch.cuda.synchronize()
    sampled_ms = s0.elapsed_time(s1)
    sc1 = ss.counters()
    ss.free()
    pre = prefill_timing(model, info, max_pos, SPEC_SEED + 7)
    plain_res = plain_decode_timing(model, prompt, min(args.steps, 64)) if not args.quick else None
    batch_res = batch_decode_timing(model, prompt, min(args.steps, 32)) if not args.quick and world == 1 else None
    if world > 1:
        import torch.distributed as dist

        ms, wall_ms, forced_ms = max_over_ranks([ms, wall * 1e3, forced_ms], torch.device("cuda", local))
        wall = wall_ms / 1e3
        tt = torch.tensor([emitted, forced_tokens], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt)
        emitted_all, forced_all = tt.tolist()
    else:
        emitted_all, forced_all = emitted, forced_tokens
    if rank != 0:
        return
    rounds = args.steps
    s_round = ms / 1e3 / rounds
    peak, peak_kind = peaks()
    alg, kern_ms = dominant_gemv_timing(torch.device("cuda", local))
    achieved = alg / (kern_ms / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "gemv_pair_q4k_n4_traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    verify_bytes = info.decode_bytes
    round_bytes = verify_bytes + k * (info.mtp_bytes + info.lm_head_bytes)
    line = {
        "metric": "decode tok/s (greedy, --spec 3) Qwen3.8-27B Q4_K_M", "value": round(emitted_all / (ms / 1e3), 3),
        "unit": "tok/s", "n_gpus": world, "steps": rounds, "warmup": args.warmup, "ms_per_step": round(ms / rounds, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "Q4_K_M weights x Q8_K activations, f32",
        "data": "synthetic (seeded N(0,0.02) weights in the Q4_K_M recipe; seeded uniform prompt ids)",
        "config": {"workload": f"{preset} --spec 3 (BASELINE config {4 if PROMPT_LEN <= 1024 else 5})", "prompt": PROMPT_LEN, "k": k,
                   "global_batch": world, "parallelism": f"replicas x{world}",
                   "l2": f"weights {info.weight_bytes / 1e9:.1f} GB >> 126 MB L2"},
        "spec": {"s_per_round": round(s_round, 6), "accepted_per_round": (c1["accepted"] - c0["accepted"]) / rounds,
                 "emitted_per_round": (c1["emitted"] - c0["emitted"]) / rounds,
                 "forced_drafts_tok_s": round(forced_all / (forced_ms / 1e3), 3),
                 "forced_s_per_round": round(forced_ms / 1e3 / n_forced, 6),
                 "sampled": {"sampler": "temperature 0.8, top_k 20, top_p 0.95", "rounds": n_samp,
                             "tok_s_rank0": round(s_tokens / (sampled_ms / 1e3), 3),
                             "s_per_round": round(sampled_ms / 1e3 / n_samp, 6),
                             "accepted_per_round": (sc1["accepted"] - sc0["accepted"]) / n_samp}},
        # through the C ABI from the host: x_p in (4 bytes), {keep, emitted ids} out, one round per call
        "e2e": {"value": round(emitted_all / wall, 3), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * (k + 2)},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "kq_gemv7m_kernel (integer lanes on mma.sync): ffn_gate + ffn_up Q4_K 2 x 17408x5120, N=4 (one launch)",
                     "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "alg_bytes_per_launch": alg,
                     "launch_us": round(kern_ms * 1e3, 2),
                     "round": {"alg_bytes": round_bytes, "achieved": round(round_bytes / s_round / 1e9, 1),
                               "frac": round(round_bytes / s_round / 1e9 / peak, 4),
                               "north_star_frac": round(17.8e9 / s_round / 1e9 / peak, 4)}},
        "clocks": clk.summary(),
        "prefill": pre,
        # qdec_open: the GGUF data section read by several threads into pinned staging, uploaded chunk by chunk,
        # repacked in place (the checkpoint file sits in /dev/shm, so this is the memory-to-HBM path)
        "load": {"seconds": round(load_s, 3), "gb_s": round(info.weight_bytes / load_s / 1e9, 2)},
    }
    if plain_res is not None:
        line["plain_decode"] = plain_res
    if batch_res is not None:
        line["batch_decode"] = batch_res
    if not args.quick:
        line["gemv"] = gemv_table(torch.device("cuda", local))
        line["long_kv"] = long_kv_timing(path, local, k, min(args.steps, 20))
    if tp_res is not None:
        s_r, b = tp_res.pop("_s_round"), tp_res.pop("_bytes")
        if s_r:
            tp_res["round_frac_per_rank"] = round(b / s_r / 1e9 / peak, 4)
        line["tp"] = tp_res
    if world == 1 and not args.no_cpu_baseline:
        tok_s, s_rnd, stats, cores = oracle_spec_sample(path, k, PROMPT_LEN, 3)
        line["cpu_baseline"] = {"value": round(tok_s, 5), "unit": "tok/s", "cores": cores, "kind": CPU_KIND,
                                "variant": CPU_VARIANT,
                                "sample": f"{stats['rounds']} --spec {k} rounds after the {PROMPT_LEN}-token prompt "
                                          f"({s_rnd:.2f} s/round; prompt prefill {stats['prefill_seconds']:.1f} s)"}
        # parity on the full 27B checkpoint: the GPU's ids for the CPU leg's prompt and round count
        want = stats["ids"]
        got = gpu_spec_ids(model, k, stats["prompt"], len(want))
        line["parity"] = {"ids_equal": got == want, "n_ids": len(want), "prompt_len": len(stats["prompt"]),
                          "against": "the CPU oracle's --spec 3 loop on the same checkpoint and prompt (the cpu_baseline run)"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["qdec", "reference"], default="qdec")
    ap.add_argument("--workload", choices=["spec", "gemv"], default="spec")
    ap.add_argument("--preset", default="27b", help="synthetic checkpoint of the spec workload")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="only the headline rounds (no plain decode, GEMV table or 8K-KV run)")
    ap.add_argument("--no-tp", action="store_true", help="with --gpus > 1: replicas only (no tensor-parallel run)")
    ap.add_argument("--prompt-len", type=int, default=None,
                    help="prompt ids before the timed rounds (default 128; 8064 grows the KV cache to ~8192: config 5)")
    ap.add_argument("--profile-gemv", action="store_true",
                    help="run the dominant GEMV (ffn_gate + ffn_up, Q4_K 2 x 17408x5120, N=4, one launch) 4 times and exit: "
                         "the ncu capture target")
    ap.add_argument("--no-gemv-mma", action="store_true",
                    help="with --profile-gemv: the CUDA-core (dp4a) form of the 4-column Q4_K GEMV instead of the warp-MMA form")
    ap.add_argument("--profile-prefill-gemm", action="store_true",
                    help="run the prefill's tensor-core GEMM (Q4_K 17408x5120, 32 columns) 4 times, print its event time "
                         "and exit: the ncu capture target")
    args = ap.parse_args()
    if args.profile_gemv or args.profile_prefill_gemm:
        import torch

        import qdec

        torch.cuda.set_device(0)
        if args.no_gemv_mma:
            qdec.tune_gemv(10, 0)
        n = 32 if args.profile_prefill_gemm else 4
        _, ms = dominant_gemv_timing(torch.device("cuda", 0), launches=4, n=n)
        print(json.dumps({"kernel": f"Q4_K 2 x 17408x5120 (gate + up) x {n} columns", "us_per_launch": round(ms * 1e3, 2)}))
        return
    if args.prompt_len:
        global PROMPT_LEN
        PROMPT_LEN = args.prompt_len
    if args.steps is None:
        args.steps = 2000 if args.workload == "gemv" else 50
    if args.warmup is None:
        args.warmup = 20 if args.workload == "gemv" else 5
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        # the CPU arm needs no process group: rank 0 runs, the other ranks exit without work
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup("nccl")
    if args.workload == "spec":
        run_spec_qdec(args, world, rank, local)
    else:
        run_qdec(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
