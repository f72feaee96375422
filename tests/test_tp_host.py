"""Host side of tensor parallelism, without a GPU: the shard plan partitions every split dimension of the tiny and
27B configurations exactly (each row / head on one rank, in order), unsplittable worlds are rejected, and the
handle exchange and max-over-ranks timing reduction work across two gloo ranks."""
import os

import pytest

import qdec

TINY = dict(hidden=256, ffn=768, vocab=4096, n_head=4, n_head_kv=2, dn_k_heads=2, dn_v_heads=4)
B27 = dict(hidden=5120, ffn=17408, vocab=248320, n_head=24, n_head_kv=4, dn_k_heads=16, dn_v_heads=48)


def plans(d, world):
    return [qdec.tp_plan_dims(**d, rank=r, world=world) for r in range(world)]


def ranges_partition(ps, lo, cnt, total, align=1):
    at = 0
    for p in ps:
        assert p[lo] == at and p[cnt] > 0 and p[lo] % align == 0 and p[cnt] % align == 0
        at += p[cnt]
    assert at == total


@pytest.mark.parametrize("d,world", [(TINY, 1), (TINY, 2), (B27, 1), (B27, 2), (B27, 4), (B27, 8)])
def test_plan_partitions_every_split(d, world):
    ps = plans(d, world)
    ranges_partition(ps, "kh_lo", "nk", d["dn_k_heads"])
    ranges_partition(ps, "qh_lo", "nq", d["n_head"])
    ranges_partition(ps, "ff_lo", "ff_rows", d["ffn"], align=256)
    ranges_partition(ps, "h_lo", "h_rows", d["hidden"], align=8)
    ranges_partition(ps, "v_lo", "v_rows", d["vocab"], align=8)
    # V head p reads K head p % n_k: the V heads of a rank are exactly those tied to its K heads
    owner = {}
    for p in ps:
        assert p["nv"] == p["nk"] * d["dn_v_heads"] // d["dn_k_heads"]
        for g in range(d["dn_v_heads"] // d["dn_k_heads"]):
            for j in range(p["nk"]):
                v = g * d["dn_k_heads"] + p["kh_lo"] + j
                assert v not in owner
                owner[v] = p["rank"]
                assert p["kh_lo"] <= v % d["dn_k_heads"] < p["kh_lo"] + p["nk"]
    assert sorted(owner) == list(range(d["dn_v_heads"]))
    # every query head of a rank reads a kv head the rank holds, through the local map h' / (nq / nkv)
    group = d["n_head"] // d["n_head_kv"]
    for p in ps:
        for hl in range(p["nq"]):
            assert (p["qh_lo"] + hl) // group == p["kv_lo"] + hl // (p["nq"] // p["nkv"])
        assert 0 <= p["kv_lo"] and p["kv_lo"] + p["nkv"] <= d["n_head_kv"]


@pytest.mark.parametrize("d,world", [(TINY, 4), (B27, 3), (B27, 16), (B27, 0)])
def test_plan_rejects_worlds_that_do_not_split(d, world):
    with pytest.raises(qdec.QdecError) as e:
        qdec.tp_plan_dims(**d, rank=0, world=world)
    assert e.value.code in (qdec.EFORMAT, qdec.EINVAL)


def test_plan_from_the_gguf_header(tmp_path):
    path = tmp_path / "tiny.gguf"
    qdec.synth_gguf(path, "tiny", 5)
    for world in (1, 2):
        for r in range(world):
            assert qdec.tp_plan(path, r, world) == qdec.tp_plan_dims(**TINY, rank=r, world=world)


def _gloo_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        hs = qdec.gather_handles(bytes([rank]) * qdec.TP_HANDLE_BYTES)
        import bench

        worst = bench.max_over_ranks([float(10 + rank), float(5 - rank)], torch.device("cpu"))
        q.put((rank, [h[0] for h in hs], [len(h) for h in hs], worst))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_handles_in_rank_order_and_take_the_max():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, first_bytes, lens, worst in res:
        assert first_bytes == [0, 1] and lens == [qdec.TP_HANDLE_BYTES] * 2
        assert worst == [11.0, 5.0]
