"""Host logic of the tensor-parallel Qwen2 decode, on CPU: the library's shard
plan (tq_qwen_shard_plan, the one tq_qwen_create uses) covers every head, row
and column exactly once per replica group, and the NCCL id reaches every rank
of a world-size-2 gloo process group."""
import os

import pytest

from conftest import free_port
import torch.distributed as dist
import torch.multiprocessing as mp

from tensai_b200.decode import QWEN_7B, broadcast_nccl_id, qwen_shard_plan


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plan_partitions_the_model(world):
    cfg = QWEN_7B
    plans = [qwen_shard_plan(cfg, world, r) for r in range(world)]
    for key, total in (("o_rows", cfg["d"]), ("ffn", cfg["ffn"]), ("vocab", cfg["vocab"])):
        covered = sorted(p[key] for p in plans)
        assert covered[0][0] == 0 and covered[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))
        assert all((b - a) % (64 if key != "vocab" else 2) == 0 for a, b in covered)
    heads = set()
    for p in plans:
        heads.update(range(*p["q_heads"]))
        a0, a1 = p["att_dims"]
        o0, o1 = p["o_rows"]
        assert a0 <= o0 and o1 <= a1  # o_proj rows lie in this rank's attention output
        g = cfg["n_head"] // cfg["n_kv"]
        assert p["q_heads"][0] // g == p["kv_heads"][0] and p["q_heads"][1] // g == p["kv_heads"][1]
    assert heads == set(range(cfg["n_head"]))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_plan_seen_by_gloo_ranks(world):
    """Every rank of a gloo group asks the library for its own slice; together
    the slices partition the model (the check above, across processes)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_plan_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(got) == list(range(world))
    rows = sorted(got[r]["o_rows"] for r in range(world))
    assert rows[0][0] == 0 and rows[-1][1] == QWEN_7B["d"]
    assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))


def _plan_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = qwen_shard_plan(QWEN_7B, dist.get_world_size(), dist.get_rank())
        out = [None] * world
        dist.all_gather_object(out, plan)  # every rank sees the whole plan
        assert out[rank] == plan
        q.put((rank, plan))
    finally:
        dist.destroy_process_group()


def test_shard_plan_rejects_uneven_splits():
    with pytest.raises(ValueError):
        qwen_shard_plan(QWEN_7B, 3, 0)
    with pytest.raises(ValueError):
        qwen_shard_plan(dict(QWEN_7B, ffn=18944 + 64), 8, 0)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, broadcast_nccl_id(dist)))
    finally:
        dist.destroy_process_group()


def test_nccl_id_reaches_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(got[0]) == 128 and got[0] == got[1]
