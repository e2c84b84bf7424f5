"""Host side of the N > 1 paths on CPU with gloo, world_size 2: the tensor-parallel shard plan of
each rank tiles every split dimension exactly once, and bench.py's cross-rank timing reduction
takes the slowest rank."""
import os
import sys

import pytest
import torch.distributed as dist
import torch.multiprocessing as tmp

from scalatorch import ffm
from scalatorch.models import LlamaConfig, shard_plan

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LLAMA70B = dict(vocab_size=128256, hidden_size=8192, intermediate_size=28672, num_layers=80,
                num_attention_heads=64, num_key_value_heads=8, max_positions=8192, tie_word_embeddings=False)


def _worker(rank, world, port, results):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "scala-torch_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from scalatorch.models import LlamaConfig as C, shard_plan as plan
        p = plan(C(**LLAMA70B), rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, p)
        import bench
        slowest = bench.max_over_ranks([1.0 + rank, 10.0 - rank], device=None)
        results[rank] = (gathered, slowest)
    finally:
        dist.destroy_process_group()


def _tiles(ranges, total):
    ranges = sorted(ranges)
    return ranges[0][0] == 0 and ranges[-1][1] == total and all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))


def test_shard_plans_tile_the_model_over_gloo_ranks():
    world = 2
    mgr = tmp.Manager()
    results = mgr.dict()
    port = 29500 + os.getpid() % 1000
    tmp.spawn(_worker, args=(world, port, results), nprocs=world, join=True)
    plans, slowest = results[0]
    assert results[1][0] == plans
    c = LlamaConfig(**LLAMA70B)
    assert _tiles([p.heads for p in plans], c.num_attention_heads)
    assert _tiles([p.kv_heads for p in plans], c.num_key_value_heads)
    assert _tiles([p.intermediate for p in plans], c.intermediate_size)
    assert _tiles([p.vocab for p in plans], c.vocab_size)
    assert _tiles([p.o_cols for p in plans], c.hidden_size)
    assert _tiles([p.down_cols for p in plans], c.intermediate_size)
    whole = shard_plan(c, 0, 1).weight_bytes
    embed = c.vocab_size * c.hidden_size * 2
    assert sum(p.weight_bytes for p in plans) == whole + (world - 1) * embed  # the embedding is replicated
    assert slowest == [2.0, 10.0]  # max over ranks, element-wise


def test_uneven_splits_are_rejected_before_any_device_work():
    smol = LlamaConfig(vocab_size=49152, hidden_size=576, intermediate_size=1536, num_layers=30,
                       num_attention_heads=9, num_key_value_heads=3)
    assert shard_plan(smol, 0, 1).heads == (0, 9)
    with pytest.raises(ffm.IllegalArgumentException):
        shard_plan(smol, 0, 2)  # 9 heads / 3 KV heads do not split over 2 ranks


def _dying_worker(rank, world, port, results):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "scala-torch_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # a rank that leaves between steps, with nothing in flight
    try:
        import bench
        bench.max_over_ranks([1.0], device=None)
        results[rank] = "no error"
    except Exception as e:  # the survivor learns of it through the collective's error
        results[rank] = type(e).__name__


def test_a_rank_that_leaves_makes_the_next_collective_fail_not_hang():
    mgr = tmp.Manager()
    results = mgr.dict()
    port = 30500 + os.getpid() % 1000
    ctx = tmp.get_context("spawn")
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert results.get(0) not in (None, "no error")
