"""The shape-sharded search's host logic with world_size 2 over gloo on CPU: the GPU search step is replaced by a
fake, everything else (queue, per-rank rows, shared winner cache, barriers, summary) is the real code."""
from __future__ import annotations

import json
import os

import torch.distributed as dist
import torch.multiprocessing as tmp_mp

from cs464_b200 import shard
from cs464_b200.winner_cache import WinnerCache

ENV = {"hw_id": "test-gpu", "kernel_src": "k1", "torch": "t", "cuda_runtime": "c", "driver": "d", "clock_lock": None}


def fake_search(shape, k=3, space=None):
    us = 1e-6 * shape["M"] * shape["N"] * shape["K"]
    return {"M": shape["M"], "N": shape["N"], "K": shape["K"], "chosen": "bm128_bn128_bk64_w4_s6_g8_sk1",
            "chosen_screen_us": us * 1.02, "best_key": "bm256_bn256_bk64_w4_s3_g8_sk1", "best_us": us, "gap": 0.02,
            "n_screened": 10, "wall_s": 0.0}


def _rank_main(rank, world, port, queue, out, cache, results_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    dist.barrier()
    res = shard.run_rank(rank, queue, out, cache, search=fake_search, cache_env=ENV)
    stats = [None] * world
    dist.all_gather_object(stats, res)
    if rank == 0:
        with open(results_path, "w") as f:
            json.dump(stats, f)
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_claim_every_shape_once(tmp_path):
    shapes = [{"M": 16 * (i + 1), "N": 64, "K": 128} for i in range(23)]
    queue = str(tmp_path / "queue.jsonl")
    shard.ShapeQueue.create(queue, shapes)
    cache = str(tmp_path / "wc.jsonl")
    results = str(tmp_path / "stats.json")
    port = 29500 + os.getpid() % 1000
    tmp_mp.spawn(_rank_main, args=(2, port, queue, str(tmp_path), cache, results), nprocs=2, join=True)
    claims = shard.ShapeQueue(queue).claims()
    assert sorted(c["i"] for c in claims) == list(range(23))
    assert {c["rank"] for c in claims} == {0, 1}
    rows = [json.loads(x) for r in (0, 1) for x in (tmp_path / f"search_rank{r}.jsonl").read_text().splitlines()]
    assert sorted(r["i"] for r in rows) == list(range(23))
    assert len(WinnerCache(cache, env=ENV)) == 23
    stats = json.loads(open(results).read())
    s = shard.summarize(str(tmp_path), stats)
    assert s["shapes"] == 23 and s["ranks"] == 2 and abs(s["gap_median"] - 0.02) < 1e-9


def test_queue_orders_biggest_first(tmp_path):
    q = shard.ShapeQueue.create(tmp_path / "q.jsonl", [{"M": 1, "N": 1, "K": 1}, {"M": 64, "N": 64, "K": 64}])
    assert q.claim(0)[0] == 1 and q.claim(0)[0] == 0 and q.claim(0) is None


def test_worker_threads_split_the_host():
    from cs464_b200.shard import worker_threads
    n = os.cpu_count() or 1
    assert worker_threads(1) == n
    assert worker_threads(8) == max(1, n // 8)
    assert worker_threads(10 ** 6) == 1
