"""The shape-sharded search's host logic on CPU: the GPU search step is replaced by a fake, everything else (unit
queue, heartbeats, in-flight blame, restarts, per-shape rows, shared winner cache, summary) is the real code.
World size 2 over gloo, spawned workers, and ranks that die mid-unit (the failure is made on the host)."""
from __future__ import annotations

import json
import os
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as tmp_mp

from cs464_b200 import shard
from cs464_b200.winner_cache import WinnerCache

ENV = {"hw_id": "test-gpu", "kernel_src": "k1", "torch": "t", "cuda_runtime": "c", "driver": "d", "clock_lock": None}
SEL = "bm128_bn128_bk64_w4_s6_g8_sk1"
BEST = "bm256_bn256_bk64_w4_s3_g8_sk1"


def fake_search(shape, unit, k=3, space=None, crashed=(), on_config=None):
    """One unit: the selected config runs 2 % slower than the unit's best on this 'GPU'."""
    us = 1e-6 * shape["M"] * shape["N"] * shape["K"] * (1.0 + 0.01 * unit["slice"])
    if on_config:
        on_config(SEL)
    row = {"i": unit["i"], "slice": unit["slice"], "of": unit["of"], "M": shape["M"], "N": shape["N"],
           "K": shape["K"], "top": [SEL], "crashed": sorted(crashed), "n_screened": 2, "wall_s": 0.0,
           "screen": [[SEL, us * 1.02, "ok"], [f"{BEST}" if unit["slice"] == 0 else f"bm256_bn128_bk64_w4_s{3 + unit['slice']}_g8_sk1", us, "ok"]]}
    if unit["slice"] == 0:
        row.update(chosen=SEL, chosen_short_us=us)
    return row


def _units(shapes, of=1):
    return [{"u": n, "i": i, "slice": j, "of": of, "cost": float(s["M"] * s["N"] * s["K"])}
            for n, (i, s, j) in enumerate((i, s, j) for i, s in enumerate(shapes) for j in range(of))]


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


def test_two_ranks_run_every_unit_once(tmp_path):
    shapes = [{"M": 16 * (i + 1), "N": 64, "K": 128} for i in range(11)]
    queue = str(tmp_path / "queue.jsonl")
    shard.ShapeQueue.create(queue, shapes, units=_units(shapes, of=2))
    cache = str(tmp_path / "wc.jsonl")
    results = str(tmp_path / "stats.json")
    port = 29500 + os.getpid() % 1000
    tmp_mp.spawn(_rank_main, args=(2, port, queue, str(tmp_path), cache, results), nprocs=2, join=True)
    q = shard.ShapeQueue(queue)
    claims = q.claims()
    assert sorted(c["u"] for c in claims) == list(range(22))
    assert {c["rank"] for c in claims} == {0, 1}
    assert q.finished()
    assert len(WinnerCache(cache, env=ENV)) == 11
    s = shard.summarize(str(tmp_path), json.loads(open(results).read()))
    # gap per GPU: the selected config is 2 % over each unit's best, whatever the units' absolute times
    assert s["shapes"] == 11 and s["ranks"] == 2 and abs(s["gap_median"] - 0.02) < 1e-9
    assert all(r["best_key"] == BEST and r["units"] == 2 for r in s["results"])


def test_queue_runs_costliest_units_first(tmp_path):
    shapes = [{"M": 1, "N": 1, "K": 1}, {"M": 64, "N": 64, "K": 64}]
    q = shard.ShapeQueue.create(tmp_path / "q.jsonl", shapes, units=_units(shapes))
    assert q.claim(0)[0]["i"] == 1 and q.claim(0)[0]["i"] == 0 and q.claim(0) is None


def test_plan_units_slices_long_shapes():
    big, small = {"M": 8192, "N": 8192, "K": 8192}, {"M": 64, "N": 64, "K": 64}
    units = shard.plan_units([small, big], space=64, target_s=0.2)
    per = {i: [u for u in units if u["i"] == i] for i in (0, 1)}
    assert len(per[0]) < len(per[1])
    assert sorted(u["slice"] for u in per[1]) == list(range(per[1][0]["of"]))


def test_create_starts_a_fresh_run(tmp_path):
    """Rows of an earlier run in the same directory are neither kept nor counted."""
    shapes = [{"M": 64, "N": 64, "K": 64}]
    queue = tmp_path / "queue.jsonl"
    shard.ShapeQueue.create(queue, shapes, units=_units(shapes))
    shard.run_rank(0, str(queue), str(tmp_path), None, search=fake_search)
    first = shard.summarize(str(tmp_path))
    (tmp_path / "search_rank0.jsonl").write_text('{"i": 0, "gap": 9.9}\n')  # an old-format leftover
    shard.ShapeQueue.create(queue, shapes, units=_units(shapes))
    assert not (tmp_path / "search_rank0.jsonl").exists()
    assert shard.summarize(str(tmp_path))["shapes"] == 0
    shard.run_rank(0, str(queue), str(tmp_path), None, search=fake_search)
    second = shard.summarize(str(tmp_path))
    assert second["shapes"] == 1 and second["run"] != first["run"]


def test_dead_rank_unit_is_reclaimed_with_blame(tmp_path):
    """Rank 0 claims a unit, records a config in flight and stops answering; once its heartbeat is stale rank 1
    takes the unit over and the in-flight config is recorded as crashed for the shape."""
    shapes = [{"M": 64, "N": 64, "K": 64}]
    q0 = shard.ShapeQueue.create(tmp_path / "q.jsonl", shapes, units=_units(shapes), stale_s=0.3)
    unit, _, crashed = q0.claim(0)
    assert crashed == set()
    q0.set_inflight(0, unit["u"], SEL)
    q1 = shard.ShapeQueue(tmp_path / "q.jsonl", stale_s=0.3)
    assert q1.claim(1) is None  # rank 0 is still alive
    time.sleep(0.5)
    unit1, _, crashed1 = q1.claim(1)
    assert unit1["u"] == unit["u"] and crashed1 == {SEL}
    assert q1.status()["crashed"] == {0: [SEL]}


def test_release_dead_blames_and_frees_at_once(tmp_path):
    shapes = [{"M": 64, "N": 64, "K": 64}, {"M": 32, "N": 32, "K": 32}]
    q = shard.ShapeQueue.create(tmp_path / "q.jsonl", shapes, units=_units(shapes))
    unit, _, _ = q.claim(3)
    q.set_inflight(3, unit["u"], BEST)
    assert q.release_dead(3) == [unit["u"]]
    again, _, crashed = q.claim(4)
    assert again["u"] == unit["u"] and crashed == {BEST}


def flaky_worker(rank, device, args, results):
    """Spawned worker that dies (exit status 3, a poisoned context) on its first start after claiming a unit and
    recording a config in flight; restarted, it finishes the queue."""
    starts = os.path.join(args["out"], f"starts{rank}")
    first = not os.path.exists(starts)
    with open(starts, "a") as f:
        f.write("x\n")
    if rank == 1:  # rank 0 claims a unit, dies and is restarted before rank 1 takes any work
        deadline = time.time() + 60
        while time.time() < deadline:
            p0 = os.path.join(args["out"], "starts0")
            if os.path.exists(p0) and len(open(p0).read().split()) >= 2:
                break
            time.sleep(0.05)
    if rank == 0 and first:
        q = shard.ShapeQueue(args["queue"])
        unit, _, _ = q.claim(rank)
        q.set_inflight(rank, unit["u"], SEL)
        os._exit(shard.EXIT_POISONED)
    res = shard.run_rank(rank, args["queue"], args["out"], args["cache"], search=fake_search, cache_env=ENV)
    results.put({"rank": rank, "ok": True, **res})


def silent_worker(rank, device, args, results):
    """Spawned worker that exits without putting a result (the parent must not wait for it forever)."""
    os._exit(0)


def test_spawned_worker_that_dies_is_restarted(tmp_path):
    shapes = [{"M": 16 * (i + 1), "N": 64, "K": 64} for i in range(6)]
    queue = str(tmp_path / "queue.jsonl")
    shard.ShapeQueue.create(queue, shapes, units=_units(shapes))
    logs = []
    stats = shard.run_spawned(queue, str(tmp_path), str(tmp_path / "wc.jsonl"), 2, worker=flaky_worker,
                              poll_s=0.1, log=logs.append)
    q = shard.ShapeQueue(queue)
    assert q.finished()
    assert any("rank 0 failed" in x for x in logs)
    assert sorted(s["rank"] for s in stats) == [0, 1]
    s = shard.summarize(str(tmp_path), stats)
    assert s["shapes"] == 6 and s["crashed"] == 1
    assert len(WinnerCache(str(tmp_path / "wc.jsonl"), env=ENV)) == 6


def test_spawned_worker_without_result_does_not_hang(tmp_path):
    shapes = [{"M": 64, "N": 64, "K": 64}]
    queue = str(tmp_path / "queue.jsonl")
    shard.ShapeQueue.create(queue, shapes, units=_units(shapes))
    logs = []
    t0 = time.time()
    stats = shard.run_spawned(queue, str(tmp_path), None, 1, worker=silent_worker, max_restarts=1, poll_s=0.1,
                              log=logs.append)
    assert stats == [] and time.time() - t0 < 60
    assert len(logs) == 2  # the first start and its one restart both reported


def test_worker_threads_split_the_host():
    n = os.cpu_count() or 1
    assert shard.worker_threads(1) == n
    assert shard.worker_threads(8) == max(1, n // 8)
    assert shard.worker_threads(10 ** 6) == 1


@pytest.mark.parametrize("ratios,expect", [((1.02, 1.0), 0.02), ((1.0, 1.05), 0.05)])
def test_combine_takes_the_worst_per_gpu_ratio(ratios, expect):
    rows = []
    for j, r in enumerate(ratios):
        base = 10.0 * (j + 1)  # a different 'GPU speed' per unit: only the ratio inside each unit matters
        rows.append({"i": 0, "slice": j, "of": 2, "M": 1, "N": 1, "K": 1, "n_screened": 2,
                     "screen": [[SEL, base * r, "ok"], [BEST if j == 0 else "x", base, "ok"]],
                     **({"chosen": SEL} if j == 0 else {})})
    res = shard.combine(rows)
    assert abs(res["gap"] - expect) < 1e-9
    assert shard.combine(rows[:1]) is None
