"""Shape-sharded selector search over the GPUs of one host.

A GEMM runs on one GPU; what shards is the search: shapes are independent units. One process per GPU claims shapes
from a shared work queue (a flock-protected JSONL of claims, biggest problems first, so long shapes do not end up
last), searches each on its own GPU, writes a result row to its own JSONL and appends the winner to the ONE shared
winner cache file (flock + fsync, tune/winner_cache.py's concurrency rule). There is no collective on the data path;
with torchrun the process group only carries start/end barriers.

Per shape a rank runs the selector (the ranker's top-k, validated and short-timed: `search.search_shape`) and the
full-space screen (`search.screen_shape`), which gives best-in-pool; the row's `gap` = screen time of the selected
config / best screen time - 1 (the reference's regret, results/README.md:79).

    python -m cs464_b200.shard --gpus 8 --suite config5 [--limit N] [--space N] [--out DIR]
"""
from __future__ import annotations

import argparse
import fcntl
import json
import os
import statistics
import sys
import time
from pathlib import Path


class ShapeQueue:
    """Dynamic work queue of shapes shared by processes: `<path>.shapes.json` (the list) + `<path>` (claims)."""

    def __init__(self, path: str | os.PathLike):
        self.path = Path(path)
        self.shapes = json.loads(self.path.with_suffix(".shapes.json").read_text())["shapes"]
        flops = [2 * s["M"] * s["N"] * s["K"] for s in self.shapes]
        self.order = sorted(range(len(self.shapes)), key=lambda i: (-flops[i], i))

    @classmethod
    def create(cls, path: str | os.PathLike, shapes: list[dict]) -> "ShapeQueue":
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        tmp.write_text(json.dumps({"shapes": shapes}))
        os.replace(tmp, path.with_suffix(".shapes.json"))
        path.write_text("")
        return cls(path)

    def claim(self, rank: int) -> tuple[int, dict] | None:
        with open(self.path, "a+") as f:
            fcntl.flock(f, fcntl.LOCK_EX)
            f.seek(0)
            taken = set()
            for line in f.read().splitlines():
                try:
                    taken.add(int(json.loads(line)["i"]))
                except (ValueError, KeyError, TypeError):
                    continue
            for i in self.order:
                if i not in taken:
                    f.seek(0, os.SEEK_END)
                    f.write(json.dumps({"i": i, "rank": rank, "t": time.time()}) + "\n")
                    f.flush()
                    os.fsync(f.fileno())
                    return i, self.shapes[i]
        return None

    def claims(self) -> list[dict]:
        out = []
        for line in self.path.read_text().splitlines():
            try:
                out.append(json.loads(line))
            except ValueError:
                continue
        return out


def _append_row(path: Path, row: dict) -> None:
    with open(path, "a") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        f.write(json.dumps(row) + "\n")
        f.flush()
        os.fsync(f.fileno())


def search_one(shape: dict, *, k: int = 3, space: int | None = None, ranker=None) -> dict:
    """Selector + full-space screen for one shape on the current GPU."""
    import torch

    from cs464_b200.gate import make_inputs, reference
    from cs464_b200.keys import parse_key
    from cs464_b200.search import choose, measure, screen_shape, shape_space
    from cs464_b200.matmul import B200Matmul
    M, N, K = shape["M"], shape["N"], shape["K"]
    t0 = time.perf_counter()
    a, b = make_inputs(M, N, K, torch.float16, scale_b=shape.get("weight_std", 1.0))
    ref = reference(a, b)
    if ranker is None:
        from cs464_b200.search import _ranker_default
        ranker = _ranker_default()
    t_rank = time.perf_counter()
    keys = ranker.rank(M, N, K, k, order="diverse")
    t_rank = time.perf_counter() - t_rank
    sel = measure(M, N, K, torch.float16, [("b200_sm100a_v1", key, B200Matmul(parse_key(key))) for key in keys],
                  inputs=(a, b, ref))
    choice = choose(sel["candidates"])
    t_select = time.perf_counter() - t0
    pool = shape_space(M, N, K)
    if space is not None and space < len(pool):
        step = max(1, len(pool) // space)
        pool = pool[::step][:space]
    have = {c.key() for c in pool}
    pool += [parse_key(x) for x in keys if x not in have]  # the selector's picks are always in the pool
    scr = screen_shape(M, N, K, pool, inputs=(a, b, ref))
    us = {r["key"]: r["us"] for r in scr["rows"] if r["us"] is not None}
    chosen = choice.get("key")
    gap = (us[chosen] / scr["best_us"] - 1.0) if chosen in us and scr["best_us"] else None
    return {"M": M, "N": N, "K": K, "chosen": chosen, "chosen_short_us": choice.get("us"),
            "screen": [[r["key"], round(r["us"], 3)] for r in scr["rows"] if r["status"] in ("ok", "slow")],
            "chosen_screen_us": us.get(chosen), "best_key": scr["best_key"], "best_us": scr["best_us"], "gap": gap,
            "n_screened": scr["n_configs"], "n_ok": sum(1 for r in scr["rows"] if r["status"] == "ok"),
            "select_s": t_select, "rank_s": t_rank,
            "validate_s": sum(x.get("setup_s", 0.0) for x in sel["candidates"]),
            "timing_s": sum(x.get("time_s", 0.0) for x in sel["candidates"]), "wall_s": time.perf_counter() - t0}


def run_rank(rank: int, queue_path: str, out_dir: str, cache_path: str | None, *, k: int = 3, space: int | None = None,
             search=search_one, max_shapes: int | None = None, cache_env: dict | None = None) -> dict:
    """Claim and search shapes until the queue is empty; returns {"rank", "n", "wall_s"}."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    q = ShapeQueue(queue_path)
    wc = None
    if cache_path:
        from cs464_b200.winner_cache import WinnerCache
        wc = WinnerCache(cache_path, env=cache_env)
    t0 = time.perf_counter()
    n = 0
    while max_shapes is None or n < max_shapes:
        got = q.claim(rank)
        if got is None:
            break
        i, shape = got
        row = {"i": i, "rank": rank, **search(shape, k=k, space=space)}
        _append_row(out / f"search_rank{rank}.jsonl", row)
        if wc is not None and row.get("best_key"):
            wc.put(shape["M"], shape["N"], shape["K"], "fp16", k=int(row.get("n_screened") or 1),
                   choice={"key": row["best_key"], "family": "b200_sm100a_v1", "us": row["best_us"],
                           "mode": "screen"}, extra={"selected": row.get("chosen"), "gap": row.get("gap")})
        n += 1
    return {"rank": rank, "n": n, "wall_s": time.perf_counter() - t0}


def summarize(out_dir: str, rank_stats: list[dict]) -> dict:
    rows = []
    for p in sorted(Path(out_dir).glob("search_rank*.jsonl")):
        rows += [json.loads(x) for x in p.read_text().splitlines() if x.strip()]
    gaps = sorted(r["gap"] for r in rows if r.get("gap") is not None)
    wall = max((s["wall_s"] for s in rank_stats), default=0.0)

    def pct(p):
        return gaps[min(len(gaps) - 1, int(round(p / 100 * (len(gaps) - 1))))] if gaps else None
    return {"shapes": len(rows), "ranks": len(rank_stats), "wall_s": wall,
            "shapes_per_s": (len(rows) / wall) if wall > 0 else None, "gap_median": pct(50), "gap_p95": pct(95),
            "gap_mean": statistics.fmean(gaps) if gaps else None}


def worker_threads(gpus: int) -> int:
    """Host threads per search process: the host's cores split between the processes. The ranker's tree-ensemble
    predict starts one OpenMP thread per core in every process; with one process per GPU those spinning pools
    oversubscribe the host (measured on 2 GPUs: the ranking step went from 33 ms to 2.2 s per shape)."""
    return max(1, (os.cpu_count() or 1) // max(1, gpus))


def limit_host_threads(n: int) -> None:
    """Cap this process's CPU thread pools (OpenMP of the ranker's predict, BLAS, torch's intra-op pool) at n."""
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(n)
    except ImportError:
        pass
    import torch
    torch.set_num_threads(n)


def _worker(rank: int, device: int, args: dict, results):
    os.environ["CUDA_VISIBLE_DEVICES"] = str(device)
    limit_host_threads(worker_threads(args.get("gpus", 1)))
    res = run_rank(rank, args["queue"], args["out"], args["cache"], k=args["k"], space=args["space"],
                   max_shapes=args.get("max_shapes"))
    results.put(res)


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--suite", default="config5")
    ap.add_argument("--limit", type=int, default=None, help="first N shapes of the suite")
    ap.add_argument("--space", type=int, default=None, help="screen N configs per shape (default: all)")
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--out", default="search_out")
    ap.add_argument("--cache", default=None, help="shared winner cache file (default: <out>/winner_cache.jsonl)")
    a = ap.parse_args(argv)
    from cs464_b200 import suites
    shapes = suites.load(a.suite)[: a.limit]
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    cache = a.cache or str(out / "winner_cache.jsonl")
    queue = str(out / "queue.jsonl")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:  # torchrun: one process per GPU, barriers only
        import torch
        import torch.distributed as dist
        rank = int(os.environ["RANK"])
        limit_host_threads(worker_threads(int(os.environ.get("LOCAL_WORLD_SIZE", world))))
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group("gloo")
        if rank == 0:
            ShapeQueue.create(queue, shapes)
        dist.barrier()
        res = run_rank(rank, queue, str(out), cache, k=a.k, space=a.space)
        stats = [None] * world
        dist.all_gather_object(stats, res)
        dist.destroy_process_group()
        summary = summarize(str(out), stats) if rank == 0 else {}
    else:
        import multiprocessing as mp
        ShapeQueue.create(queue, shapes)
        ctx = mp.get_context("spawn")
        results = ctx.Queue()
        args = {"queue": queue, "out": str(out), "cache": cache, "k": a.k, "space": a.space, "gpus": a.gpus}
        procs = [ctx.Process(target=_worker, args=(r, r, args, results)) for r in range(a.gpus)]
        for p in procs:
            p.start()
        stats = [results.get() for _ in procs]
        for p in procs:
            p.join()
        summary = summarize(str(out), stats)
    if summary:
        summary.update({"gpus": max(world, a.gpus), "suite": a.suite, "space": a.space, "k": a.k})
        (out / "summary.json").write_text(json.dumps(summary, indent=1))
        print(json.dumps(summary), flush=True)
    return summary


if __name__ == "__main__":
    sys.exit(0 if main() is not None else 1)
