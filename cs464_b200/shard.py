"""Shape-sharded selector search over the GPUs of one host.

A GEMM runs on one GPU; what shards is the search: shapes are independent. Each shape's work is cut into units —
strided slices of its screen — so one long shape no longer sets the tail: with N ranks the units of the biggest
shapes are spread over all of them. One process per GPU claims units from a shared queue (an append-only, flock'd
JSONL event log next to the unit list; costliest units first), runs each on its own GPU and appends its row to the
shape's result file. There is no collective on the data path.

Per shape: the ranker's top k are proposed (deterministic, so every unit knows them); unit 0 also runs the selector
(validate + short-time the top k, `search.measure` / `search.choose`). Every unit screens the top k plus its slice of
the shape-pruned space (`search.screen_shape`, the reference's stage-1 rule, tune/sweep.py:216-274). The selector's
gap (the reference's regret, results/README.md:79) is combined per GPU: each unit times the selected config and its
slice's best on the same GPU, and gap = max over units of t_selected / t_best - 1, which equals the one-GPU figure
without mixing clocks of different GPUs. The shape's winner (the fastest over all units) goes to the shared winner
cache (flock + fsync) as soon as its last unit is in.

Failure handling (the reference's in-flight blame and restart, tune/runner.py:174-184, :222-249 and
tune/sweep.py:292-352):
  * a rank touches a heartbeat file and records the config it is validating or timing (`inflight_rank<r>.json`)
    before every config;
  * a unit whose owner's heartbeat went stale (the process died or hangs) is claimable again; the config that owner
    had in flight is recorded as crashed for the shape, and every later unit of the shape skips it
    ("invalid: crashed");
  * a worker that meets a poisoned CUDA context (`ContextPoisoned`) blames the culprit, releases its unit and exits
    with status 3; in spawn mode the parent restarts a worker on that GPU (up to --max-restarts), and a worker that
    dies without a result is handled the same way;
  * under torchrun the survivors reclaim a dead rank's units once its heartbeat is stale; nothing waits on a
    collective after the start barrier.
Each run has an id: `ShapeQueue.create` clears the previous run's files in the directory, and the summary counts
only rows of this run.

    python -m cs464_b200.shard --gpus 8 --suite config5 [--limit N] [--space N] [--out DIR]
"""
from __future__ import annotations

import argparse
import fcntl
import json
import math
import os
import shutil
import statistics
import sys
import time
import uuid
from pathlib import Path

EXIT_POISONED = 3
STALE_S = 90.0             # a heartbeat older than this marks its rank dead (a config never takes this long)
UNIT_TARGET_S = 0.5        # estimated screening seconds per unit: well under a rank's share at 8 GPUs
POLL_S = 0.05              # how often a rank with nothing claimable looks at the queue again
SCREEN_SAMPLES_EST = 16    # samples a config that is not cut gets (1 + the screen's 15)
PER_CONFIG_HOST_S = 2.5e-3 # validation and launch overheads per config, measured on B200 runs of the screen
FLUSH_S = 1.2e-4           # one L2 flush of the cold protocol


def _now() -> float:
    return time.time()


def est_kernel_s(M: int, N: int, K: int) -> float:
    """Rough GPU time of one good config: a fixed cost plus the tensor work at ~1.2 PFLOP/s."""
    return 5e-6 + 2.0 * M * N * K / 1.2e15


def est_config_s(M: int, N: int, K: int) -> float:
    return PER_CONFIG_HOST_S + SCREEN_SAMPLES_EST * (est_kernel_s(M, N, K) + FLUSH_S)


def shape_pool(M: int, N: int, K: int, space: int | None) -> list:
    """The configs screened for a shape: the shape-pruned space, strided down to `space` configs when given."""
    from cs464_b200.search import shape_space
    pool = shape_space(M, N, K)
    if space is not None and space < len(pool):
        step = max(1, len(pool) // space)
        pool = pool[::step][:space]
    return pool


def plan_units(shapes: list[dict], space: int | None, *, target_s: float = UNIT_TARGET_S,
               max_slices: int = 16) -> list[dict]:
    """Units of work: each shape's screen cut into `of` strided slices sized to ~target_s of estimated work."""
    units = []
    for i, s in enumerate(shapes):
        n_cfg = len(shape_pool(s["M"], s["N"], s["K"], space))
        cost = max(1, n_cfg) * est_config_s(s["M"], s["N"], s["K"])
        of = int(max(1, min(max_slices, max(1, n_cfg // 8), math.ceil(cost / target_s))))
        for j in range(of):
            units.append({"u": len(units), "i": i, "slice": j, "of": of, "cost": cost / of})
    return units


class ShapeQueue:
    """Work queue of (shape, slice) units shared by the processes of one host.

    Files next to `path` (the event log, JSONL, appended under flock):
      <path>.shapes.json        {"run", "shapes", "units", "space"}
      <path>                    events: claim {u, rank} / done {u, rank} / release {u, rank} / crashed {i, key}
      <dir>/hb/rank<r>          heartbeat: its mtime is the rank's last sign of life
      <dir>/inflight_rank<r>.json  {"run", "u", "i", "key"}: the config rank r has in flight
    """

    def __init__(self, path: str | os.PathLike, stale_s: float = STALE_S):
        self.path = Path(path)
        doc = json.loads(self.path.with_suffix(".shapes.json").read_text())
        self.run = doc["run"]
        self.shapes = doc["shapes"]
        self.units = doc["units"]
        self.space = doc.get("space")
        self.stale_s = stale_s
        self.order = sorted(range(len(self.units)), key=lambda u: (-self.units[u]["cost"], u))
        self.dir = self.path.parent

    @classmethod
    def create(cls, path: str | os.PathLike, shapes: list[dict], *, space: int | None = None,
               units: list[dict] | None = None, stale_s: float = STALE_S) -> "ShapeQueue":
        """A fresh run in the queue's directory: the previous run's rows, heartbeats and in-flight records go."""
        path = Path(path)
        d = path.parent
        d.mkdir(parents=True, exist_ok=True)
        for p in list(d.glob("search_rank*.jsonl")) + list(d.glob("inflight_rank*.json")) + \
                list(d.glob("rank*.stats.json")):
            p.unlink(missing_ok=True)
        for sub in ("units", "hb"):
            if (d / sub).exists():
                shutil.rmtree(d / sub)
        (d / "units").mkdir()
        (d / "hb").mkdir()
        if units is None:
            units = plan_units(shapes, space)
        doc = {"run": uuid.uuid4().hex[:12], "shapes": shapes, "units": units, "space": space}
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        tmp.write_text(json.dumps(doc))
        os.replace(tmp, path.with_suffix(".shapes.json"))
        path.write_text("")
        return cls(path, stale_s)

    # -------------------------------------------------------------------------------------------- liveness
    def heartbeat(self, rank: int) -> None:
        p = self.dir / "hb" / f"rank{rank}"
        try:
            os.utime(p)
        except FileNotFoundError:
            p.touch()

    def alive(self, rank: int, now: float | None = None) -> bool:
        try:
            return (now or _now()) - (self.dir / "hb" / f"rank{rank}").stat().st_mtime < self.stale_s
        except FileNotFoundError:
            return False

    def set_inflight(self, rank: int, u: int | None, key: str | None) -> None:
        p = self.dir / f"inflight_rank{rank}.json"
        tmp = p.with_suffix(f".tmp{os.getpid()}")
        tmp.write_text(json.dumps({"run": self.run, "u": u, "i": None if u is None else self.units[u]["i"],
                                   "key": key}))
        os.replace(tmp, p)

    def inflight(self, rank: int) -> dict | None:
        try:
            d = json.loads((self.dir / f"inflight_rank{rank}.json").read_text())
        except (OSError, ValueError):
            return None
        return d if d.get("run") == self.run else None

    # -------------------------------------------------------------------------------------------- event log
    def _append(self, f, ev: dict) -> None:
        f.seek(0, os.SEEK_END)
        f.write(json.dumps(ev) + "\n")
        f.flush()
        os.fsync(f.fileno())

    @staticmethod
    def _state(lines) -> tuple[dict, set, dict]:
        """(owner per unit {u: (rank, t)}, done units, crashed keys per shape)."""
        owner, done, crashed = {}, set(), {}
        for line in lines:
            try:
                e = json.loads(line)
            except ValueError:
                continue  # a torn line from a process that died mid-write
            ev = e.get("ev", "claim")
            if ev == "claim":
                owner[e["u"]] = (e["rank"], e.get("t", 0.0))
            elif ev == "done":
                done.add(e["u"])
            elif ev == "release":
                if owner.get(e["u"], (None,))[0] == e.get("rank"):
                    owner.pop(e["u"], None)
            elif ev == "crashed":
                crashed.setdefault(e["i"], set()).add(e["key"])
        return owner, done, crashed

    def _blame(self, f, rank: int, u: int) -> None:
        """Record the config a dead `rank` had in flight on unit u as crashed for the unit's shape."""
        d = self.inflight(rank)
        if d and d.get("u") == u and d.get("key"):
            self._append(f, {"ev": "crashed", "i": self.units[u]["i"], "key": d["key"], "rank": rank})

    def claim(self, rank: int) -> tuple[dict, dict, set] | None:
        """The next unit for `rank`: (unit, shape, crashed keys of the shape), or None when nothing is claimable
        right now (everything done, or the rest held by live ranks)."""
        self.heartbeat(rank)
        now = _now()
        with open(self.path, "a+") as f:
            fcntl.flock(f, fcntl.LOCK_EX)
            f.seek(0)
            owner, done, crashed = self._state(f.read().splitlines())
            for u in self.order:
                if u in done:
                    continue
                o = owner.get(u)
                if o is not None and (o[0] == rank or self.alive(o[0], now)):
                    continue
                if o is not None:  # its owner died: blame what it had in flight, then take the unit over
                    self._blame(f, o[0], u)
                    f.seek(0)
                    _, _, crashed = self._state(f.read().splitlines())
                self._append(f, {"ev": "claim", "u": u, "rank": rank, "t": now})
                unit = self.units[u]
                return unit, self.shapes[unit["i"]], set(crashed.get(unit["i"], ()))
        return None

    def mark(self, ev: str, u: int, rank: int, **extra) -> None:
        with open(self.path, "a+") as f:
            fcntl.flock(f, fcntl.LOCK_EX)
            self._append(f, {"ev": ev, "u": u, "rank": rank, **extra})

    def release_dead(self, rank: int) -> list[int]:
        """A rank known dead (its process exited): blame its in-flight config and release its open units now,
        without waiting for the heartbeat to go stale. Returns the released units."""
        with open(self.path, "a+") as f:
            fcntl.flock(f, fcntl.LOCK_EX)
            f.seek(0)
            owner, done, _ = self._state(f.read().splitlines())
            out = [u for u, (r, _) in owner.items() if r == rank and u not in done]
            for u in out:
                self._blame(f, rank, u)
                self._append(f, {"ev": "release", "u": u, "rank": rank})
        return out

    def status(self) -> dict:
        owner, done, crashed = self._state(self.path.read_text().splitlines())
        return {"units": len(self.units), "done": len(done), "open": len(self.units) - len(done),
                "crashed": {i: sorted(k) for i, k in crashed.items()}}

    def finished(self) -> bool:
        return self.status()["open"] == 0

    def events(self) -> list[dict]:
        out = []
        for line in self.path.read_text().splitlines():
            try:
                out.append(json.loads(line))
            except ValueError:
                continue
        return out

    def claims(self) -> list[dict]:
        return [e for e in self.events() if e.get("ev", "claim") == "claim"]

    # -------------------------------------------------------------------------------------------- results
    def unit_file(self, i: int) -> Path:
        return self.dir / "units" / f"{i}.jsonl"

    def add_row(self, row: dict) -> list[dict]:
        """Append a unit's row to its shape's file; returns every row of this run for the shape (under the lock)."""
        p = self.unit_file(row["i"])
        with open(p, "a+") as f:
            fcntl.flock(f, fcntl.LOCK_EX)
            f.seek(0, os.SEEK_END)
            f.write(json.dumps({**row, "run": self.run}) + "\n")
            f.flush()
            os.fsync(f.fileno())
            f.seek(0)
            rows = []
            for line in f.read().splitlines():
                try:
                    r = json.loads(line)
                except ValueError:
                    continue
                if r.get("run") == self.run:
                    rows.append(r)
        return rows


def combine(rows: list[dict]) -> dict | None:
    """A shape's result from its unit rows (one per slice), or None while slices are missing. Unit 0 carries the
    selector's choice; gap = max over units of (the selected config's time / the unit's best time) - 1, each
    ratio taken on one GPU."""
    if not rows:
        return None
    of = rows[0]["of"]
    by_slice = {}
    for r in rows:
        by_slice.setdefault(r["slice"], r)
    if len(by_slice) < of:
        return None
    sel = by_slice.get(0, {})
    chosen = sel.get("chosen")
    best_key, best_us, ratio, n_scr, n_ok = None, None, None, 0, 0
    for r in by_slice.values():
        times = {k: us for k, us, st in r["screen"] if us is not None}
        ok = {k: us for k, us, st in r["screen"] if st == "ok" and us is not None}
        n_scr += r["n_screened"]
        n_ok += len(ok)
        if not ok:
            continue
        kb = min(ok, key=ok.get)
        if best_us is None or ok[kb] < best_us:
            best_key, best_us = kb, ok[kb]
        if chosen in times:
            q = times[chosen] / ok[kb]
            ratio = q if ratio is None else max(ratio, q)
    s0 = by_slice[min(by_slice)]
    return {"i": s0["i"], "M": s0["M"], "N": s0["N"], "K": s0["K"], "chosen": chosen,
            "chosen_short_us": sel.get("chosen_short_us"), "best_key": best_key, "best_us": best_us,
            "gap": None if ratio is None else max(0.0, ratio - 1.0), "units": of, "n_screened": n_scr, "n_ok": n_ok,
            "crashed": sorted({k for r in by_slice.values() for k in r.get("crashed", [])}),
            "wall_s": sum(r.get("wall_s", 0.0) for r in by_slice.values())}


def search_unit(shape: dict, unit: dict, *, k: int = 3, space: int | None = None, ranker=None, crashed=(),
                on_config=None) -> dict:
    """One unit on the current GPU: inputs and fp32 reference, the ranker's top k, the selector (unit 0 only), and
    the screen of the top k plus this unit's slice of the pool."""
    import torch

    from cs464_b200.gate import make_inputs, reference
    from cs464_b200.keys import parse_key
    from cs464_b200.matmul import B200Matmul
    from cs464_b200.search import FAMILY, choose, measure, screen_shape, selection_keys
    M, N, K = shape["M"], shape["N"], shape["K"]
    t0 = time.perf_counter()
    if ranker is None:
        from cs464_b200.search import _ranker_default
        ranker = _ranker_default()
    a, b = make_inputs(M, N, K, torch.float16, scale_b=shape.get("weight_std", 1.0))
    ref = reference(a, b)
    t_rank = time.perf_counter()
    top = selection_keys(ranker, M, N, K, k)
    t_rank = time.perf_counter() - t_rank
    row = {"i": unit["i"], "slice": unit["slice"], "of": unit["of"], "M": M, "N": N, "K": K, "top": top,
           "crashed": sorted(crashed), "rank_s": t_rank}
    if unit["slice"] == 0:
        ts = time.perf_counter()
        sel = measure(M, N, K, torch.float16, [(FAMILY, key, B200Matmul(parse_key(key))) for key in top],
                      inputs=(a, b, ref), skip=crashed, on_config=on_config)
        choice = choose(sel["candidates"])
        row.update(chosen=choice.get("key"), chosen_short_us=choice.get("us"), select_s=time.perf_counter() - ts)
    pool = shape_pool(M, N, K, space)[unit["slice"]::unit["of"]]
    cfgs = [parse_key(x) for x in top] + [c for c in pool if c.key() not in set(top)]
    scr = screen_shape(M, N, K, cfgs, inputs=(a, b, ref), skip=crashed, on_config=on_config)
    row.update(screen=[[r["key"], None if r["us"] is None else round(r["us"], 3), r["status"]] for r in scr["rows"]],
               n_screened=scr["n_configs"], wall_s=time.perf_counter() - t0)
    del a, b, ref
    return row


def _put_winner(wc, res: dict) -> None:
    if wc is None or not res or not res.get("best_key"):
        return
    wc.put(res["M"], res["N"], res["K"], "fp16", k=int(res.get("n_screened") or 1),
           choice={"key": res["best_key"], "family": "b200_sm100a_v1", "us": res["best_us"], "mode": "screen"},
           extra={"selected": res.get("chosen"), "gap": res.get("gap")})


def run_rank(rank: int, queue_path: str, out_dir: str, cache_path: str | None, *, k: int = 3,
             space: int | None = None, search=search_unit, max_units: int | None = None,
             cache_env: dict | None = None, wait_others: bool = True, deadline_s: float | None = None,
             stale_s: float = STALE_S) -> dict:
    """Claim and run units until the queue is finished (or, with wait_others=False, until nothing is claimable).
    A rank whose units all sit with live ranks waits, so a peer that dies is covered once its heartbeat is stale.
    Returns {"rank", "units", "shapes_finished", "wall_s"}; also written to <out>/rank<r>.stats.json."""
    from cs464_b200.gate import ContextPoisoned
    out = Path(out_dir)
    q = ShapeQueue(queue_path, stale_s=stale_s)
    wc = None
    if cache_path:
        from cs464_b200.winner_cache import WinnerCache
        wc = WinnerCache(cache_path, env=cache_env)
    t0 = time.perf_counter()
    n = finished = 0
    while max_units is None or n < max_units:
        got = q.claim(rank)
        if got is None:
            if not wait_others or q.finished():
                break
            if deadline_s is not None and time.perf_counter() - t0 > deadline_s:
                break
            time.sleep(POLL_S)
            continue
        unit, shape, crashed = got
        u = unit["u"]

        def on_config(key, _u=u):
            q.heartbeat(rank)
            q.set_inflight(rank, _u, key)

        try:
            row = search(shape, unit, k=k, space=space, crashed=crashed, on_config=on_config)
        except ContextPoisoned as e:
            q.mark("crashed", u, rank, i=unit["i"], key=e.culprit.split(":", 1)[-1])
            q.mark("release", u, rank)
            raise
        q.set_inflight(rank, None, None)
        rows = q.add_row({**row, "u": u, "rank": rank})
        q.mark("done", u, rank)
        n += 1
        res = combine(rows)
        if res is not None and len(rows) >= unit["of"]:
            finished += 1
            _put_winner(wc, res)
    stats = {"rank": rank, "units": n, "shapes_finished": finished, "wall_s": time.perf_counter() - t0}
    (out / f"rank{rank}.stats.json").write_text(json.dumps({**stats, "run": q.run}))
    return stats


def summarize(out_dir: str, rank_stats: list[dict] | None = None, queue_path: str | None = None) -> dict:
    """Per-shape results of the current run (from the unit files) and the throughput over `rank_stats` (or the
    ranks' stats files): shapes/s = finished shapes / the longest rank wall time."""
    out = Path(out_dir)
    q = ShapeQueue(queue_path or out / "queue.jsonl")
    if rank_stats is None:
        rank_stats = []
        for p in sorted(out.glob("rank*.stats.json")):
            d = json.loads(p.read_text())
            if d.get("run") == q.run:
                rank_stats.append(d)
    results = []
    for i in range(len(q.shapes)):
        p = q.unit_file(i)
        if not p.exists():
            continue
        rows = []
        for line in p.read_text().splitlines():
            try:
                r = json.loads(line)
            except ValueError:
                continue
            if r.get("run") == q.run:
                rows.append(r)
        res = combine(rows)
        if res is not None:
            results.append(res)
    gaps = sorted(r["gap"] for r in results if r.get("gap") is not None)
    wall = max((s["wall_s"] for s in rank_stats), default=0.0)

    def pct(p):
        return gaps[min(len(gaps) - 1, int(round(p / 100 * (len(gaps) - 1))))] if gaps else None
    return {"run": q.run, "shapes": len(results), "shapes_total": len(q.shapes), "units": len(q.units),
            "ranks": len(rank_stats), "wall_s": wall, "shapes_per_s": (len(results) / wall) if wall > 0 else None,
            "gap_median": pct(50), "gap_p95": pct(95), "gap_mean": statistics.fmean(gaps) if gaps else None,
            "crashed": sum(len(r["crashed"]) for r in results), "results": results}


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
    """Spawned worker: one GPU, units until the queue is finished. Puts exactly one result, even on failure; a
    poisoned CUDA context exits with status 3 after its unit was blamed and released."""
    os.environ["CUDA_VISIBLE_DEVICES"] = str(device)
    try:
        limit_host_threads(worker_threads(args.get("gpus", 1)))
        res = run_rank(rank, args["queue"], args["out"], args["cache"], k=args["k"], space=args["space"],
                       stale_s=args.get("stale_s", STALE_S))
        results.put({"rank": rank, "ok": True, **res})
    except BaseException as e:  # noqa: BLE001 (the parent must always hear back)
        from cs464_b200.gate import ContextPoisoned
        poisoned = isinstance(e, ContextPoisoned)
        results.put({"rank": rank, "ok": False, "poisoned": poisoned, "error": f"{type(e).__name__}: {e}"[:300]})
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(EXIT_POISONED if poisoned else 1)


def run_spawned(queue: str, out: str, cache: str | None, gpus: int, *, k: int = 3, space: int | None = None,
                max_restarts: int = 4, stale_s: float = STALE_S, worker=_worker, poll_s: float = 0.5,
                log=print) -> list[dict]:
    """One spawned process per GPU; a worker that dies or reports an error is released (its in-flight config
    blamed) and restarted on its GPU, up to max_restarts per GPU. Returns the per-rank stats of the finished
    workers."""
    import multiprocessing as mp
    import queue as queue_mod
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    args = {"queue": queue, "out": out, "cache": cache, "k": k, "space": space, "gpus": gpus, "stale_s": stale_s}
    q = ShapeQueue(queue, stale_s=stale_s)
    procs = {r: ctx.Process(target=worker, args=(r, r, args, results)) for r in range(gpus)}
    restarts = {r: 0 for r in range(gpus)}
    heard: dict[int, dict] = {}
    for p in procs.values():
        p.start()
    stats = []
    while procs:
        try:
            msg = results.get(timeout=poll_s)
            heard[msg["rank"]] = msg
        except queue_mod.Empty:
            pass
        for r, p in list(procs.items()):
            if p.is_alive():
                continue
            p.join()
            msg = heard.pop(r, None)
            if p.exitcode == 0 and msg and msg.get("ok"):
                stats.append({x: msg[x] for x in ("rank", "units", "shapes_finished", "wall_s") if x in msg})
                del procs[r]
                continue
            released = q.release_dead(r)
            why = (msg or {}).get("error") or f"exit code {p.exitcode} without a result"
            log(f"[shard] rank {r} failed ({why}); released units {released}")
            if restarts[r] < max_restarts and not q.finished():
                restarts[r] += 1
                procs[r] = ctx.Process(target=worker, args=(r, r, args, results))
                procs[r].start()
            else:
                del procs[r]
    return stats


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--suite", default="config5")
    ap.add_argument("--limit", type=int, default=None, help="first N shapes of the suite")
    ap.add_argument("--space", type=int, default=None, help="screen N configs per shape (default: all)")
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--out", default="search_out")
    ap.add_argument("--cache", default=None, help="shared winner cache file (default: <out>/winner_cache.jsonl)")
    ap.add_argument("--max-restarts", type=int, default=4)
    a = ap.parse_args(argv)
    from cs464_b200 import suites
    shapes = suites.load(a.suite)[: a.limit]
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    cache = a.cache or str(out / "winner_cache.jsonl")
    queue = str(out / "queue.jsonl")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:  # torchrun: one process per GPU; the process group only carries the start barrier
        from datetime import timedelta

        import torch
        import torch.distributed as dist
        rank = int(os.environ["RANK"])
        limit_host_threads(worker_threads(int(os.environ.get("LOCAL_WORLD_SIZE", world))))
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
        if rank == 0:
            ShapeQueue.create(queue, shapes, space=a.space)
        dist.barrier()
        dist.destroy_process_group()
        run_rank(rank, queue, str(out), cache, k=a.k, space=a.space)
        summary = summarize(str(out)) if rank == 0 else {}
    else:
        ShapeQueue.create(queue, shapes, space=a.space)
        t0 = time.perf_counter()
        stats = run_spawned(queue, str(out), cache, a.gpus, k=a.k, space=a.space, max_restarts=a.max_restarts)
        summary = summarize(str(out), stats or None)
        summary["parent_wall_s"] = time.perf_counter() - t0
    if summary:
        results = summary.pop("results")
        summary.update({"gpus": max(world, a.gpus), "suite": a.suite, "space": a.space, "k": a.k})
        (out / "summary.json").write_text(json.dumps(summary, indent=1))
        (out / "results.jsonl").write_text("".join(json.dumps(r) + "\n" for r in results))
        print(json.dumps(summary), flush=True)
    return summary


if __name__ == "__main__":
    sys.exit(0 if main() is not None else 1)
