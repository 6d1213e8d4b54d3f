"""cuBLASLt best-of-search (the reference's B3+ comparator, baselines/cublaslt_search.py:93-133, :188-237): a budgeted
search of cuBLASLt's configuration space beyond its heuristic's top-N, run in a subprocess per shape.

Measurement only: the sm_100a family never dispatches here. The search, in this module's own order:
  1. seeds: the heuristic's best-fit top 32, and for every algorithm id the heuristic's picks restricted to that
     algorithm (search mode "limited by algo id");
  2. neighbourhood: each valid seed with one attribute changed at a time — split-K over {2, 3, 4, 6, 8, 12, 16}
     (each split keeping at least 64 of K), every reduction scheme the algorithm allows, CTA swizzle on or off, each
     stages id and tile id the algorithm lists, custom options 0..3 — every variant filtered by
     cublasLtMatmulAlgoCheck and the 32 MiB workspace cap;
  3. the rest of the space (algorithm x tile x stages x split-K x reduction x swizzle x custom) in a seeded random
     order, while the time budget lasts.
Candidates are screened by device time (hot, bursts of 5 launches behind the timer's gate, 3 samples) in that order
until the budget runs out; the fastest `top_k` distinct configs come back as runnable backends (family
"cublaslt_deep"), which the caller validates and times with its own protocol. The best over these and the heuristic's
top 16 (`cs464_b200.cublaslt.candidates`) is B3+.

The search runs in a child process (`python -m cs464_b200.cublaslt_deep M N K --out F`), so a configuration that
faults cannot take the caller down; its result is cached as JSON per shape and budget. `search_batch_isolated` fills
that cache for a whole suite from one child (`--batch shapes.json --cache-dir D`).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import random
import subprocess
import sys
import time
from pathlib import Path

import torch

from cs464_b200.cublaslt import (CUBLAS_COMPUTE_32F, CUDA_R_32F, WORKSPACE_BYTES, _DT, CublasLtMatmul, _Algo, _Heur,
                                 _Problem, _check, _handle, _lib)

VERSION = 1
CAP_SPLITK, CAP_REDUCTION_MASK, CAP_SWIZZLE, CAP_TILE_IDS, CAP_CUSTOM_MAX, CAP_STAGES_IDS = 0, 1, 2, 6, 7, 13
ATTR_ID, ATTR_TILE, ATTR_SPLITK, ATTR_REDUCTION, ATTR_SWIZZLE, ATTR_CUSTOM, ATTR_STAGES = 0, 1, 2, 3, 4, 5, 6
ATTR_INNER, ATTR_CLUSTER = 7, 8
FIELDS = {"algo_id": ATTR_ID, "tile_id": ATTR_TILE, "stages_id": ATTR_STAGES, "splitk": ATTR_SPLITK,
          "reduction": ATTR_REDUCTION, "swizzle": ATTR_SWIZZLE, "custom": ATTR_CUSTOM, "inner": ATTR_INNER,
          "cluster": ATTR_CLUSTER}
SETTABLE = ("tile_id", "stages_id", "splitk", "reduction", "swizzle", "custom", "inner", "cluster")
SPLITS = (2, 3, 4, 6, 8, 12, 16)
CUSTOM_MAX = 3
SEARCH_LIMITED_BY_ALGO_ID = 1


def _declare(lib) -> None:
    V, P = C.c_void_p, C.POINTER
    if getattr(lib, "_b2g_deep_declared", False):
        return
    lib.cublasLtMatmulAlgoGetIds.argtypes = [V, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                             P(C.c_int), P(C.c_int)]
    lib.cublasLtMatmulAlgoInit.argtypes = [V, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                           P(_Algo)]
    lib.cublasLtMatmulAlgoCapGetAttribute.argtypes = [P(_Algo), C.c_int, V, C.c_size_t, P(C.c_size_t)]
    lib.cublasLtMatmulAlgoConfigSetAttribute.argtypes = [P(_Algo), C.c_int, V, C.c_size_t]
    lib.cublasLtMatmulAlgoConfigGetAttribute.argtypes = [P(_Algo), C.c_int, V, C.c_size_t, P(C.c_size_t)]
    lib.cublasLtMatmulAlgoCheck.argtypes = [V, V, V, V, V, V, P(_Algo), P(_Heur)]
    lib._b2g_deep_declared = True


def _caps_list(lib, algo, cap) -> list[int]:
    n = C.c_size_t(0)
    lib.cublasLtMatmulAlgoCapGetAttribute(C.byref(algo), cap, None, 0, C.byref(n))
    if n.value < 4:
        return []
    buf = (C.c_uint32 * (n.value // 4))()
    if lib.cublasLtMatmulAlgoCapGetAttribute(C.byref(algo), cap, buf, C.sizeof(buf), C.byref(n)):
        return []
    return [int(x) for x in buf]


def _cap(lib, algo, cap) -> int:
    v, n = C.c_int32(0), C.c_size_t(0)
    return int(v.value) if not lib.cublasLtMatmulAlgoCapGetAttribute(C.byref(algo), cap, C.byref(v), 4, C.byref(n)) \
        else 0


def describe(lib, algo: _Algo) -> dict:
    """The configuration attributes of an algorithm struct."""
    out = {}
    for name, attr in FIELDS.items():
        v, n = C.c_uint32(0), C.c_size_t(0)
        if not lib.cublasLtMatmulAlgoConfigGetAttribute(C.byref(algo), attr, C.byref(v), 4, C.byref(n)):
            out[name] = int(v.value)
    return out


def _ident(cfg: dict) -> tuple:
    return tuple(int(cfg.get(k) or 0) for k in FIELDS)


class Space:
    """cuBLASLt's configurations for one problem."""

    def __init__(self, prob: _Problem):
        self.prob = prob
        self.lib = _lib()
        _declare(self.lib)
        self.handle = _handle(prob.device)
        self.ctype = _DT[prob.dtype]

    def init(self, algo_id: int) -> _Algo | None:
        a = _Algo()
        st = self.lib.cublasLtMatmulAlgoInit(self.handle, CUBLAS_COMPUTE_32F, CUDA_R_32F, self.ctype, self.ctype,
                                             self.ctype, self.ctype, algo_id, C.byref(a))
        return a if st == 0 else None

    def build(self, cfg: dict) -> _Heur | None:
        """A checked (algorithm, workspace) for `cfg`, or None if cuBLASLt refuses it or it needs > 32 MiB."""
        a = self.init(cfg["algo_id"])
        if a is None:
            return None
        for name in SETTABLE:
            if cfg.get(name) is None:
                continue
            v = C.c_uint32(int(cfg[name]))
            if self.lib.cublasLtMatmulAlgoConfigSetAttribute(C.byref(a), FIELDS[name], C.byref(v), 4):
                return None
        res = _Heur()
        p = self.prob
        if self.lib.cublasLtMatmulAlgoCheck(self.handle, p.desc, p.la, p.lb, p.lc, p.lc, C.byref(a), C.byref(res)):
            return None
        if res.workspaceSize > WORKSPACE_BYTES:
            return None
        res.algo = a
        return res

    def algo_ids(self) -> list[int]:
        ids, n = (C.c_int * 512)(), C.c_int(0)
        self.lib.cublasLtMatmulAlgoGetIds(self.handle, CUBLAS_COMPUTE_32F, CUDA_R_32F, self.ctype, self.ctype,
                                          self.ctype, self.ctype, 512, ids, C.byref(n))
        return list(ids[:n.value])

    def seeds(self) -> list[dict]:
        out = [describe(self.lib, h.algo) for h in self.prob.heuristics(32)]
        pref = C.c_void_p()
        _check(self.lib.cublasLtMatmulPreferenceCreate(C.byref(pref)), "PreferenceCreate")
        ws = C.c_uint64(WORKSPACE_BYTES)
        mode = C.c_uint32(SEARCH_LIMITED_BY_ALGO_ID)
        self.lib.cublasLtMatmulPreferenceSetAttribute(pref, 1, C.byref(ws), 8)
        self.lib.cublasLtMatmulPreferenceSetAttribute(pref, 0, C.byref(mode), 4)
        p = self.prob
        for aid in self.algo_ids():
            a = self.init(aid)
            if a is None:
                continue
            res = (_Heur * 8)()
            for i in range(8):  # the restricted search reads the algorithm id from each slot
                res[i].algo = a
            cnt = C.c_int(0)
            if not self.lib.cublasLtMatmulAlgoGetHeuristic(self.handle, p.desc, p.la, p.lb, p.lc, p.lc, pref, 8, res,
                                                           C.byref(cnt)):
                out += [describe(self.lib, res[i].algo) for i in range(cnt.value) if res[i].state == 0]
        self.lib.cublasLtMatmulPreferenceDestroy(pref)
        return _unique(out)

    def caps(self, algo_id: int) -> dict:
        a = self.init(algo_id)
        if a is None:
            return {}
        return {"tiles": _caps_list(self.lib, a, CAP_TILE_IDS), "stages": _caps_list(self.lib, a, CAP_STAGES_IDS),
                "splitk": _cap(self.lib, a, CAP_SPLITK) == 1, "reductions": _cap(self.lib, a, CAP_REDUCTION_MASK),
                "swizzle": _cap(self.lib, a, CAP_SWIZZLE) == 1, "custom_max": _cap(self.lib, a, CAP_CUSTOM_MAX)}

    def neighbours(self, cfg: dict, caps: dict, K: int) -> list[dict]:
        out = []
        if caps.get("splitk"):
            reds = [r for r in (1, 2, 4) if caps["reductions"] & r] or [0]
            out += [dict(cfg, splitk=s, reduction=r) for s in SPLITS if K // s >= 64 for r in reds]
        if caps.get("swizzle"):
            out.append(dict(cfg, swizzle=1 - int(cfg.get("swizzle") or 0)))
        out += [dict(cfg, stages_id=s) for s in caps.get("stages", [])]
        out += [dict(cfg, tile_id=t) for t in caps.get("tiles", [])]
        out += [dict(cfg, custom=c) for c in range(min(caps.get("custom_max", 0), CUSTOM_MAX) + 1)]
        return out

    def everything(self, caps_by_id: dict, K: int) -> list[dict]:
        out = []
        for aid, caps in caps_by_id.items():
            splits = [1] + [s for s in SPLITS if caps.get("splitk") and K // s >= 64]
            reds = [r for r in (1, 2, 4) if caps.get("reductions", 0) & r] or [0]
            for t in caps.get("tiles") or [0]:
                for st in caps.get("stages") or [0]:
                    for s in splits:
                        for r in ([0] if s == 1 else reds):
                            for sw in ([0, 1] if caps.get("swizzle") else [0]):
                                for c in range(min(caps.get("custom_max", 0), CUSTOM_MAX) + 1):
                                    out.append({"algo_id": aid, "tile_id": t, "stages_id": st, "splitk": s,
                                                "reduction": r, "swizzle": sw, "custom": c})
        return out


def _unique(cfgs: list[dict]) -> list[dict]:
    seen, out = set(), []
    for c in cfgs:
        k = _ident(c)
        if k not in seen:
            seen.add(k)
            out.append(c)
    return out


def _screen_us(space: Space, res: _Heur, a, b, c, ws) -> float:
    from cs464_b200.timing import Protocol, measure_us
    p, lib = space.prob, space.lib
    algo = res.algo
    size = int(res.workspaceSize)

    def run():
        st = lib.cublasLtMatmul(space.handle, p.desc, C.byref(p.alpha), b.data_ptr(), p.la, a.data_ptr(), p.lb,
                                C.byref(p.beta), c.data_ptr(), p.lc, c.data_ptr(), p.lc, C.byref(algo),
                                ws.data_ptr(), size, torch.cuda.current_stream().cuda_stream)
        if st:
            raise RuntimeError(f"cublasLtMatmul status {st}")
    return measure_us(run, Protocol(mode="hot", burst=5, samples=3, max_samples=3, warmup=1, ci_target=float("inf"),
                                    max_s=0.5), keep_samples=False).median_us


def search(M: int, N: int, K: int, dtype=torch.float16, budget_s: float = 10.0, top_k: int = 8, seed: int = 0) -> dict:
    """Screen cuBLASLt configurations of one shape for up to `budget_s` seconds; returns the fastest `top_k`."""
    t0 = time.perf_counter()
    dev = torch.cuda.current_device()
    space = Space(_Problem(M, N, K, dtype, dev))
    seeds = space.seeds()
    caps_by_id = {aid: space.caps(aid) for aid in sorted({s["algo_id"] for s in seeds} | set(space.algo_ids()))}
    near = _unique([n for s in seeds for n in space.neighbours(s, caps_by_id.get(s["algo_id"], {}), K)])
    rest = space.everything(caps_by_id, K)
    random.Random(seed).shuffle(rest)
    order = _unique(seeds + near + rest)
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn((M, K), generator=g, device="cuda").to(dtype)
    b = torch.randn((K, N), generator=g, device="cuda").to(dtype)
    c = torch.empty((M, N), device="cuda", dtype=dtype)
    ws = torch.empty(WORKSPACE_BYTES, dtype=torch.uint8, device="cuda")
    t_setup = time.perf_counter() - t0
    timed, refused, failed = [], 0, 0
    t1 = time.perf_counter()
    for i, cfg in enumerate(order):
        if time.perf_counter() - t1 > budget_s:
            break
        res = space.build(cfg)
        if res is None:
            refused += 1
            continue
        try:
            us = _screen_us(space, res, a, b, c, ws)
        except RuntimeError:
            failed += 1
            continue
        timed.append({"cfg": describe(space.lib, res.algo), "us": us, "from": "seed" if i < len(seeds) else
                      ("neighbour" if i < len(seeds) + len(near) else "space")})
    timed.sort(key=lambda x: x["us"])
    top = []
    seen = set()
    for t in timed:
        if _ident(t["cfg"]) not in seen:
            seen.add(_ident(t["cfg"]))
            top.append(t)
        if len(top) == top_k:
            break
    return {"version": VERSION, "M": M, "N": N, "K": K, "dtype": str(dtype).replace("torch.", ""),
            "budget_s": budget_s, "n_seeds": len(seeds), "n_neighbours": len(near), "n_space": len(rest),
            "n_timed": len(timed), "n_refused": refused, "n_failed": failed,
            "exhausted": len(timed) + refused + failed >= len(order), "setup_s": round(t_setup, 3),
            "screen_s": round(time.perf_counter() - t1, 3),
            "best_seed_us": min((t["us"] for t in timed if t["from"] == "seed"), default=None), "top": top}


def _cache_path(cache_dir: str | Path, M: int, N: int, K: int, dtype: str, budget_s: float) -> Path:
    return Path(cache_dir) / f"{M}x{N}x{K}_{dtype}_b{budget_s:g}.json"


def _cached(path: Path) -> dict | None:
    if path.exists():
        try:
            d = json.loads(path.read_text())
        except ValueError:
            return None
        if d.get("version") == VERSION:
            return d
    return None


def search_isolated(M: int, N: int, K: int, cache_dir: str | Path, *, dtype: str = "float16", budget_s: float = 10.0,
                    top_k: int = 8, timeout_s: float = 300.0) -> dict:
    """`search` in a child process on the current GPU, cached as JSON per (shape, dtype, budget)."""
    path = _cache_path(cache_dir, M, N, K, dtype, budget_s)
    d = _cached(path)
    if d is not None:
        return d
    path.parent.mkdir(parents=True, exist_ok=True)
    cmd = [sys.executable, "-m", "cs464_b200.cublaslt_deep", str(M), str(N), str(K), "--dtype", dtype,
           "--budget-s", str(budget_s), "--top-k", str(top_k), "--device", str(torch.cuda.current_device()),
           "--out", str(path)]
    try:
        r = subprocess.run(cmd, cwd=Path(__file__).resolve().parent.parent, capture_output=True, text=True,
                           timeout=timeout_s)
        err = None if (r.returncode == 0 and path.exists()) else ((r.stderr.strip().splitlines() or ["?"])[-1][:300])
    except subprocess.TimeoutExpired:
        err = f"timeout after {timeout_s:g} s"
    if err is not None:
        d = {"version": VERSION, "M": M, "N": N, "K": K, "dtype": dtype, "budget_s": budget_s, "error": err,
             "top": []}
        path.write_text(json.dumps(d))
        return d
    return json.loads(path.read_text())


def search_batch_isolated(shapes: list[tuple[int, int, int]], cache_dir: str | Path, *, dtype: str = "float16",
                          budget_s: float = 10.0, top_k: int = 8) -> int:
    """Fill `search_isolated`'s cache for many shapes from ONE child process: one interpreter and CUDA start-up
    (several seconds) instead of one per shape. The child writes each shape's file as soon as it is done, so a child
    that dies part-way (a configuration that faults) loses only the shapes after it; `search_isolated` then searches
    those in a child of their own. Returns how many shapes the child was given."""
    todo = [(M, N, K) for M, N, K in dict.fromkeys(tuple(x) for x in shapes)
            if _cached(_cache_path(cache_dir, M, N, K, dtype, budget_s)) is None]
    if not todo:
        return 0
    Path(cache_dir).mkdir(parents=True, exist_ok=True)
    lst = Path(cache_dir) / f"batch_{os.getpid()}.json"
    lst.write_text(json.dumps(todo))
    cmd = [sys.executable, "-m", "cs464_b200.cublaslt_deep", "--batch", str(lst), "--cache-dir", str(cache_dir),
           "--dtype", dtype, "--budget-s", str(budget_s), "--top-k", str(top_k), "--device",
           str(torch.cuda.current_device())]
    try:
        subprocess.run(cmd, cwd=Path(__file__).resolve().parent.parent, capture_output=True, text=True,
                       timeout=60.0 + len(todo) * (budget_s + 10.0))
    except subprocess.TimeoutExpired:
        pass
    finally:
        lst.unlink(missing_ok=True)
    return len(todo)


def backends(result: dict, dtype=torch.float16) -> list:
    """Runnable backends (family "cublaslt_deep") for a search result's top configs, on the current GPU."""
    prob = _Problem(result["M"], result["N"], result["K"], dtype, torch.cuda.current_device())
    space = Space(prob)
    out = []
    for i, t in enumerate(result.get("top", [])):
        res = space.build(t["cfg"])
        if res is None:
            continue
        be = CublasLtMatmul(prob, res, i)
        be.family = "cublaslt_deep"
        be.key = "d{}_a{algo_id}_t{tile_id}_s{stages_id}_sk{splitk}_r{reduction}_sw{swizzle}_c{custom}".format(
            i, **{k: t["cfg"].get(k, 0) for k in FIELDS})
        be.cfg = {**be.cfg, **t["cfg"], "screen_us": t["us"]}
        out.append(be)
    return out


def _main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="budgeted cuBLASLt configuration search for one shape (or a batch)")
    ap.add_argument("M", type=int, nargs="?")
    ap.add_argument("N", type=int, nargs="?")
    ap.add_argument("K", type=int, nargs="?")
    ap.add_argument("--dtype", default="float16")
    ap.add_argument("--budget-s", type=float, default=10.0)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--out", help="result file of the one shape")
    ap.add_argument("--batch", help="JSON list of [M, N, K] shapes, each written to --cache-dir as it finishes")
    ap.add_argument("--cache-dir")
    a = ap.parse_args(argv)
    torch.cuda.set_device(a.device)
    if a.batch:
        if not a.cache_dir:
            ap.error("--batch needs --cache-dir")
        for M, N, K in json.loads(Path(a.batch).read_text()):
            path = _cache_path(a.cache_dir, M, N, K, a.dtype, a.budget_s)
            if _cached(path) is None:
                d = search(M, N, K, getattr(torch, a.dtype), a.budget_s, a.top_k)
                path.write_text(json.dumps(d))
        return
    if a.M is None or a.N is None or a.K is None or not a.out:
        ap.error("give M N K and --out, or --batch")
    d = search(a.M, a.N, a.K, getattr(torch, a.dtype), a.budget_s, a.top_k)
    Path(a.out).write_text(json.dumps(d))


if __name__ == "__main__":
    _main()
