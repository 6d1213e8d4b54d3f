"""Per-shape comparison of the sm_100a family with cuBLASLt and torch.matmul (BASELINE.json configs 3 and 4).

For every shape of a suite, on one GPU, with one timing protocol (cold L2, CUDA events, trimmed mean of the samples):
  * `sel`   the family's first-use pick: the ranker's top-k and the zero-search rule's config, validated and
            short-timed, the fastest kept (`search.search_shape` + `choose`), then re-timed with the full protocol;
  * `best`  the family's best-in-pool over a screen of the shape-pruned space (`--space N` configs, 0 = skip);
  * `lt`    cuBLASLt's heuristic top-`lt_n`, each validated and timed: `lt0` = rank 0 (B2), `lt_best` = best (B3);
            with `--lt-deep-s S`, also the fastest configs of a budgeted search of cuBLASLt's configuration space
            (`cublaslt_deep`, S seconds per shape in a child process): `lt_best` is then B3+;
  * `torch` torch.matmul (B1).
The row's `gap_sel_vs_lt` = sel / lt_best - 1 and `gap_sel_vs_best` = sel / best - 1 (the reference's regret,
results/README.md:79); the summary gives their median and p95.

    python -m cs464_b200.compare --suite config3 [--limit N] [--k 3] [--space 0] [--lt-n 16] [--lt-deep-s 5]
                                 [--out rows.jsonl]
"""
from __future__ import annotations

import argparse
import json
import math
import sys
import time

import torch

from cs464_b200 import cublaslt, suites
from cs464_b200.baselines import TorchMatmul
from cs464_b200.gate import make_inputs, reference, validate
from cs464_b200.keys import parse_key
from cs464_b200.matmul import B200Matmul
from cs464_b200.search import choose, measure, screen_shape, selection_keys, shape_space
from cs464_b200.timing import Protocol, measure_us

FULL = Protocol(mode="cold", samples=20, max_samples=100, warmup=3, ci_target=0.01, max_s=1.0)


def _time(backend, a, b) -> float:
    return measure_us(backend.make_runner(a, b), FULL, keep_samples=False).trimmed_us


def compare_shape(shape: dict, *, k: int = 3, space: int = 0, lt_n: int = 16, ranker=None, lt_deep_s: float = 0.0,
                  deep_cache: str = "lt_deep_cache") -> dict:
    M, N, K = shape["M"], shape["N"], shape["K"]
    dtype = torch.float16
    a, b = make_inputs(M, N, K, dtype, scale_b=shape.get("weight_std", 1.0))
    ref = reference(a, b)
    flops = 2.0 * M * N * K
    byts = 2.0 * (M * K + K * N + M * N)
    row = {"M": M, "N": N, "K": K, **{x: shape[x] for x in ("suite", "layer") if x in shape}}
    t0 = time.perf_counter()
    if ranker is None:
        from cs464_b200.search import _ranker_default
        ranker = _ranker_default()
    keys = selection_keys(ranker, M, N, K, k)
    sel = measure(M, N, K, dtype, [("b200_sm100a_v1", x, B200Matmul(parse_key(x))) for x in keys], inputs=(a, b, ref))
    choice = choose(sel["candidates"])
    row["select_s"] = time.perf_counter() - t0
    row["sel_key"] = choice.get("key")
    row["sel_us"] = _time(B200Matmul(parse_key(choice["key"])), a, b) if choice.get("key") else None
    if space:
        pool = shape_space(M, N, K)
        if space > 0 and space < len(pool):
            step = max(1, len(pool) // space)
            pool = pool[::step][:space]
        have = {c.key() for c in pool}
        pool += [parse_key(x) for x in keys if x not in have]
        scr = screen_shape(M, N, K, pool, inputs=(a, b, ref))
        if scr["best_key"]:
            row["best_key"] = scr["best_key"]
            row["best_us"] = min(_time(B200Matmul(parse_key(scr["best_key"])), a, b), row["sel_us"] or math.inf)
    lts = []
    for c in cublaslt.candidates(M, N, K, dtype, lt_n):
        if validate(c, M, N, K, dtype, ref=ref, inputs=(a, b), norm_rel=True).valid:
            lts.append((c.rank, _time(c, a, b)))
    if lt_deep_s > 0:
        from cs464_b200 import cublaslt_deep
        res = cublaslt_deep.search_isolated(M, N, K, deep_cache, budget_s=lt_deep_s)
        row["lt_deep"] = {x: res.get(x) for x in ("n_timed", "n_seeds", "exhausted", "error")}
        for c in cublaslt_deep.backends(res, dtype):
            if validate(c, M, N, K, dtype, ref=ref, inputs=(a, b), norm_rel=True).valid:
                lts.append((100 + c.rank, _time(c, a, b)))
    if lts:
        row["lt0_us"] = dict(lts).get(0)
        row["lt_best_us"] = min(t for _, t in lts)
        row["lt_n_valid"] = len(lts)
    row["torch_us"] = _time(TorchMatmul(), a, b)
    for name in ("sel", "best", "lt_best", "torch"):
        t = row.get(f"{name}_us")
        if t:
            row[f"{name}_tflops"] = flops / t / 1e6
            row[f"{name}_gbs"] = byts / t / 1e3
    if row.get("sel_us") and row.get("lt_best_us"):
        row["gap_sel_vs_lt"] = row["sel_us"] / row["lt_best_us"] - 1.0
    if row.get("sel_us") and row.get("best_us"):
        row["gap_sel_vs_best"] = row["sel_us"] / row["best_us"] - 1.0
    if row.get("best_us") and row.get("lt_best_us"):
        row["gap_best_vs_lt"] = row["best_us"] / row["lt_best_us"] - 1.0
    return row


def _pct(xs: list[float], p: float):
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(round(p / 100 * (len(xs) - 1))))] if xs else None


def summarize(rows: list[dict]) -> dict:
    out = {"shapes": len(rows)}
    for g in ("gap_sel_vs_lt", "gap_sel_vs_best", "gap_best_vs_lt"):
        xs = [r[g] for r in rows if r.get(g) is not None]
        if xs:
            out[g] = {"median": _pct(xs, 50), "p95": _pct(xs, 95), "max": max(xs), "n": len(xs)}
    return out


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--suite", default="config3")
    ap.add_argument("--limit", type=int, default=None)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--space", type=int, default=0)
    ap.add_argument("--lt-n", type=int, default=16)
    ap.add_argument("--lt-deep-s", type=float, default=0.0, help="cuBLASLt configuration search budget per shape")
    ap.add_argument("--deep-cache", default="lt_deep_cache")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    shapes = suites.load(a.suite)[: a.limit]
    if a.lt_deep_s > 0:  # one child process searches cuBLASLt's space for every shape first (cached per shape)
        from cs464_b200 import cublaslt_deep
        cublaslt_deep.search_batch_isolated([(s["M"], s["N"], s["K"]) for s in shapes], a.deep_cache,
                                            budget_s=a.lt_deep_s)
    rows = []
    for s in shapes:
        r = compare_shape(s, k=a.k, space=a.space, lt_n=a.lt_n, lt_deep_s=a.lt_deep_s, deep_cache=a.deep_cache)
        rows.append(r)
        print(json.dumps(r), flush=True)
        if a.out:
            with open(a.out, "a") as f:
                f.write(json.dumps(r) + "\n")
    summary = summarize(rows)
    print(json.dumps({"summary": summary, "suite": a.suite, "k": a.k, "space": a.space, "lt_n": a.lt_n,
                      "lt_deep_s": a.lt_deep_s}), flush=True)
    return summary


if __name__ == "__main__":
    main()
    sys.exit(0)
