"""Candidate expansion, first-use selection and the full-space screen for the sm_100a family.

Mirrors the reference's callers of its GEMM family:
  * `candidates_for(spec, M, N, K)`: backend spec strings -> `Candidate`s (tune/runner.py:42-142); specs here:
    `b200:handpicked`, `b200:heuristic`, `b200:rank[:k]`, `b200:space[:n]`, `b200:<config key>`, `torch` (B1).
  * `measure`: validate, then short-time each candidate on one placement; a burst-amortised pass when the fastest
    cold time is under 50 us, a sustained pass (under the power cap's settled clock) when the fastest is 1 ms or
    more; optional reverse-order confirmation (tune/online.py:244-329).
  * `choose` (tune/online.py:125-138), `search_shape` (:332-363), `select_kernel` with the winner cache and the
    call-count k policy (:58-77, :379-483).
  * `screen_shape`: times every statically and shape-pruned config with the reference's stage-1 rule (one cold sample;
    cut at 1.5x the best so far; else more samples) (tune/sweep.py:216-274). This is best-in-pool for the selector's
    gap metric.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass

import torch

from cs464_b200.config_space import HANDPICKED, HwLimits, full_space, prune, shape_violations
from cs464_b200.gate import ContextPoisoned, context_poisoned, make_inputs, reference, validate
from cs464_b200.keys import parse_key
from cs464_b200.matmul import B200Matmul, MatmulConfig
from cs464_b200.timing import LONG_US, SHORT_BURST, SHORT_COLD, SMALL_US, Protocol, measure_us, sustained

FAMILY = B200Matmul.family
DTYPE_NAMES = {torch.float16: "fp16", torch.bfloat16: "bf16"}
SLOW_FACTOR = 1.5
SCREEN_SAMPLES = 15


@dataclass
class Candidate:
    family: str
    config_key: str
    config: dict
    backend: object


@dataclass(frozen=True)
class KPolicy:
    """k = candidates to time for a new shape; shapes the caller expects to launch often get k_frequent."""
    k: int = 3
    k_frequent: int = 5
    frequent_calls: int = 1_000_000

    def k_for(self, calls: int | None = None, frequent: bool | None = None) -> int:
        if frequent or (calls is not None and calls >= self.frequent_calls):
            return self.k_frequent
        return self.k


_SPACE_CACHE: dict = {}


def pruned_space(hw: HwLimits | None = None) -> list[MatmulConfig]:
    hw = hw or HwLimits.b200()
    if hw not in _SPACE_CACHE:
        _SPACE_CACHE[hw] = prune(full_space(), hw)[0]
    return _SPACE_CACHE[hw]


SOFT_RULES = ("block_m_oversized", "block_n_oversized", "block_k_oversized", "group_m_noop")


def shape_space(M: int, N: int, K: int, hw: HwLimits | None = None) -> list[MatmulConfig]:
    """Every statically kept config with no shape-rule violation for (M, N, K). When every config breaks a rule (a
    dimension smaller than the smallest tile, e.g. N = 16), the tile-oversize rules are treated as soft: the configs
    that break only those and overshoot the least are kept, so no shape is left without a candidate."""
    pool = pruned_space(hw)
    out = [c for c in pool if not shape_violations(c, M, N, K)]
    if out:
        return out
    soft = [c for c in pool if all(r in SOFT_RULES for r in shape_violations(c, M, N, K))]
    if not soft:
        return []

    def overshoot(c: MatmulConfig) -> tuple:
        return (c.BLOCK_M / max(M, 1) + c.BLOCK_N / max(N, 1) + c.BLOCK_K / max(K, 1), c.key())
    best = min(overshoot(c)[0] for c in soft)
    return [c for c in soft if overshoot(c)[0] <= best * 1.5]


_DEFAULT_RANKER = None


def _ranker_default():
    global _DEFAULT_RANKER
    if _DEFAULT_RANKER is None:
        from cs464_b200.ranker import default_ranker
        _DEFAULT_RANKER = default_ranker()
    return _DEFAULT_RANKER


def candidates_for(spec: str, M: int, N: int, K: int, prune_shapes: bool = False, ranker=None) -> list[Candidate]:
    from cs464_b200.baselines import TorchMatmul
    from cs464_b200.select import heuristic_config
    if spec == "torch":
        b = TorchMatmul()
        return [Candidate(b.family, "default", {}, b)]
    if not spec.startswith("b200:"):
        raise ValueError(f"unknown backend spec {spec!r}")
    which = spec.split(":", 1)[1]
    extra: dict[str, dict] = {}
    if which == "handpicked":
        cfgs = list(HANDPICKED.values())
    elif which == "heuristic":
        cfgs = [heuristic_config(M, N, K)]
    elif which == "rank" or which.startswith("rank:"):
        k = int(which.split(":", 1)[1]) if ":" in which else 3
        r = ranker or _ranker_default()
        keys = r.rank(M, N, K, k, order="diverse")
        cfgs = [parse_key(x) for x in keys]
        extra = {x: {"rank": i} for i, x in enumerate(keys)}
    elif which == "space" or which.startswith("space:"):
        cfgs = shape_space(M, N, K)
        if ":" in which:
            n = int(which.split(":", 1)[1])
            step = max(1, len(cfgs) // max(n, 1))
            cfgs = cfgs[::step][:n]
    else:
        cfgs = [c for c in HANDPICKED.values() if c.key() == which] or [parse_key(which)]
    out = []
    for c in cfgs:
        v = shape_violations(c, M, N, K)
        if "split_k_workspace_too_large" in v or (prune_shapes and v):
            continue
        out.append(Candidate(FAMILY, c.key(), {**c.to_dict(), **extra.get(c.key(), {})}, B200Matmul(c)))
    return out


def measure(M: int, N: int, K: int, dtype, backends: list[tuple], *, inputs=None, confirm: int = 0,
            norm_rel: bool = True, skip=(), on_config=None) -> dict:
    """Validate then short-time each (family, key, backend) on one placement; returns {"candidates": [...]}.
    Keys in `skip` (configs that crashed an earlier process on this shape) are recorded invalid without running;
    `on_config(key)` is called before each candidate runs (the sharded search's in-flight record)."""
    if inputs is None:
        a, b = make_inputs(M, N, K, dtype)
        ref = reference(a, b)
    else:
        a, b, ref = inputs
    cands, bk = [], {}
    for family, key, backend in backends:
        if key in skip:
            cands.append({"config_key": key, "family": family, "valid": False, "failure_reason": "crashed",
                          "setup_s": 0.0})
            continue
        if on_config is not None:
            on_config(key)
        t = time.perf_counter()
        chk = validate(backend, M, N, K, dtype, ref=ref, inputs=(a, b), norm_rel=norm_rel)
        if context_poisoned(chk.failure_reason):
            raise ContextPoisoned(f"{family}:{key}", chk.failure_reason)
        torch.cuda.synchronize()
        x = {"config_key": key, "family": family, "valid": chk.valid, "failure_reason": chk.failure_reason,
             "setup_s": time.perf_counter() - t}
        if chk.valid:
            t = time.perf_counter()
            x["cold_us"] = measure_us(backend.make_runner(a, b), SHORT_COLD, keep_samples=False).median_us
            x["time_s"] = time.perf_counter() - t
        cands.append(x)
        bk[key] = backend
    ok = [x for x in cands if x["valid"]]
    if ok and min(x["cold_us"] for x in ok) < SMALL_US:
        for x in ok:
            t = time.perf_counter()
            x["burst_us"] = measure_us(bk[x["config_key"]].make_runner(a, b), SHORT_BURST,
                                       keep_samples=False).median_us
            x["time_s"] += time.perf_counter() - t
    elif ok and min(x["cold_us"] for x in ok) >= LONG_US:
        for x in ok:
            t = time.perf_counter()
            x["sustained_us"] = measure_us(bk[x["config_key"]].make_runner(a, b), sustained(x["cold_us"]),
                                           keep_samples=False).median_us
            x["time_s"] += time.perf_counter() - t
    if confirm > 0 and ok:
        metric = _metric(ok)
        proto = {"burst_us": lambda x: SHORT_BURST, "cold_us": lambda x: SHORT_COLD,
                 "sustained_us": lambda x: sustained(x["cold_us"])}[metric]
        for x in reversed(sorted(ok, key=lambda x: x[metric])[:confirm]):
            t = time.perf_counter()
            again = measure_us(bk[x["config_key"]].make_runner(a, b), proto(x), keep_samples=False).median_us
            x["confirm_us"] = 0.5 * (x[metric] + again)
            x["time_s"] += time.perf_counter() - t
        for x in ok:
            x.setdefault("confirm_us", x[metric])
    return {"candidates": cands}


def _metric(ok: list[dict]) -> str:
    """The time a set of valid candidates is compared by: burst time when every one has it (the fastest cold time
    was under SMALL_US), sustained time when every one has it (the fastest was LONG_US or more), else cold time."""
    if all(x.get("burst_us") is not None for x in ok) and min(x["cold_us"] for x in ok) < SMALL_US:
        return "burst_us"
    if all(x.get("sustained_us") is not None for x in ok):
        return "sustained_us"
    return "cold_us"


def choose(cands: list[dict], k: int | None = None) -> dict:
    """Fastest valid candidate among the first k (all for None), by `_metric`'s time; `confirm_us` overrides when
    present."""
    c = cands if k is None else cands[:k]
    ok = [x for x in c if x["valid"] and x.get("cold_us") is not None]
    cost = {"setup_s": sum(x.get("setup_s", 0.0) for x in c), "time_s": sum(x.get("time_s", 0.0) for x in c)}
    if not ok:
        return {"key": None, "mode": None, **cost}
    metric = _metric(ok)
    best = min(ok, key=lambda x: x.get("confirm_us", x[metric]))
    return {"key": best["config_key"], "family": best.get("family", FAMILY), "rank": c.index(best),
            "mode": metric[:-3], "us": best.get("confirm_us", best[metric]), **cost}


def selection_keys(ranker, M: int, N: int, K: int, k: int, order: str = "diverse") -> list[str]:
    """The configs a first-use selection times: the ranker's top k and the zero-search rule's config (when it is not
    among them). The rule covers what the ranker's training data predates (e.g. decode split counts whose clusters fit
    the GPU at once)."""
    from cs464_b200.select import heuristic_config
    ranker = ranker or _ranker_default()
    return list(dict.fromkeys(list(ranker.rank(M, N, K, k, order=order)) + [heuristic_config(M, N, K).key()]))


def search_shape(ranker, M: int, N: int, K: int, k: int, dtype=torch.float16, order: str = "diverse",
                 confirm: int = 0) -> dict:
    """Rank, then validate + short-time the top k and the zero-search rule's config."""
    t0 = time.perf_counter()
    keys = selection_keys(ranker, M, N, K, k, order=order)
    rank_s = time.perf_counter() - t0
    backends = [(FAMILY, key, B200Matmul(parse_key(key))) for key in keys]
    r = measure(M, N, K, dtype, backends, confirm=confirm)
    return {"rank_s": rank_s, "candidates": r["candidates"]}


def select_kernel(ranker, M: int, N: int, K: int, *, calls: int | None = None, frequent: bool | None = None,
                  policy: KPolicy = KPolicy(), dtype=torch.float16, cache=True, confirm: int = 0,
                  serve_stale: bool = False, extra=None) -> dict:
    """First-use selection for one shape: a cached winner from a search at least this wide is returned without any
    GPU work; otherwise the ranker's top k and the zero-search rule's config are validated and timed, the fastest is
    stored and returned.
    Returns {"k", "reason", "choice", "candidates", "rank_s", "cached"}."""
    import warnings

    from cs464_b200.winner_cache import WinnerCache, backend_for, default_enabled
    k = policy.k_for(calls, frequent)
    dname = DTYPE_NAMES[dtype]
    wc = None
    if cache is True and default_enabled():
        try:
            wc = WinnerCache()
        except Exception as e:
            warnings.warn(f"winner cache unavailable ({type(e).__name__}: {e}); searching without it")
    elif cache not in (None, False, True):
        wc = cache
    if wc is not None:
        try:
            wc.refresh()
            hit = wc.get(M, N, K, dname, k=k, allow_stale=serve_stale)
            if hit is not None and backend_for(hit["choice"]) is not None:
                if not hit["stale"] or validate(backend_for(hit["choice"]), M, N, K, dtype).valid:
                    return {"k": hit["k"], "reason": "cached_stale" if hit["stale"] else "cached", "rank_s": 0.0,
                            "choice": hit["choice"], "candidates": [], "cached": True, "stale": hit["stale"]}
        except Exception as e:
            warnings.warn(f"winner cache lookup failed ({type(e).__name__}: {e}); searching")
    r = search_shape(ranker, M, N, K, k, dtype, confirm=confirm)
    choice = choose(r["candidates"])
    reason = "frequent" if k == policy.k_frequent and k != policy.k else "default"
    if wc is not None and choice.get("key") is not None:
        try:
            wc.put(M, N, K, dname, k=k, choice=choice, candidates=r["candidates"],
                   extra=extra() if callable(extra) else extra)
        except Exception as e:
            warnings.warn(f"winner cache write failed ({type(e).__name__}: {e})")
    return {"k": k, "reason": reason, "rank_s": r["rank_s"], "cached": False, "choice": choice,
            "candidates": r["candidates"]}


def screen_shape(M: int, N: int, K: int, configs: list[MatmulConfig] | None = None, dtype=torch.float16, *,
                 slow_factor: float = SLOW_FACTOR, samples: int = SCREEN_SAMPLES, inputs=None,
                 log=None, skip=(), on_config=None) -> dict:
    """Time every config (default: the shape-pruned space) with early cut-off. Each config: validate; one cold sample
    (its median of `1` after warm-up); cut as "slow" if above slow_factor x the best so far; else `samples` cold samples,
    summarised by their trimmed mean: per-launch event timestamps on this GPU fall on a ~1 us grid, so the median of a
    few samples of a 10 us kernel moves in 10 % steps, while the mean of the middle samples resolves finer.
    Keys in `skip` are recorded "invalid: crashed" without running; `on_config(key)` runs before each config.
    Returns {"rows": [{key, status, us, n}], "best_key", "best_us", "n_configs", "wall_s"}."""
    t0 = time.perf_counter()
    cfgs = configs if configs is not None else shape_space(M, N, K)
    if inputs is None:
        a, b = make_inputs(M, N, K, dtype)
        ref = reference(a, b)
    else:
        a, b, ref = inputs
    one = Protocol(mode="cold", samples=1, max_samples=1, warmup=1, ci_target=math.inf, max_s=1.0)
    more = Protocol(mode="cold", samples=samples, max_samples=samples, warmup=0, ci_target=math.inf, max_s=2.0)
    rows, best = [], math.inf
    for c in cfgs:
        if c.key() in skip:
            rows.append({"key": c.key(), "status": "invalid: crashed", "us": None, "n": 0})
            continue
        if on_config is not None:
            on_config(c.key())
        be = B200Matmul(c)
        chk = validate(be, M, N, K, dtype, ref=ref, inputs=(a, b), norm_rel=True)
        if context_poisoned(chk.failure_reason):
            raise ContextPoisoned(c.key(), chk.failure_reason)
        if not chk.valid:
            rows.append({"key": c.key(), "status": f"invalid: {chk.failure_reason}", "us": None, "n": 0})
            continue
        run = be.make_runner(a, b)
        us = measure_us(run, one, keep_samples=False).median_us
        if us > slow_factor * best:
            rows.append({"key": c.key(), "status": "slow", "us": us, "n": 1})
            continue
        us = measure_us(run, more, keep_samples=False).trimmed_us
        best = min(best, us)
        rows.append({"key": c.key(), "status": "ok", "us": us, "n": samples})
        if log:
            log(f"{c.key()}: {us:.2f} us")
    ok = [r for r in rows if r["status"] == "ok"]
    b = min(ok, key=lambda r: r["us"]) if ok else None
    return {"M": M, "N": N, "K": K, "rows": rows, "n_configs": len(cfgs), "best_key": b["key"] if b else None,
            "best_us": b["us"] if b else None, "wall_s": time.perf_counter() - t0}
