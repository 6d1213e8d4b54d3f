"""Candidate ranking for the online search: which configs of the sm_100a space to time for a new shape.

The reference ranks its Triton pool with a LightGBM model over config and shape features (analysis/learned.py:461-535,
features analysis/selectors.py:130-151 and analysis/learned.py:264-285, with RTX 3080 roofline constants at :242). Its
models rank Triton keys, so they cannot rank this family; lightgbm is not installed here either. This module keeps
the ranker interface (`rank(M, N, K, k, order)`, `scores`, `cfgs`, `pool_keys`, `load`) with two rankers:
  * `AnalyticRanker`: a roofline model of this kernel on B200 (waves over 148 SMs, tensor time per tile, L2->SM and
    HBM bytes, per-K-step issue overhead, split-K and staging costs); needs no training data;
  * `LearnedRanker`: gradient-boosted trees (scikit-learn) over the same features, fitted on measured screens of
    this family on B200 (`fit(rows)`), saved as <stem>.trees.npz (the trees as plain arrays, scored natively) +
    <stem>.json.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

from cs464_b200.config_space import HwLimits, full_space, mma_tile, prune, shape_violations, smem_bytes, swapped
from cs464_b200.matmul import MatmulConfig

# B200 model constants (per GPU, as measured on this pool: MEASURED_PEAKS.json)
PEAK_FLOPS = 1.63e15
HBM_BPS = 6.55e12
SM_COUNT = 148
CLOCK_HZ = 1.85e9
L2_BYTES_PER_CLK_PER_SM = 64.0   # TMA fill rate of one SM measured on B200 (~16 KB box per 256 clocks)
# The per-K-block cost and the launch/fix-up costs below are fitted (grid search, top-3 regret) to a screen of the 200
# config-3 shapes x ~385 configs on B200.
KBLOCK_OVERHEAD_CLK = 250.0
LAUNCH_S = 4.5e-6                 # fixed cost of one launch of this kernel (prologue, first copy, drain)
EXTRA_KERNEL_S = 5.0e-6           # the split-K reduce or an operand-staging kernel
CLUSTER_LAUNCH_S = 2.0e-6
STREAMK_FIXUP_S = 15.0e-6


def config_params(cfg: MatmulConfig) -> dict:
    """The tunables as numbers (the reference's config_params, analysis/learned.py:75-79, plus the new knobs)."""
    return {k: float(v) for k, v in cfg.to_dict().items()}


def _geometry(M: int, N: int, K: int, cfg: MatmulConfig) -> dict:
    tm, tn = mma_tile(cfg)
    rows_a, rows_b = (N, M) if swapped(cfg) else (M, N)
    tiles_m = -(-rows_a // tm)
    tiles_n = -(-rows_b // tn)
    nkb = max(1, -(-K // cfg.BLOCK_K))
    split = cfg.SPLIT_K
    units = tiles_m * tiles_n * split
    sms_per_unit = 2 if cfg.CLUSTER == 2 else 1
    slots = SM_COUNT // sms_per_unit if cfg.PERSISTENT else units
    waves = units / max(1, SM_COUNT // sms_per_unit)
    return {"tm": tm, "tn": tn, "rows_a": rows_a, "rows_b": rows_b, "tiles_m": tiles_m, "tiles_n": tiles_n,
            "nkb": nkb, "kb_per_unit": -(-nkb // split), "units": units, "sms_per_unit": sms_per_unit,
            "slots": slots, "waves": waves, "fill_m": rows_a / (tiles_m * tm), "fill_n": rows_b / (tiles_n * tn)}


def analytic_time_s(M: int, N: int, K: int, cfg: MatmulConfig) -> float:
    """Predicted kernel time of `cfg` on a row-major (M, N, K) problem (seconds)."""
    g = _geometry(M, N, K, cfg)
    per_sm_flops_clk = PEAK_FLOPS / SM_COUNT / CLOCK_HZ
    # tensor work of one K block on one SM (a pair splits the tile's rows over two SMs)
    mma_n_eff = min(1.0, g["tn"] / 64.0) ** 0.5  # narrow N wastes tensor issue slots
    kb_flops = 2.0 * g["tm"] * g["tn"] * cfg.BLOCK_K / g["sms_per_unit"]
    t_mma = kb_flops / (per_sm_flops_clk * max(mma_n_eff, 0.25))
    kb_bytes = (g["tm"] + g["tn"]) * cfg.BLOCK_K * 2.0 / g["sms_per_unit"]
    t_load = kb_bytes / L2_BYTES_PER_CLK_PER_SM
    per_kb = max(t_mma, t_load) + KBLOCK_OVERHEAD_CLK
    # pipeline latency cover: a shallow ring stalls on load latency
    ring_clk = cfg.num_stages * max(t_mma, t_load)
    per_kb += max(0.0, 2500.0 - ring_clk) / cfg.num_stages
    unit_clk = g["kb_per_unit"] * per_kb
    acc_cols = g["tn"] if cfg.CLUSTER == 2 else (g["tm"] // 128) * g["tn"]
    epi_clk = g["tm"] * g["tn"] * (2.0 if cfg.SPLIT_K == 1 else 4.0) / g["sms_per_unit"] / (16.0 * cfg.num_warps)
    if 2 * acc_cols > 512:  # single accumulator: the epilogue does not overlap the next tile's main loop
        unit_clk += epi_clk
    if cfg.PERSISTENT == 2:  # stream-K: every worker gets an equal share of the K blocks of all tiles
        workers = max(1, SM_COUNT // g["sms_per_unit"])
        iters = g["tiles_m"] * g["tiles_n"] * g["nkb"]
        share = math.ceil(iters / min(workers, iters))
        tiles_per_worker = math.ceil(g["tiles_m"] * g["tiles_n"] / min(workers, iters))
        t = (share * per_kb + tiles_per_worker * (epi_clk if 2 * acc_cols > 512 else 0.0)) / CLOCK_HZ
        t += epi_clk / CLOCK_HZ + STREAMK_FIXUP_S
    else:
        waves = math.ceil(g["units"] / max(1, g["slots"])) if cfg.PERSISTENT else math.ceil(g["waves"])
        t = waves * unit_clk / CLOCK_HZ + (0.0 if 2 * acc_cols > 512 else epi_clk / CLOCK_HZ)
    # DRAM floor: compulsory operand bytes (B re-read per tile row group is assumed to hit L2)
    dram = 2.0 * (M * K + K * N + M * N)
    if cfg.SPLIT_K > 1:
        dram += 4.0 * cfg.SPLIT_K * M * N * 2 + 2.0 * M * N
    t = max(t, dram / HBM_BPS)
    t += LAUNCH_S + (EXTRA_KERNEL_S if cfg.SPLIT_K > 1 else 0.0) + (CLUSTER_LAUNCH_S if cfg.CLUSTER == 2 else 0.0)
    return t


def candidate_features(M: int, N: int, K: int, cfg: MatmulConfig) -> dict:
    """Shape + config + derived features (tile fill, waves, per-unit work, analytic terms), all numeric."""
    g = _geometry(M, N, K, cfg)
    f = {"log2_M": math.log2(M), "log2_N": math.log2(N), "log2_K": math.log2(K),
         "log2_MNK": math.log2(M) + math.log2(N) + math.log2(K), **config_params(cfg),
         "swapped": float(swapped(cfg)), "smem_kib": smem_bytes(cfg) / 1024.0, "fill_m": g["fill_m"],
         "fill_n": g["fill_n"], "waves": g["waves"], "waves_frac": g["waves"] - math.floor(g["waves"]),
         "log2_units": math.log2(g["units"]), "kb_per_unit": float(g["kb_per_unit"]),
         "log_analytic_us": math.log(analytic_time_s(M, N, K, cfg) * 1e6),
         "log_dram_floor_us": math.log(2.0 * (M * K + K * N + M * N) / HBM_BPS * 1e6 + 1e-3),
         "log_tensor_floor_us": math.log(2.0 * M * N * K / PEAK_FLOPS * 1e6 + 1e-3)}
    return f


FEATURES = list(candidate_features(64, 64, 64, MatmulConfig(128, 128, 64)).keys())


class _Pool:
    """Per-config arrays of a pool, so a shape's features and analytic times are computed for all configs at once."""

    def __init__(self, cfgs: list[MatmulConfig]):
        self.cfgs = cfgs
        f = lambda name: np.array([getattr(c, name) for c in cfgs], dtype=np.float64)  # noqa: E731
        self.params = {name: f(name) for name in ("BLOCK_M", "BLOCK_N", "BLOCK_K", "num_warps", "num_stages",
                                                   "GROUP_M", "SPLIT_K", "PERSISTENT", "CLUSTER")}
        self.swapped = (self.params["BLOCK_M"] <= 64).astype(np.float64)
        self.tm = np.where(self.swapped > 0, self.params["BLOCK_N"], self.params["BLOCK_M"])
        self.tn = np.where(self.swapped > 0, self.params["BLOCK_M"], self.params["BLOCK_N"])
        self.smem_kib = np.array([smem_bytes(c) for c in cfgs], dtype=np.float64) / 1024.0
        self.spu = np.where(self.params["CLUSTER"] == 2, 2.0, 1.0)

    def analytic_log_us(self, M: int, N: int, K: int) -> np.ndarray:
        return np.log(self.analytic_s(M, N, K) * 1e6)

    def geometry(self, M: int, N: int, K: int) -> dict:
        P = self.params
        rows_a = np.where(self.swapped > 0, N, M).astype(np.float64)
        rows_b = np.where(self.swapped > 0, M, N).astype(np.float64)
        tiles_m = np.ceil(rows_a / self.tm)
        tiles_n = np.ceil(rows_b / self.tn)
        nkb = np.maximum(1.0, np.ceil(K / P["BLOCK_K"]))
        units = tiles_m * tiles_n * P["SPLIT_K"]
        slots_all = np.floor(SM_COUNT / self.spu)
        slots = np.where(P["PERSISTENT"] > 0, slots_all, units)
        return {"rows_a": rows_a, "rows_b": rows_b, "tiles_m": tiles_m, "tiles_n": tiles_n, "nkb": nkb,
                "kb_per_unit": np.ceil(nkb / P["SPLIT_K"]), "units": units, "slots": slots,
                "waves": units / np.maximum(1.0, slots_all), "fill_m": rows_a / (tiles_m * self.tm),
                "fill_n": rows_b / (tiles_n * self.tn)}

    def analytic_s(self, M: int, N: int, K: int) -> np.ndarray:
        """Vectorised `analytic_time_s` over the pool (same model, same constants)."""
        P, g = self.params, self.geometry(M, N, K)
        per_sm = PEAK_FLOPS / SM_COUNT / CLOCK_HZ
        eff = np.maximum(np.minimum(1.0, self.tn / 64.0) ** 0.5, 0.25)
        t_mma = 2.0 * self.tm * self.tn * P["BLOCK_K"] / self.spu / (per_sm * eff)
        t_load = (self.tm + self.tn) * P["BLOCK_K"] * 2.0 / self.spu / L2_BYTES_PER_CLK_PER_SM
        per_kb = np.maximum(t_mma, t_load) + KBLOCK_OVERHEAD_CLK
        per_kb = per_kb + np.maximum(0.0, 2500.0 - P["num_stages"] * np.maximum(t_mma, t_load)) / P["num_stages"]
        unit_clk = g["kb_per_unit"] * per_kb
        acc_cols = np.where(P["CLUSTER"] == 2, self.tn, np.floor(self.tm / 128) * self.tn)
        single = 2 * acc_cols > 512
        epi = self.tm * self.tn * np.where(P["SPLIT_K"] == 1, 2.0, 4.0) / self.spu / (16.0 * P["num_warps"])
        unit_clk = unit_clk + np.where(single, epi, 0.0)
        workers = np.maximum(1.0, np.floor(SM_COUNT / self.spu))
        iters = g["tiles_m"] * g["tiles_n"] * g["nkb"]
        share = np.ceil(iters / np.minimum(workers, iters))
        tpw = np.ceil(g["tiles_m"] * g["tiles_n"] / np.minimum(workers, iters))
        t_sk = (share * per_kb + tpw * np.where(single, epi, 0.0)) / CLOCK_HZ + epi / CLOCK_HZ + STREAMK_FIXUP_S
        waves = np.where(P["PERSISTENT"] > 0, np.ceil(g["units"] / np.maximum(1.0, g["slots"])), np.ceil(g["waves"]))
        t_pt = waves * unit_clk / CLOCK_HZ + np.where(single, 0.0, epi / CLOCK_HZ)
        t = np.where(P["PERSISTENT"] == 2, t_sk, t_pt)
        dram = 2.0 * (M * K + K * N + M * N) + np.where(P["SPLIT_K"] > 1, 4.0 * P["SPLIT_K"] * M * N * 2 + 2.0 * M * N,
                                                        0.0)
        t = np.maximum(t, dram / HBM_BPS)
        return (t + LAUNCH_S + np.where(P["SPLIT_K"] > 1, EXTRA_KERNEL_S, 0.0)
                + np.where(P["CLUSTER"] == 2, CLUSTER_LAUNCH_S, 0.0))

    def features(self, M: int, N: int, K: int) -> np.ndarray:
        """The `candidate_features` matrix (rows = configs, columns = FEATURES)."""
        g = self.geometry(M, N, K)
        n = len(self.cfgs)
        col = {"log2_M": np.full(n, math.log2(M)), "log2_N": np.full(n, math.log2(N)),
               "log2_K": np.full(n, math.log2(K)), "log2_MNK": np.full(n, math.log2(M) + math.log2(N) + math.log2(K)),
               **self.params, "swapped": self.swapped, "smem_kib": self.smem_kib, "fill_m": g["fill_m"],
               "fill_n": g["fill_n"], "waves": g["waves"], "waves_frac": g["waves"] - np.floor(g["waves"]),
               "log2_units": np.log2(g["units"]), "kb_per_unit": g["kb_per_unit"],
               "log_analytic_us": self.analytic_log_us(M, N, K),
               "log_dram_floor_us": np.full(n, math.log(2.0 * (M * K + K * N + M * N) / HBM_BPS * 1e6 + 1e-3)),
               "log_tensor_floor_us": np.full(n, math.log(2.0 * M * N * K / PEAK_FLOPS * 1e6 + 1e-3))}
        return np.stack([col[f] for f in FEATURES], axis=1)


class AnalyticRanker:
    """Ranks the statically pruned space by the analytic time model (lower = better)."""

    kind = "analytic"

    def __init__(self, pool: list[MatmulConfig] | None = None, hw: HwLimits | None = None):
        self.hw = hw or HwLimits.b200()
        self.cfgs = pool if pool is not None else prune(full_space(), self.hw)[0]
        self.pool_keys = [c.key() for c in self.cfgs]
        self._pool = _Pool(self.cfgs) if self.cfgs else None
        self.stem = None

    def scores(self, M: int, N: int, K: int) -> np.ndarray:
        if self._pool is None:
            return np.zeros(0)
        return self._pool.analytic_log_us(M, N, K)

    def rank(self, M: int, N: int, K: int, k: int, order: str = "plain") -> list[str]:
        """Top-k keys among configs with no shape violation. "diverse" takes at most one config per tile
        (BLOCK_M, BLOCK_N, BLOCK_K, SPLIT_K, CLUSTER) before repeating any tile."""
        s = self.scores(M, N, K)
        idx = [i for i in np.argsort(s, kind="stable") if not shape_violations(self.cfgs[i], M, N, K)]
        if not idx:  # every config overshoots a tiny dimension: rank the least-oversized ones
            from cs464_b200.search import shape_space
            allowed = {c.key() for c in shape_space(M, N, K)}
            idx = [i for i in np.argsort(s, kind="stable") if self.pool_keys[i] in allowed]
        if order == "plain":
            return [self.pool_keys[i] for i in idx[:k]]
        out, seen, rest = [], set(), []
        for i in idx:
            c = self.cfgs[i]
            tile = (c.BLOCK_M, c.BLOCK_N, c.BLOCK_K, c.SPLIT_K, c.CLUSTER)
            if tile in seen:
                rest.append(i)
                continue
            seen.add(tile)
            out.append(i)
            if len(out) == k:
                break
        out += rest[: k - len(out)]
        return [self.pool_keys[i] for i in out]


class Forest:
    """A regression tree ensemble as plain arrays, scored by the library's native predictor (`b2g_forest_predict`):
    the shipped model needs neither the training library nor its version. Node n: feature (-1 at a leaf), threshold,
    left / right child (global node indices), missing-value direction, value; roots[t] is tree t's first node."""

    FIELDS = ("feature", "threshold", "left", "right", "missing_left", "value", "roots")

    def __init__(self, feature, threshold, left, right, missing_left, value, roots, base: float):
        self.feature = np.ascontiguousarray(feature, dtype=np.int32)
        self.threshold = np.ascontiguousarray(threshold, dtype=np.float64)
        self.left = np.ascontiguousarray(left, dtype=np.int32)
        self.right = np.ascontiguousarray(right, dtype=np.int32)
        self.missing_left = np.ascontiguousarray(missing_left, dtype=np.uint8)
        self.value = np.ascontiguousarray(value, dtype=np.float64)
        self.roots = np.ascontiguousarray(roots, dtype=np.int32)
        self.base = float(base)

    @classmethod
    def from_sklearn(cls, model) -> "Forest":
        """Flatten a fitted scikit-learn HistGradientBoostingRegressor (numeric features, one output)."""
        parts, roots, off = [], [], 0
        for (pred,) in model._predictors:
            nd = pred.nodes
            if nd["is_categorical"].any():
                raise ValueError("categorical splits are not supported")
            leaf = nd["is_leaf"].astype(bool)
            parts.append((np.where(leaf, -1, nd["feature_idx"]), nd["num_threshold"],
                          np.where(leaf, -1, nd["left"] + off), np.where(leaf, -1, nd["right"] + off),
                          nd["missing_go_to_left"], nd["value"]))
            roots.append(off)
            off += len(nd)
        cols = [np.concatenate([p[i] for p in parts]) for i in range(6)]
        return cls(*cols, roots, float(np.ravel(model._baseline_prediction)[0]))

    def predict(self, X: np.ndarray, threads: int | None = None) -> np.ndarray:
        import ctypes
        import os

        from cs464_b200 import _abi
        X = np.ascontiguousarray(X, dtype=np.float64)
        out = np.empty(X.shape[0], dtype=np.float64)
        ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        n_threads = threads or int(os.environ.get("OMP_NUM_THREADS") or os.cpu_count() or 1)
        rc = _abi.load().b2g_forest_predict(ptr(self.feature), ptr(self.threshold), ptr(self.left), ptr(self.right),
                                            ptr(self.missing_left), ptr(self.value), ptr(self.roots),
                                            len(self.roots), self.base, ptr(X), X.shape[0], X.shape[1], ptr(out),
                                            n_threads)
        _abi.check(rc, "b2g_forest_predict")
        return out

    def save(self, path: str | Path) -> None:
        np.savez_compressed(path, base=np.array([self.base]), **{f: getattr(self, f) for f in self.FIELDS})

    @classmethod
    def load(cls, path: str | Path) -> "Forest":
        z = np.load(path)
        return cls(*(z[f] for f in cls.FIELDS), float(z["base"][0]))


class LearnedRanker(AnalyticRanker):
    """Gradient-boosted trees over `candidate_features`, predicting log(time / best time of the shape). Trained
    with scikit-learn, stored and scored as a `Forest` (<stem>.trees.npz + <stem>.json)."""

    kind = "learned"

    def __init__(self, model=None, pool: list[MatmulConfig] | None = None, hw: HwLimits | None = None):
        super().__init__(pool, hw)
        self.model = model

    def fit(self, rows: list[dict], **kw) -> "LearnedRanker":
        """rows: {"M", "N", "K", "key", "us"} timings of valid candidates (several per shape)."""
        from sklearn.ensemble import HistGradientBoostingRegressor

        from cs464_b200.keys import parse_key
        by_shape: dict[tuple, list[dict]] = {}
        for r in rows:  # timings are compared within a shape (and within the unit / GPU they were taken on)
            by_shape.setdefault((r["M"], r["N"], r["K"], r.get("group")), []).append(r)
        Xs, ys = [], []
        for (M, N, K, _), rs in by_shape.items():
            best = min(r["us"] for r in rs)
            Xs.append(_Pool([parse_key(r["key"]) for r in rs]).features(M, N, K))
            ys.append(np.log(np.array([r["us"] for r in rs]) / best))
        X = np.concatenate(Xs)
        y = np.concatenate(ys)
        params = {"max_iter": 600, "learning_rate": 0.05, "max_leaf_nodes": 63, "random_state": 0}
        params.update(kw)
        self.model = Forest.from_sklearn(HistGradientBoostingRegressor(**params).fit(X, y))
        return self

    def scores(self, M: int, N: int, K: int) -> np.ndarray:
        if self.model is None or self._pool is None:
            return super().scores(M, N, K)
        return self.model.predict(self._pool.features(M, N, K))

    def save(self, stem: str | Path, info: dict | None = None) -> None:
        stem = Path(stem)
        stem.parent.mkdir(parents=True, exist_ok=True)
        self.model.save(f"{stem}.trees.npz")
        Path(f"{stem}.json").write_text(json.dumps({"features": FEATURES, "info": info or {}, "pool": self.pool_keys}))
        self.stem = str(stem)

    @classmethod
    def load(cls, stem: str | Path) -> "LearnedRanker":
        from cs464_b200.keys import parse_key
        meta = json.loads(Path(f"{stem}.json").read_text())
        if meta["features"] != FEATURES:
            raise ValueError(f"{stem}: feature list differs from this version's; retrain")
        r = cls(Forest.load(f"{stem}.trees.npz"), [parse_key(k) for k in meta["pool"]])
        r.stem = str(stem)
        return r


MODEL_STEM = Path(__file__).resolve().parent / "models" / "ranker_b200"


def default_ranker():
    """The shipped learned ranker when its files exist (cs464_b200/models/ranker_b200.{trees.npz,json}), else the analytic
    one. A model whose feature list no longer matches this code is ignored (warned)."""
    if Path(f"{MODEL_STEM}.trees.npz").exists() and Path(f"{MODEL_STEM}.json").exists():
        try:
            return LearnedRanker.load(MODEL_STEM)
        except Exception as e:
            import warnings
            warnings.warn(f"learned ranker not usable ({type(e).__name__}: {e}); using the analytic ranker")
    return AnalyticRanker()


def rows_from_search(paths) -> list[dict]:
    """Training rows {M, N, K, key, us, group} from sharded-search outputs: the per-shape unit files
    (<out>/units/<i>.jsonl, screen entries [key, us, status]) or older per-rank files (entries [key, us]); a directory
    stands for its units/*.jsonl. `group` names the unit a timing came from: each unit ran on one GPU, so timings are
    normalised within their unit."""
    from cs464_b200.keys import parse_key
    files = []
    for p in map(Path, paths):
        files += sorted((p / "units").glob("*.jsonl")) if p.is_dir() else [p]
    out = []
    for f in files:
        for line in f.read_text().splitlines():
            if not line.strip():
                continue
            try:
                r = json.loads(line)
            except ValueError:
                continue
            group = f"{f}:{r.get('i', '')}:{r.get('slice', 0)}:{r.get('run', '')}"
            for entry in r.get("screen", []):
                key, us = entry[0], entry[1]
                try:
                    parse_key(key)
                except ValueError:
                    continue
                if us and us > 0:
                    out.append({"M": r["M"], "N": r["N"], "K": r["K"], "key": key, "us": float(us), "group": group})
    return out


def _main(argv=None) -> None:
    import argparse
    ap = argparse.ArgumentParser(description="train the learned ranker from sharded-search screens")
    ap.add_argument("rows", nargs="+", help="sharded-search output directories (or unit / rank JSONL files)")
    ap.add_argument("--out", default=str(MODEL_STEM))
    ap.add_argument("--max-iter", type=int, default=600)
    a = ap.parse_args(argv)
    rows = rows_from_search(a.rows)
    import sklearn
    r = LearnedRanker().fit(rows, max_iter=a.max_iter)
    info = {"rows": len(rows), "shapes": len({(x["M"], x["N"], x["K"]) for x in rows}), "max_iter": a.max_iter,
            "sources": [Path(x).name for x in a.rows], "sklearn": sklearn.__version__}
    r.save(a.out, info)
    print(json.dumps({**info, "out": a.out}))


if __name__ == "__main__":
    _main()
