"""Shape suites of BASELINE.json's configs, generated deterministically (also written under cs464_b200/suite_data/).

  * config 2 `square_sweep`: M = N = K in {256, ..., 16384}.
  * config 3 `random_suite(seed=1)`: 200 shapes, M, N, K log-uniform in [16, 16384] rounded to multiples of 8, and 20 %
    of them (indices drawn with the same RNG) with M redrawn log-uniform in [16, 64] (skinny, bandwidth-bound). The
    reference's S7 suite is the same idea without the skinny quota (suites/generate.py:112-117).
  * config 4 `llama_suite`: hidden 4096, FFN 14336, 32 q / 8 kv heads x 128: QKV (K 4096 -> N 6144), O (4096 -> 4096),
    gate+up (4096 -> 28672), down (14336 -> 4096), tokens M in {1, 16, 128, 2048, 8192}; weights N(0, 0.02^2).
  * config 5 `fresh_suite(seed=2)`: 1000 fresh shapes from config 3's sampler with seed 2 (config 2 is a fixed
    7-point list, so "its distribution" is read as config 3's sampler).
  * `edge_suite`: the correctness-only edge shapes (degenerate, prime, K below one K step).
"""
from __future__ import annotations

import json
import math
import random
from pathlib import Path

DATA = Path(__file__).resolve().parent / "suite_data"
SQUARE_SIZES = [256, 512, 1024, 2048, 4096, 8192, 16384]
LLAMA_LAYERS = {"qkv": (4096, 6144), "o": (4096, 4096), "gate_up": (4096, 28672), "down": (14336, 4096)}
LLAMA_TOKENS = [1, 16, 128, 2048, 8192]
WEIGHT_STD = 0.02


def square_sweep() -> list[dict]:
    return [{"M": n, "N": n, "K": n, "suite": "square"} for n in SQUARE_SIZES]


def _loguniform8(rng: random.Random, lo: int, hi: int) -> int:
    x = math.exp(rng.uniform(math.log(lo), math.log(hi)))
    return int(min(hi, max(lo, 8 * round(x / 8))))


def random_suite(n: int = 200, seed: int = 1, skinny_frac: float = 0.2, name: str = "random") -> list[dict]:
    rng = random.Random(seed)
    shapes = [{"M": _loguniform8(rng, 16, 16384), "N": _loguniform8(rng, 16, 16384), "K": _loguniform8(rng, 16, 16384),
               "suite": name} for _ in range(n)]
    for i in sorted(rng.sample(range(n), int(round(skinny_frac * n)))):
        shapes[i]["M"] = _loguniform8(rng, 16, 64)
        shapes[i]["skinny"] = True
    return shapes


def llama_suite() -> list[dict]:
    return [{"M": m, "N": n, "K": k, "suite": "llama", "layer": layer, "weight_std": WEIGHT_STD}
            for layer, (k, n) in LLAMA_LAYERS.items() for m in LLAMA_TOKENS]


def fresh_suite(n: int = 1000, seed: int = 2) -> list[dict]:
    return random_suite(n, seed, name="fresh")


def edge_suite() -> list[dict]:
    """Correctness-only shapes at the kernels' edges, the dimensions of the reference's edge suite
    (suites/generate.py:120-131): every (M, N, K) of M in {1, 17, 64, 129, 257}, N in {1, 15, 64, 127, 257},
    K in {1, 3, 16, 33, 255, 1031} (degenerate, prime and off-by-one sizes, K below one K step); cubes of the sizes
    around powers of two from 1 to 257; and four extremes (a 1 x 1 dot product of length 16384, a GEMV, a one-column
    output with a prime K, and K = 8)."""
    shapes = [{"M": m, "N": n, "K": k, "suite": "edge"}
              for m in (1, 17, 64, 129, 257) for n in (1, 15, 64, 127, 257) for k in (1, 3, 16, 33, 255, 1031)]
    shapes += [{"M": d, "N": d, "K": d, "suite": "edge"}
               for d in (1, 2, 3, 7, 15, 16, 17, 31, 33, 63, 65, 127, 129, 255, 257)]
    shapes += [{"M": m, "N": n, "K": k, "suite": "edge"}
               for m, n, k in ((1, 1, 16384), (1, 4096, 4096), (4093, 1, 4093), (2048, 2048, 8))]
    return shapes


SUITES = {"config2": square_sweep, "config3": random_suite, "config4": llama_suite, "config5": fresh_suite,
          "edge": edge_suite}


def load(name: str) -> list[dict]:
    """A suite by config name (config2..config5) or a JSON file path ({"shapes": [...]})."""
    if name in SUITES:
        return SUITES[name]()
    return json.loads(Path(name).read_text())["shapes"]


def write_all() -> None:
    DATA.mkdir(exist_ok=True)
    for name, fn in SUITES.items():
        (DATA / f"{name}.json").write_text(json.dumps({"suite": name, "shapes": fn()}, indent=0) + "\n")


if __name__ == "__main__":
    write_all()
