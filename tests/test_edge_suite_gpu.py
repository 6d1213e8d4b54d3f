"""The reference's edge suite as a GPU parity fixture (suites/generate.py:120-131, `python -m tune check --suite edge`
in the reference): 169 shapes with degenerate, prime and off-by-one dimensions and K below one K step. Every
HANDPICKED config and every config the bench's first-use selection can pick for a square size (the ranker's top 3
and the zero-search rule, for each of BASELINE config 2's sizes) runs each shape into a NaN-filled output through the
C ABI, against the C oracle under both bounds: the reference gate |C-ref| <= 1e-2*|ref| + 1e-2*sqrt(K) and
|C-ref|_ij <= 2e-3 * ||A_i,:|| * ||B_:,j||. Shapes whose split-K workspace a config's rules refuse are skipped, as the
reference's kernel tests do."""
from __future__ import annotations

import pytest
import torch

from cs464_b200 import suites
from cs464_b200.config_space import HANDPICKED, shape_violations
from cs464_b200.keys import parse_key
from cs464_b200.matmul import B200Matmul
from cs464_b200.ranker import default_ranker
from cs464_b200.select import heuristic_config
from oracle import oracle

pytestmark = pytest.mark.gpu

SHAPES = suites.edge_suite()


def _configs():
    r = default_ranker()
    keys = [c.key() for c in HANDPICKED.values()]
    for n in suites.SQUARE_SIZES:
        keys += r.rank(n, n, n, 3, order="diverse") + [heuristic_config(n, n, n).key()]
    return [parse_key(k) for k in dict.fromkeys(keys)]


@pytest.mark.parametrize("block", range(0, len(SHAPES), 24), ids=lambda i: f"shapes{i}")
def test_edge_suite_matches_oracle(block):
    cfgs = _configs()
    for s in SHAPES[block:block + 24]:
        M, N, K = s["M"], s["N"], s["K"]
        a, b = oracle.make_inputs(M, N, K, seed=0)
        ref = oracle.gemm_f32(a, b)
        a_dev, b_dev = a.cuda(), b.cuda()
        for cfg in cfgs:
            if "split_k_workspace_too_large" in shape_violations(cfg, M, N, K):
                continue
            out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float16)
            run = B200Matmul(cfg).make_runner(a_dev, b_dev, out=out)
            c = run()
            torch.cuda.synchronize()
            run.raise_on_status()
            c32 = c.float().cpu().numpy()
            r = oracle.check_output(c32, ref, K)
            assert r.valid, (M, N, K, cfg.key(), r)
            ok, worst = oracle.norm_rel_check(c32, ref, a, b)
            assert ok, (M, N, K, cfg.key(), worst)
