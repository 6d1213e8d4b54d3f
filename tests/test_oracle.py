"""The CPU oracle against the reference's own outputs (tests/golden, made by tests/golden/make_golden.py).

Pins: the reference's seeded input streams (bit-exact), its fp32 GEMM results (within fp32 reordering noise), its
gate's verdicts (identical), and the oracle's fp16/bf16 rounding against torch's casts (bit-exact)."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = json.loads((GOLDEN / "gemm_cases.json").read_text())["cases"]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("h", json.loads((GOLDEN / "inputs_hash.json").read_text())["inputs"],
                         ids=lambda h: f"{h['M']}x{h['N']}x{h['K']}_{h['dtype']}_s{h['seed']}")
def test_make_inputs_bit_exact(h):
    a, b = oracle.make_inputs(h["M"], h["N"], h["K"], dtype=getattr(torch, h["dtype"]), seed=h["seed"])
    assert hashlib.sha256(_bits(a).tobytes()).hexdigest() == h["a_sha256"]
    assert hashlib.sha256(_bits(b).tobytes()).hexdigest() == h["b_sha256"]


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "gemm_cases.npz")


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_golden_inputs_regenerate(case, golden):
    a, b = oracle.make_inputs(case["M"], case["N"], case["K"], dtype=getattr(torch, case["dtype"]),
                              seed=case["seed"])
    assert np.array_equal(_bits(a), golden[f"{case['name']}_a"])
    assert np.array_equal(_bits(b), golden[f"{case['name']}_b"])


@pytest.mark.parametrize("acc_double", [False, True])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_oracle_gemm_matches_reference(case, golden, acc_double):
    dt = getattr(torch, case["dtype"])
    a = torch.from_numpy(golden[f"{case['name']}_a"].view(np.int16)).view(dt)
    b = torch.from_numpy(golden[f"{case['name']}_b"].view(np.int16)).view(dt)
    ref = golden[f"{case['name']}_ref"]
    got = oracle.gemm_f32(a, b, acc_double=acc_double)
    # fp32 accumulation order differs from the reference's BLAS: bound the gap by fp32 rounding of the dot products
    an = np.sqrt((a.float().numpy().astype(np.float64) ** 2).sum(1))
    bn = np.sqrt((b.float().numpy().astype(np.float64) ** 2).sum(0))
    scale = an[:, None] * bn[None, :]
    assert np.all(np.abs(got.astype(np.float64) - ref) <= 4 * case["K"] * 2.0 ** -24 * scale + 1e-30)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_gate_verdicts_match_reference(case, golden):
    """oracle.check_output restates tune/correctness.py:116-127: same verdicts and errors on the same arrays."""
    dt = getattr(torch, case["dtype"])
    ref = golden[f"{case['name']}_ref"]
    K = case["K"]
    rounded = torch.from_numpy(ref).to(dt).float().numpy()
    arrays = {"rounded": rounded}
    if "corrupt_tile" in case["verdicts"]:
        bad = torch.from_numpy(ref).to(dt)
        bad[:16, :16] += float(max(1.0, 0.05 * np.sqrt(K)) * 10)
        arrays["corrupt_tile"] = bad.float().numpy()
    nan = rounded.copy()
    nan[-1] = np.nan
    arrays["nan_row"] = nan
    for kind, arr in arrays.items():
        want = case["verdicts"][kind]
        got = oracle.check_output(arr, ref, K, case["dtype"])
        assert got.valid == want["valid"], (kind, got, want)
        assert got.failure_reason == want["failure_reason"], (kind, got, want)
        if np.isfinite(want["max_abs_err"]):
            assert got.max_abs_err == pytest.approx(want["max_abs_err"], rel=1e-6, abs=1e-9)


def test_rounding_matches_torch_bit_exact():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-8, 1e-5, 1, 300, 7e4)] +
                       [np.array([0.0, -0.0, np.inf, -np.inf, 65504, 65519.99, 65520, 6.1e-5, 5.96e-8, 2.98e-8,
                                  2.99e-8, 1e-45], dtype=np.float32)])
    h = oracle.round_to(x, bf16=False)
    assert np.array_equal(h, torch.from_numpy(x).half().view(torch.int16).numpy().view(np.uint16))
    bf = oracle.round_to(x, bf16=True)
    assert np.array_equal(bf, torch.from_numpy(x).bfloat16().view(torch.int16).numpy().view(np.uint16))


def test_decode_all_fp16_bit_patterns():
    bits = np.arange(65536, dtype=np.uint16)
    finite = ~(((bits >> 10) & 0x1F) == 0x1F)
    # the oracle's decode via gemm_f32 of a 1x1 times 1.0
    one = np.array([[0x3C00]], dtype=np.uint16)
    vals = np.array([oracle.gemm_f32(np.array([[v]], dtype=np.uint16), one)[0, 0] for v in bits[finite][::97]])
    want = bits[finite][::97].view(np.float16).astype(np.float32)
    assert np.array_equal(vals, want)


def test_splitk_reduce_restatement():
    rng = np.random.default_rng(1)
    ws = rng.standard_normal((5, 7, 9)).astype(np.float32)
    acc = np.zeros((7, 9), dtype=np.float32)
    for s in range(5):
        acc = (acc + ws[s]).astype(np.float32)
    assert np.array_equal(oracle.splitk_reduce(ws), oracle.round_to(acc))


def test_norm_rel_check_catches_errors():
    a, b = oracle.make_inputs(32, 48, 256, seed=5)
    ref = oracle.gemm_f32(a, b, acc_double=True)
    good = oracle.bits_to_f32(oracle.round_to(ref))
    assert oracle.norm_rel_check(good, ref, a, b)[0]
    bad = good.copy()
    bad[3, 4] += 0.05 * np.sqrt(256)
    ok, worst = oracle.norm_rel_check(bad, ref, a, b)
    assert not ok and worst > oracle.NORM_REL_TOL
