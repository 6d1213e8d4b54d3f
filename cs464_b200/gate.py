"""Correctness gate every candidate passes before it is timed (same interface and verdicts as tune/correctness.py).

Reference: an fp32 GEMM of the (fp16-rounded) inputs with TF32 off (tune/correctness.py:100-102), computed with torch
on the operands' device. Inputs are N(0,1), so each reference element has std ~ sqrt(K).

Pass criterion, elementwise, as in the reference (tune/correctness.py:116-127):
    |C - ref| <= rtol * |ref| + atol_frac * sqrt(K)
The output is pre-filled with NaN, so a kernel that leaves elements unwritten fails (`non_finite_output(n)`).

The north star adds a scale-free bound that does not assume unit-variance inputs (BASELINE.json config 4 draws weights from
N(0, 0.02^2), where atol_frac * sqrt(K) is 50x too loose):
    |C - ref|_ij <= 2e-3 * ||A_i,:||_2 * ||B_:,j||_2          (`check_norm_relative`, `validate(..., norm_rel=True)`)

A kernel of this family that gave up a bounded device wait reports it through its runner's status word; `validate`
turns that into the failure `device_wait_timeout(...)`, which leaves the CUDA context usable (not a poisoning fault).
"""
from __future__ import annotations

import math
import random
from contextlib import contextmanager
from dataclasses import dataclass

import torch

TOLERANCES = {
    torch.float16: {"rtol": 1e-2, "atol_frac": 1e-2},
    torch.bfloat16: {"rtol": 3e-2, "atol_frac": 3e-2},
}
NORM_REL_TOL = 2e-3
PLACEMENT_MAX_TRIES = 8
CONTEXT_POISON_MARKERS = ("illegal", "misaligned", "unspecified launch failure", "device-side assert",
                          "an illegal instruction")


@contextmanager
def strict_fp32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def make_inputs(M: int, N: int, K: int, dtype=torch.float16, seed: int = 0, device: str = "cuda",
                scale_b: float = 1.0):
    """Seeded A [M,K] and B [K,N]: one generator on `device`, randn A then B in fp32, cast (tune/correctness.py:36-40).
    `scale_b` multiplies B before the cast (BASELINE.json config 4's weights are N(0, 0.02^2))."""
    g = torch.Generator(device=device).manual_seed(seed)
    a = torch.randn((M, K), generator=g, device=device, dtype=torch.float32).to(dtype)
    b = torch.randn((K, N), generator=g, device=device, dtype=torch.float32)
    if scale_b != 1.0:
        b = b * scale_b
    return a, b.to(dtype)


def placed_inputs(M: int, N: int, K: int, dtype=torch.float16, seed: int = 0, placement: int = 0,
                  device: str = "cuda", avoid=frozenset()):
    """The same values as `make_inputs` at another device address per `placement` (0 = as made). Each operand is
    copied into a fresh buffer at a whole number of MiB (1-64, drawn from a string-seeded RNG per (seed, placement,
    shape)), so bases keep the allocator's alignment; an address in `avoid` is redrawn a few times. Returns
    (a, b, None) like the reference (tune/correctness.py:46-77)."""
    a, b = make_inputs(M, N, K, dtype, seed, device)
    if not placement:
        return a, b, None
    rng = random.Random(f"placement:{seed}:{placement}:{M}x{N}x{K}")
    out = []
    for t in (a, b):
        v = None
        for _ in range(PLACEMENT_MAX_TRIES):
            shift = rng.randint(1, 64) * 2**20 // t.element_size()
            v = torch.empty(shift + t.numel(), dtype=t.dtype, device=device)[shift:].view(t.shape)
            if v.data_ptr() not in avoid:
                break
        v.copy_(t)
        out.append(v)
    return out[0], out[1], None


def context_poisoned(reason: str | None) -> bool:
    """True when a failure reason is a sticky CUDA fault: nothing else can run in this process afterwards."""
    r = (reason or "").lower()
    return any(x in r for x in CONTEXT_POISON_MARKERS)


class ContextPoisoned(RuntimeError):
    """A candidate faulted the CUDA context; `culprit` names it."""

    def __init__(self, culprit: str, reason: str):
        super().__init__(f"{culprit} poisoned the CUDA context: {reason}")
        self.culprit, self.reason = culprit, reason


def reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    with strict_fp32():
        return a.float() @ b.float()


@dataclass
class CheckResult:
    valid: bool
    failure_reason: str | None
    max_abs_err: float
    max_rel_err_vs_scale: float          # max |err| / sqrt(K): error in units of one output std
    max_norm_rel_err: float | None = None  # max |err|_ij / (||A_i,:|| ||B_:,j||), when computed

    def to_dict(self) -> dict:
        return self.__dict__.copy()


def check_output(c: torch.Tensor, ref: torch.Tensor, K: int, dtype) -> CheckResult:
    tol = TOLERANCES[dtype]
    c32 = c.float()
    if not torch.isfinite(c32).all():
        n_bad = int((~torch.isfinite(c32)).sum())
        return CheckResult(False, f"non_finite_output({n_bad})", math.inf, math.inf)
    err = (c32 - ref).abs()
    scale = math.sqrt(max(K, 1))
    bound = tol["rtol"] * ref.abs() + tol["atol_frac"] * scale
    max_abs = float(err.max()) if err.numel() else 0.0
    ok = bool((err <= bound).all())
    return CheckResult(ok, None if ok else "tolerance_exceeded", max_abs, max_abs / scale)


def norm_relative_error(c: torch.Tensor, ref: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> float:
    """max_ij |C - ref|_ij / (||A_i,:||_2 * ||B_:,j||_2); a zero scale with a non-zero error counts as infinite."""
    if c.numel() == 0:
        return 0.0
    err = (c.float() - ref).abs()
    scale = a.float().norm(dim=1)[:, None] * b.float().norm(dim=0)[None, :]
    ratio = torch.where(scale > 0, err / scale.clamp_min(torch.finfo(torch.float32).tiny),
                        torch.where(err > 0, torch.full_like(err, math.inf), torch.zeros_like(err)))
    return float(ratio.max())


def check_norm_relative(c, ref, a, b, tol: float = NORM_REL_TOL) -> CheckResult:
    if not torch.isfinite(c.float()).all():
        n_bad = int((~torch.isfinite(c.float())).sum())
        return CheckResult(False, f"non_finite_output({n_bad})", math.inf, math.inf, math.inf)
    worst = norm_relative_error(c, ref, a, b)
    max_abs = float((c.float() - ref).abs().max()) if c.numel() else 0.0
    ok = worst <= tol
    return CheckResult(ok, None if ok else "norm_relative_exceeded", max_abs,
                       max_abs / math.sqrt(max(a.shape[1], 1)), worst)


def validate(backend, M: int, N: int, K: int, dtype=torch.float16, seed: int = 0, ref: torch.Tensor | None = None,
             inputs=None, norm_rel: bool = False) -> CheckResult:
    """Run `backend.make_runner(a, b, out)` once into a NaN-filled buffer and compare with the fp32 reference
    (tune/correctness.py:130-149). Every exception becomes a failure, never a raise; a sticky fault is reported so
    the caller stops (`context_poisoned`). With `norm_rel` the north star's bound must hold as well."""
    try:
        a, b = inputs if inputs is not None else make_inputs(M, N, K, dtype, seed)
        if ref is None:
            ref = reference(a, b)
        out = torch.full((M, N), float("nan"), device=a.device, dtype=dtype)
        run = backend.make_runner(a, b, out=out)
        c = run()
        torch.cuda.synchronize()
        status = getattr(run, "device_status", None)
        if callable(status):
            s = status()
            if s:
                from cs464_b200._abi import status_string
                return CheckResult(False, f"device_wait_timeout(0x{s:x}: {status_string(s)})", math.nan, math.nan)
        if c.data_ptr() != out.data_ptr():
            out = c
        r = check_output(out, ref, K, dtype)
        if r.valid and norm_rel:
            nr = check_norm_relative(out, ref, a, b)
            r.max_norm_rel_err = nr.max_norm_rel_err
            if not nr.valid:
                r.valid, r.failure_reason = False, nr.failure_reason
        return r
    except Exception as e:  # unsupported configs, launch errors, faults
        msg = f"{type(e).__name__}: {str(e).splitlines()[0][:200] if str(e) else ''}"
        return CheckResult(False, msg, math.nan, math.nan)
