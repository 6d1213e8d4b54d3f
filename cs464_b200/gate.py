"""The correctness gate: what every candidate of the sm_100a family passes before it is timed.

Kept from the reference because they are its callers' contract (tune/correctness.py): the verdict rule, elementwise
    |C - ref| <= rtol * |ref| + atol_frac * sqrt(K)         (fp16: 1e-2, 1e-2; bf16: 3e-2, 3e-2; :20-23, :116-127)
with non-finite outputs failing first (`non_finite_output(<count>)`) and `tolerance_exceeded` otherwise; the seeded
inputs (one generator, randn A then B in fp32, then the cast; :36-40); the fp32 ground truth with TF32 off
(:100-102); a candidate's exception becoming an invalid verdict (:147-149); and the error-message markers of a
sticky CUDA fault (:80-88). The names (validate, check_output, reference, make_inputs, placed_inputs, CheckResult)
are the ones those callers use.

This module's own design:
  * `Problem` holds one shape's inputs, fp32 reference and the row/column norms of A and B, and judges any number of
    candidates against them: the search validates hundreds of configs per shape and pays for the reference once;
  * judging is one streaming pass over row blocks of the output that yields every statistic at once (non-finite
    count, largest error, the gate's verdict and the north star's norm-relative error, below), with O(block) extra
    memory instead of several M x N temporaries (a 16384^2 check needs ~0.5 GB, not ~4 GB);
  * the north star's scale-free bound, which does not assume unit-variance inputs (BASELINE config 4's weights are
    N(0, 0.02^2), where atol_frac * sqrt(K) is 50x too loose):
        |C - ref|_ij <= 2e-3 * ||A_i,:||_2 * ||B_:,j||_2
  * the kernels' device status word: a runner whose bounded device wait ran out reports
    `device_wait_timeout(...)`, a failure that leaves the context usable (not a poisoning fault);
  * placements: the same values at other addresses inside one arena per call, at offsets a hash of (seed, placement,
    shape) picks on a 4 KiB grid.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

TOLERANCES = {
    torch.float16: {"rtol": 1e-2, "atol_frac": 1e-2},
    torch.bfloat16: {"rtol": 3e-2, "atol_frac": 3e-2},
}
NORM_REL_TOL = 2e-3
# substrings of CUDA's messages for faults after which nothing else can run in the process (the callers' contract)
CONTEXT_POISON_MARKERS = ("illegal", "misaligned", "unspecified launch failure", "device-side assert",
                          "an illegal instruction")
ROW_BLOCK_ELEMS = 1 << 25   # elements of C judged per pass (128 MiB of fp32 per temporary)
PLACEMENT_GRID = 4096       # placement offsets are whole pages, so every alignment the allocator gives is kept
PLACEMENT_SPAN = 1 << 26    # and lie within 64 MiB


def reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp32 GEMM of the operands as stored (their fp16/bf16 values), full fp32 products: TF32 is switched off for
    the call and restored after."""
    saved = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return torch.matmul(a.to(torch.float32), b.to(torch.float32))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = saved


def make_inputs(M: int, N: int, K: int, dtype=torch.float16, seed: int = 0, device: str = "cuda",
                scale_b: float = 1.0):
    """Seeded operands: one generator on `device`, A [M, K] then B [K, N] drawn N(0, 1) in fp32, B times `scale_b`
    (BASELINE config 4's weights use 0.02), both cast to `dtype`."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    a32 = torch.randn(M, K, generator=gen, device=device, dtype=torch.float32)
    b32 = torch.randn(K, N, generator=gen, device=device, dtype=torch.float32)
    return a32.to(dtype), (b32 if scale_b == 1.0 else b32.mul_(scale_b)).to(dtype)


def _mix64(x: int) -> int:
    """splitmix64's finaliser (Steele, Lea & Flood 2014): a well-spread 64-bit hash of x."""
    x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return x ^ (x >> 31)


def placed_inputs(M: int, N: int, K: int, dtype=torch.float16, seed: int = 0, placement: int = 0,
                  device: str = "cuda", avoid=frozenset(), scale_b: float = 1.0):
    """The operands of `make_inputs` (same values) at other device addresses: placement 0 returns them as made; any
    other placement copies both into one fresh arena, each at a page-aligned offset hashed from (seed, placement,
    shape, operand), so timings over several placements sample different DRAM channels and L2 sets. An address in
    `avoid` moves that operand on by one more span step. Returns (A, B, None); the arena stays alive through the
    returned views."""
    a, b = make_inputs(M, N, K, dtype, seed, device, scale_b)
    if not placement:
        return a, b, None
    esz = a.element_size()
    key = _mix64(_mix64(seed) ^ _mix64(placement) ^ _mix64(M * 1_000_003 + N * 10_007 + K))
    offs = [(_mix64(key + j) % (PLACEMENT_SPAN // PLACEMENT_GRID)) * PLACEMENT_GRID for j in (1, 2)]
    size_a = -(-a.numel() * esz // PLACEMENT_GRID) * PLACEMENT_GRID
    size_b = -(-b.numel() * esz // PLACEMENT_GRID) * PLACEMENT_GRID
    tries = 4
    arena = torch.empty(offs[0] + size_a + offs[1] + size_b + 2 * tries * PLACEMENT_SPAN, dtype=torch.uint8,
                        device=device)
    out = []
    base = 0
    for t, off, size in ((a, offs[0], size_a), (b, offs[1], size_b)):
        start = base + off
        for _ in range(tries):
            if arena[start:].data_ptr() not in avoid:
                break
            start += PLACEMENT_SPAN
        v = arena[start:start + t.numel() * esz].view(t.dtype).view(t.shape)
        v.copy_(t)
        out.append(v)
        base = start + size
    return out[0], out[1], None


def context_poisoned(reason: str | None) -> bool:
    """True when a failure reason names a sticky CUDA fault: nothing else can run in this process afterwards."""
    r = (reason or "").lower()
    return any(m in r for m in CONTEXT_POISON_MARKERS)


class ContextPoisoned(RuntimeError):
    """A candidate faulted the CUDA context; `culprit` names it."""

    def __init__(self, culprit: str, reason: str):
        super().__init__(f"{culprit} poisoned the CUDA context: {reason}")
        self.culprit, self.reason = culprit, reason


@dataclass
class CheckResult:
    valid: bool
    failure_reason: str | None
    max_abs_err: float
    max_rel_err_vs_scale: float            # largest |error| / sqrt(K): in units of one output's std for N(0,1) inputs
    max_norm_rel_err: float | None = None  # largest |error|_ij / (||A_i,:|| ||B_:,j||), when the norms were given

    def to_dict(self) -> dict:
        return dict(self.__dict__)


def _judge(c: torch.Tensor, ref: torch.Tensor, K: int, dtype, row_norm=None, col_norm=None) -> dict:
    """Every statistic of one candidate output in one pass over row blocks."""
    tol = TOLERANCES[dtype]
    M, N = ref.shape
    rows = max(1, ROW_BLOCK_ELEMS // max(N, 1))
    atol = tol["atol_frac"] * math.sqrt(max(K, 1))
    bad = 0
    over = 0
    max_abs = 0.0
    worst_nr = 0.0
    for r0 in range(0, M, rows):
        r1 = min(M, r0 + rows)
        x = c[r0:r1].to(torch.float32, copy=True)  # a copy: the error is formed in place below
        finite = torch.isfinite(x)
        nb = int(finite.numel() - finite.sum())
        bad += nb
        if bad:
            continue  # the verdict is settled; only the count of non-finite elements still matters
        y = ref[r0:r1]
        err = x.sub_(y).abs_()
        if err.numel():
            max_abs = max(max_abs, float(err.max()))
        over += int((err > y.abs().mul_(tol["rtol"]).add_(atol)).sum())
        if row_norm is not None:
            scale = torch.outer(row_norm[r0:r1], col_norm)
            ratio = torch.where(scale > 0, err / scale.clamp_min(torch.finfo(torch.float32).tiny),
                                torch.where(err > 0, torch.full_like(err, math.inf), torch.zeros_like(err)))
            if ratio.numel():
                worst_nr = max(worst_nr, float(ratio.max()))
    return {"non_finite": bad, "over_gate": over, "max_abs": max_abs if not bad else math.inf,
            "norm_rel": worst_nr if not bad else math.inf}


def _verdict(s: dict, K: int, norm_rel: bool) -> CheckResult:
    scale = math.sqrt(max(K, 1))
    if s["non_finite"]:
        return CheckResult(False, f"non_finite_output({s['non_finite']})", math.inf, math.inf,
                           math.inf if norm_rel else None)
    nr = s["norm_rel"] if norm_rel else None
    if s["over_gate"]:
        return CheckResult(False, "tolerance_exceeded", s["max_abs"], s["max_abs"] / scale, nr)
    if norm_rel and nr > NORM_REL_TOL:
        return CheckResult(False, "norm_relative_exceeded", s["max_abs"], s["max_abs"] / scale, nr)
    return CheckResult(True, None, s["max_abs"], s["max_abs"] / scale, nr)


def check_output(c: torch.Tensor, ref: torch.Tensor, K: int, dtype) -> CheckResult:
    """The reference gate's verdict on one output against its fp32 reference."""
    return _verdict(_judge(c, ref, K, dtype), K, norm_rel=False)


def operand_norms(a: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """||A_i,:||_2 per row and ||B_:,j||_2 per column, in fp32."""
    return torch.linalg.vector_norm(a.to(torch.float32), dim=1), torch.linalg.vector_norm(b.to(torch.float32), dim=0)


def norm_relative_error(c: torch.Tensor, ref: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> float:
    """max_ij |C - ref|_ij / (||A_i,:|| ||B_:,j||); a zero scale with a non-zero error counts as infinite."""
    rn, cn = operand_norms(a, b)
    return _judge(c, ref, a.shape[1], _tol_dtype(c.dtype), rn, cn)["norm_rel"]


def _tol_dtype(dtype):
    """The row of TOLERANCES to use for an output dtype (fp16's for anything else, e.g. an fp32 reference)."""
    return dtype if dtype in TOLERANCES else torch.float16


def check_norm_relative(c, ref, a, b, tol: float = NORM_REL_TOL) -> CheckResult:
    """The north star's per-element bound alone (the gate's verdict is not applied)."""
    rn, cn = operand_norms(a, b)
    s = _judge(c, ref, a.shape[1], _tol_dtype(c.dtype), rn, cn)
    K = a.shape[1]
    if s["non_finite"]:
        return CheckResult(False, f"non_finite_output({s['non_finite']})", math.inf, math.inf, math.inf)
    ok = s["norm_rel"] <= tol
    return CheckResult(ok, None if ok else "norm_relative_exceeded", s["max_abs"],
                       s["max_abs"] / math.sqrt(max(K, 1)), s["norm_rel"])


class Problem:
    """One shape's operands, fp32 reference and operand norms: built once, judges any number of candidates."""

    def __init__(self, M: int, N: int, K: int, dtype=torch.float16, seed: int = 0, *, inputs=None, ref=None,
                 scale_b: float = 1.0, device: str = "cuda"):
        self.M, self.N, self.K, self.dtype = M, N, K, dtype
        self.a, self.b = inputs if inputs is not None else make_inputs(M, N, K, dtype, seed, device, scale_b)
        self.ref = ref if ref is not None else reference(self.a, self.b)
        self._norms = None

    def norms(self):
        if self._norms is None:
            self._norms = operand_norms(self.a, self.b)
        return self._norms

    def judge(self, c: torch.Tensor, norm_rel: bool = False) -> CheckResult:
        rn, cn = self.norms() if norm_rel else (None, None)
        return _verdict(_judge(c, self.ref, self.K, self.dtype, rn, cn), self.K, norm_rel)

    def check(self, backend, norm_rel: bool = False) -> CheckResult:
        """Run the backend once into a NaN-filled output (unwritten elements fail) and judge it. Never raises: an
        exception is an invalid verdict naming it; a kernel that gave up a bounded device wait is
        `device_wait_timeout(...)`."""
        try:
            out = torch.full((self.M, self.N), math.nan, device=self.a.device, dtype=self.dtype)
            run = backend.make_runner(self.a, self.b, out=out)
            c = run()
            if self.a.is_cuda:
                torch.cuda.synchronize(self.a.device)
            status = getattr(run, "device_status", None)
            if callable(status):
                code = status()
                if code:
                    from cs464_b200._abi import status_string
                    return CheckResult(False, f"device_wait_timeout(0x{code:x}: {status_string(code)})", math.nan,
                                       math.nan)
            return self.judge(c if c is not None else out, norm_rel)
        except Exception as e:  # unsupported configs, launch errors, faults
            text = str(e).splitlines()[0][:200] if str(e) else ""
            return CheckResult(False, f"{type(e).__name__}: {text}", math.nan, math.nan)


def validate(backend, M: int, N: int, K: int, dtype=torch.float16, seed: int = 0, ref: torch.Tensor | None = None,
             inputs=None, norm_rel: bool = False) -> CheckResult:
    """One candidate through the gate (and the norm-relative bound with `norm_rel`): `Problem(...).check(...)`."""
    try:
        prob = Problem(M, N, K, dtype, seed, inputs=inputs, ref=ref)
    except Exception as e:  # inputs that do not fit, a reference that fails
        return CheckResult(False, f"{type(e).__name__}: {str(e).splitlines()[0][:200] if str(e) else ''}",
                           math.nan, math.nan)
    return prob.check(backend, norm_rel)
