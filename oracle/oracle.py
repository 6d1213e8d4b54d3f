"""CPU oracle for the GEMM path. TEST INFRASTRUCTURE ONLY.

Only tests/, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg import this module, and only as the checker or
the timed CPU baseline; the product (package `cs464_b200`) never does.

What it restates, each from the reference file and line it follows:
  * `make_inputs`     tune/correctness.py:36-40   seeded N(0,1) fp32 drawn with a torch Generator, cast to fp16/bf16
  * `gemm_f32`        kernels/triton_matmul.py:67-82 and tune/correctness.py:100-102: fp32-accumulated GEMM of the
                      fp16-rounded inputs (C restatement in gemm_ref.c; fp32 FMA in k order, or double accumulation)
  * `gemm`            kernels/triton_matmul.py:82: the same, cast to the output dtype with round-to-nearest-even
  * `splitk_reduce`   kernels/triton_matmul.py:85-92: fixed-order fp32 sum of split partials, then the cast
  * `check_output`    tune/correctness.py:116-127: the reference's gate |C-ref| <= rtol*|ref| + atol_frac*sqrt(K),
                      non-finite outputs fail first
  * `norm_rel_check`  BASELINE north star: |C-ref|_ij <= 2e-3 * ||A_i,:||_2 * ||B_:,j||_2
  * `reference_cpu`   tune/correctness.py:100-102 run on the host: torch fp32 matmul of the upcast operands; this is the
                      reference's CPU path, also the timed CPU baseline (all host threads)

Parity of this oracle is pinned against fixtures generated from the reference itself (tests/golden/make_golden.py,
which imports the reference's tune/correctness.py and kernels/config_space.py in the build container).
"""
from __future__ import annotations

import ctypes
import math
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

# tune/correctness.py:20-23
TOLERANCES = {"float16": {"rtol": 1e-2, "atol_frac": 1e-2}, "bfloat16": {"rtol": 3e-2, "atol_frac": 3e-2}}
NORM_REL_TOL = 2e-3

_lib = None


def build() -> Path:
    """Compile gemm_ref.c into liboracle.so (make; gcc only)."""
    if not LIB.exists() or LIB.stat().st_mtime < (HERE / "gemm_ref.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB))
        u16p = ctypes.POINTER(ctypes.c_uint16)
        f32p = ctypes.POINTER(ctypes.c_float)
        i64 = ctypes.c_int64
        lib.oracle_gemm_f32.argtypes = [u16p, i64, i64, u16p, i64, i64, f32p, i64, i64, i64, ctypes.c_int,
                                        ctypes.c_int]
        lib.oracle_gemm_f32.restype = ctypes.c_int
        lib.oracle_round.argtypes = [f32p, u16p, i64, ctypes.c_int]
        lib.oracle_splitk_reduce.argtypes = [f32p, u16p, i64, ctypes.c_int32, ctypes.c_int]
        lib.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.oracle_f16_to_f32.restype = ctypes.c_float
        lib.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_f16.restype = ctypes.c_uint16
        lib.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
        _lib = lib
    return _lib


def _bits(x) -> tuple[np.ndarray, bool]:
    """(uint16 bit pattern array, is_bf16) of a torch fp16/bf16 tensor or a numpy float16 array."""
    try:
        import torch
        if isinstance(x, torch.Tensor):
            t = x.detach().cpu()
            if t.dtype == torch.bfloat16:
                return t.view(torch.int16).numpy().view(np.uint16), True
            if t.dtype == torch.float16:
                return t.view(torch.int16).numpy().view(np.uint16), False
            raise TypeError(f"oracle needs fp16/bf16 operands, got {t.dtype}")
    except ImportError:
        pass
    a = np.asarray(x)
    if a.dtype == np.float16:
        return a.view(np.uint16), False
    if a.dtype == np.uint16:
        return a, False
    raise TypeError(f"oracle needs fp16/bf16 operands, got {a.dtype}")


def gemm_f32(a, b, acc_double: bool = False) -> np.ndarray:
    """fp32 [M, N] = A @ B from fp16/bf16 operands of any strides (C restatement)."""
    abits, abf = _bits(a)
    bbits, bbf = _bits(b)
    if abf != bbf:
        raise TypeError("A and B must share one dtype")
    M, K = abits.shape
    K2, N = bbits.shape
    assert K == K2, (abits.shape, bbits.shape)
    out = np.empty((M, N), dtype=np.float32)
    sa = [s // 2 for s in abits.strides]
    sb = [s // 2 for s in bbits.strides]
    # keep the (possibly strided) views alive and point at their first element
    pa = abits.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))
    pb = bbits.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))
    rc = _load().oracle_gemm_f32(pa, sa[0], sa[1], pb, sb[0], sb[1],
                                 out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), M, N, K, int(abf),
                                 int(acc_double))
    if rc:
        raise MemoryError("oracle_gemm_f32 allocation failed")
    return out


def round_to(x: np.ndarray, bf16: bool = False) -> np.ndarray:
    """Round fp32 to fp16/bf16 bit patterns (uint16), nearest-even (the epilogue cast)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    _load().oracle_round(x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                         out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), x.size, int(bf16))
    return out


def gemm(a, b) -> np.ndarray:
    """Output-dtype result (uint16 bit patterns) of the GEMM: fp32 accumulate, one rounding at the end."""
    _, bf = _bits(a)
    return round_to(gemm_f32(a, b), bf)


def splitk_reduce(ws: np.ndarray, bf16: bool = False) -> np.ndarray:
    ws = np.ascontiguousarray(ws, dtype=np.float32)
    split = ws.shape[0]
    mn = int(np.prod(ws.shape[1:]))
    out = np.empty(ws.shape[1:], dtype=np.uint16)
    _load().oracle_splitk_reduce(ws.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                 out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), mn, split, int(bf16))
    return out


def bits_to_f32(bits: np.ndarray, bf16: bool = False) -> np.ndarray:
    bits = np.asarray(bits, dtype=np.uint16)
    if bf16:
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def make_inputs(M: int, N: int, K: int, dtype=None, seed: int = 0, device: str = "cpu"):
    """The reference's seeded inputs (tune/correctness.py:36-40): one torch Generator on `device` seeded with `seed`,
    randn A then B in fp32, cast. CPU and CUDA generators give different streams; the fixtures use the CPU one."""
    import torch
    dtype = dtype or torch.float16
    g = torch.Generator(device=device).manual_seed(seed)
    a = torch.randn((M, K), generator=g, device=device, dtype=torch.float32).to(dtype)
    b = torch.randn((K, N), generator=g, device=device, dtype=torch.float32).to(dtype)
    return a, b


def reference_cpu(a, b):
    """tune/correctness.py:100-102 on the host: fp32 matmul of the upcast operands (torch CPU, all threads)."""
    import torch
    return a.detach().cpu().float() @ b.detach().cpu().float()


@dataclass
class CheckResult:
    valid: bool
    failure_reason: str | None
    max_abs_err: float
    max_rel_err_vs_scale: float


def check_output(c, ref, K: int, dtype: str = "float16") -> CheckResult:
    """The reference's gate (tune/correctness.py:116-127) on numpy arrays: c as float32 (or fp16), ref float32."""
    tol = TOLERANCES[dtype]
    c32 = np.asarray(c, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    finite = np.isfinite(c32)
    if not finite.all():
        n_bad = int((~finite).sum())
        return CheckResult(False, f"non_finite_output({n_bad})", math.inf, math.inf)
    err = np.abs(c32 - ref)
    scale = math.sqrt(max(K, 1))
    bound = tol["rtol"] * np.abs(ref) + tol["atol_frac"] * scale
    max_abs = float(err.max()) if err.size else 0.0
    ok = bool((err <= bound).all())
    return CheckResult(ok, None if ok else "tolerance_exceeded", max_abs, max_abs / scale)


def norm_rel_check(c, ref, a, b, tol: float = NORM_REL_TOL) -> tuple[bool, float]:
    """(passes, max over elements of |C-ref|_ij / (||A_i,:|| * ||B_:,j||)): the north star's per-element bound.
    A row or column of zeros gives a zero scale; there the error must be zero."""
    c32 = np.asarray(c, dtype=np.float32).astype(np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    abits, abf = _bits(a)
    bbits, _ = _bits(b)
    an = np.sqrt((bits_to_f32(abits, abf).astype(np.float64) ** 2).sum(axis=1))
    bn = np.sqrt((bits_to_f32(bbits, abf).astype(np.float64) ** 2).sum(axis=0))
    scale = an[:, None] * bn[None, :]
    err = np.abs(c32 - ref)
    if not np.isfinite(c32).all():
        return False, math.inf
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = np.where(scale > 0, err / scale, np.where(err > 0, np.inf, 0.0))
    worst = float(ratio.max()) if ratio.size else 0.0
    return worst <= tol, worst
