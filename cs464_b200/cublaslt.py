"""cuBLASLt comparator (the reference's B2 / B3 baselines, baselines/cublaslt.py:114-180): the library's heuristic top-N
algorithms for a row-major fp16/bf16 GEMM, each wrapped in the make_runner protocol so the same gate and timer measure
them. Measurement only: the sm_100a family never dispatches here.

Row-major C[M,N] = A[M,K] B[K,N] is the column-major product C^T = B^T A^T, so cuBLASLt sees m = N, n = M, k = K with
"A" = B (ld N), "B" = A (ld K), C (ld N), no transposes; fp32 compute and scale, 32 MiB workspace (as the reference).
The library is the cuBLASLt torch already loaded in this process.
"""
from __future__ import annotations

import ctypes
import glob
import os
from pathlib import Path

import torch

CUBLAS_COMPUTE_32F = 68
CUDA_R_32F = 0
CUDA_R_16F = 2
CUDA_R_16BF = 14
PREF_MAX_WORKSPACE_BYTES = 1
WORKSPACE_BYTES = 32 << 20
_DT = {torch.float16: CUDA_R_16F, torch.bfloat16: CUDA_R_16BF}


class _Algo(ctypes.Structure):
    _fields_ = [("data", ctypes.c_uint64 * 8)]


class _Heur(ctypes.Structure):
    _fields_ = [("algo", _Algo), ("workspaceSize", ctypes.c_size_t), ("state", ctypes.c_int), ("wavesCount", ctypes.c_float),
                ("reserved", ctypes.c_int * 4)]


_LIB = None
_HANDLES: dict[int, ctypes.c_void_p] = {}


def _lib():
    global _LIB
    if _LIB is None:
        cands = glob.glob(os.path.join(os.path.dirname(torch.__file__), "..", "nvidia", "cublas", "lib",
                                       "libcublasLt.so*"))
        cands += ["libcublasLt.so.12", "libcublasLt.so"]
        err = None
        for c in cands:
            try:
                _LIB = ctypes.CDLL(str(Path(c).resolve()) if os.path.exists(c) else c)
                break
            except OSError as e:
                err = e
        if _LIB is None:
            raise RuntimeError(f"libcublasLt not loadable: {err}")
        V, P = ctypes.c_void_p, ctypes.POINTER
        _LIB.cublasLtCreate.argtypes = [P(V)]
        _LIB.cublasLtMatmulDescCreate.argtypes = [P(V), ctypes.c_int, ctypes.c_int]
        _LIB.cublasLtMatrixLayoutCreate.argtypes = [P(V), ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64]
        _LIB.cublasLtMatmulPreferenceCreate.argtypes = [P(V)]
        _LIB.cublasLtMatmulPreferenceSetAttribute.argtypes = [V, ctypes.c_int, V, ctypes.c_size_t]
        _LIB.cublasLtMatmulAlgoGetHeuristic.argtypes = [V, V, V, V, V, V, V, ctypes.c_int, P(_Heur), P(ctypes.c_int)]
        _LIB.cublasLtMatmul.argtypes = [V, V, V, V, V, V, V, V, V, V, V, V, P(_Algo), V, ctypes.c_size_t, V]
        for f in ("cublasLtMatmulDescDestroy", "cublasLtMatrixLayoutDestroy", "cublasLtMatmulPreferenceDestroy"):
            getattr(_LIB, f).argtypes = [V]
    return _LIB


def _check(st: int, what: str) -> None:
    if st != 0:
        raise RuntimeError(f"{what} failed: cublasStatus {st}")


def _handle(device: int) -> ctypes.c_void_p:
    if device not in _HANDLES:
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            _check(_lib().cublasLtCreate(ctypes.byref(h)), "cublasLtCreate")
        _HANDLES[device] = h
    return _HANDLES[device]


class _Problem:
    def __init__(self, M: int, N: int, K: int, dtype, device: int):
        lib = _lib()
        self.M, self.N, self.K, self.dtype, self.device = M, N, K, dtype, device
        self.desc = ctypes.c_void_p()
        _check(lib.cublasLtMatmulDescCreate(ctypes.byref(self.desc), CUBLAS_COMPUTE_32F, CUDA_R_32F), "DescCreate")
        dt = _DT[dtype]
        self.la, self.lb, self.lc = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib.cublasLtMatrixLayoutCreate(ctypes.byref(self.la), dt, N, K, N), "LayoutCreate(B)")
        _check(lib.cublasLtMatrixLayoutCreate(ctypes.byref(self.lb), dt, K, M, K), "LayoutCreate(A)")
        _check(lib.cublasLtMatrixLayoutCreate(ctypes.byref(self.lc), dt, N, M, N), "LayoutCreate(C)")
        self.alpha = ctypes.c_float(1.0)
        self.beta = ctypes.c_float(0.0)

    def heuristics(self, n: int) -> list[_Heur]:
        lib = _lib()
        pref = ctypes.c_void_p()
        _check(lib.cublasLtMatmulPreferenceCreate(ctypes.byref(pref)), "PreferenceCreate")
        ws = ctypes.c_uint64(WORKSPACE_BYTES)
        _check(lib.cublasLtMatmulPreferenceSetAttribute(pref, PREF_MAX_WORKSPACE_BYTES, ctypes.byref(ws), 8),
               "PreferenceSetAttribute")
        res = (_Heur * n)()
        cnt = ctypes.c_int(0)
        st = lib.cublasLtMatmulAlgoGetHeuristic(_handle(self.device), self.desc, self.la, self.lb, self.lc, self.lc, pref,
                                                n, res, ctypes.byref(cnt))
        lib.cublasLtMatmulPreferenceDestroy(pref)
        if st != 0:
            return []
        return [res[i] for i in range(cnt.value) if res[i].state == 0]


class CublasLtMatmul:
    """One heuristic algorithm of cuBLASLt for one problem, behind make_runner(a, b, out=None)."""

    family = "cublaslt"

    def __init__(self, problem: _Problem, heur: _Heur, rank: int):
        self.problem, self.algo, self.rank = problem, heur.algo, rank
        self.ws_bytes = int(heur.workspaceSize)
        self.key = f"h{rank}"
        self.cfg = {"heuristic_rank": rank, "workspace": self.ws_bytes, "waves": float(heur.wavesCount)}

    def make_runner(self, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None):
        p = self.problem
        assert a.is_contiguous() and b.is_contiguous() and a.shape == (p.M, p.K) and b.shape == (p.K, p.N)
        c = out if out is not None else torch.empty((p.M, p.N), device=a.device, dtype=a.dtype)
        ws = torch.empty(max(self.ws_bytes, 1), dtype=torch.uint8, device=a.device)
        lib, h = _lib(), _handle(p.device)
        algo = self.algo

        def run():
            st = lib.cublasLtMatmul(h, p.desc, ctypes.byref(p.alpha), b.data_ptr(), p.la, a.data_ptr(), p.lb,
                                    ctypes.byref(p.beta), c.data_ptr(), p.lc, c.data_ptr(), p.lc, ctypes.byref(algo),
                                    ws.data_ptr(), self.ws_bytes, torch.cuda.current_stream(a.device).cuda_stream)
            _check(st, "cublasLtMatmul")
            return c
        return run


def candidates(M: int, N: int, K: int, dtype=torch.float16, n: int = 16, device: int | None = None) -> list:
    """cuBLASLt's heuristic top-n for the shape (rank 0 = B2; the best over all of them = B3)."""
    device = torch.cuda.current_device() if device is None else device
    p = _Problem(M, N, K, dtype, device)
    return [CublasLtMatmul(p, h, i) for i, h in enumerate(p.heuristics(n))]
