"""Opt-in routing of torch.matmul / torch.mm / Tensor.matmul / Tensor.__matmul__ to this family's cached winners.

The reference's lscli client patch does the same for its Triton family (lscli/client.py:82-113, :275-345, :432-483).
Routed calls: plain 2-D CUDA fp16/bf16 tensors of one dtype on the current device, contiguous, 16-byte aligned,
0 < M, N, K <= MAX_DIM, not under stream capture, torch.compile, tracing, autocast or forward-mode AD. A call is
dispatched when the winner cache holds an entry for (M, N, K, dtype) whose stored timings pass the dispatch rule:
torch takes at least `min_kernel_us` and the winner saves at least max(min_saving_us, 4 % of torch's time) (3 % when
the entry was timed under a declared clock lock) (lscli/client.py:52-57, :99-113). Everything else goes to torch.
Under autograd the forward runs the selected kernel and the backward the original torch matmul.

MAX_DIM is 65536: the kernels take any dimension below 2^31, and BASELINE.json config 4 needs N = 28672, above the
reference's 16384.

A routed call costs one plan lookup and one launch: plans are cached per thread and re-pointed at each call's buffers
(`cs464_b200.matmul.gemm`). It does not read the kernels' device status word (that would be a host sync per call):
`check_status()` raises if a bounded device wait ran out since the last check — call it at a sync point.
"""
from __future__ import annotations

import threading
import time
import warnings

import torch

from cs464_b200.keys import parse_key
from cs464_b200.matmul import check_status, gemm  # noqa: F401 (check_status is part of this module's API)

MAX_DIM = 65536
SAVING_FRAC_UNLOCKED = 0.04
SAVING_FRAC_LOCKED = 0.03
DEFAULTS = {"min_kernel_us": 10.0, "min_saving_us": 5.0, "search_on_miss": False}
_DTYPES = {torch.float16: "fp16", torch.bfloat16: "bf16"}
_PLAIN = (torch.Tensor, torch.nn.Parameter)
_ORIG: dict = {}
_LOCK = threading.Lock()
_STATE = None


def saving_frac(entry: dict) -> float:
    lock = str((entry.get("env") or {}).get("clock_lock") or "unlocked").strip().lower()
    return SAVING_FRAC_UNLOCKED if lock in ("unlocked", "none", "off", "0") else SAVING_FRAC_LOCKED


def dispatch_rule(entry: dict, settings: dict | None = None) -> bool:
    """Dispatch only when torch's time is at least min_kernel_us and the winner saves at least
    max(min_saving_us, saving_frac * torch_us). Entries without both timings are never dispatched."""
    s = {**DEFAULTS, **(settings or {})}
    t = entry.get("torch_us")
    w = entry.get("winner_us", (entry.get("choice") or {}).get("us"))
    if t is None or w is None or t < s["min_kernel_us"]:
        return False
    return t - w >= max(s["min_saving_us"], saving_frac(entry) * t)


class _Mm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, cfg):
        ctx.save_for_backward(a, b)
        return gemm(cfg, a, b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        mm = _ORIG["matmul"]
        ga = mm(g, b.t()) if ctx.needs_input_grad[0] else None
        gb = mm(a.t(), g) if ctx.needs_input_grad[1] else None
        return ga, gb, None


def _autocast_on() -> bool:
    try:
        return torch.is_autocast_enabled("cuda")
    except TypeError:
        return torch.is_autocast_enabled()


class _Dispatcher:
    def __init__(self, cache, settings: dict):
        self.cache = cache
        self.settings = {**DEFAULTS, **settings}
        self.decisions: dict[tuple, object] = {}
        self.disabled: set = set()
        self.deciding: set = set()
        self.checked = 0.0
        self.stats = {"routed": 0, "torch": 0}

    def _refresh(self):
        now = time.monotonic()
        if self.cache is not None and now - self.checked >= 1.0:
            self.checked = now
            if self.cache.refresh():
                self.decisions.clear()

    def route(self, a, b):
        if (torch.compiler.is_compiling() or torch.jit.is_tracing() or type(a) not in _PLAIN or type(b) not in _PLAIN
                or a.ndim != 2 or b.ndim != 2 or not a.is_cuda or not b.is_cuda or a.dtype not in _DTYPES
                or b.dtype is not a.dtype):
            return None
        M, K = a.shape
        K2, N = b.shape
        if K != K2 or not (0 < M <= MAX_DIM and 0 < N <= MAX_DIM and 0 < K <= MAX_DIM):
            return None
        if not a.is_contiguous() or not b.is_contiguous() or a.data_ptr() % 16 or b.data_ptr() % 16:
            return None
        dev = a.device.index
        if (b.device.index != dev or torch.cuda.current_device() != dev or torch.cuda.is_current_stream_capturing()
                or _autocast_on()):
            return None
        key = (M, N, K, _DTYPES[a.dtype], dev)
        self._refresh()
        if key in self.decisions:
            return self.decisions[key]
        return self._decide_once(key, a.dtype)

    def _decide_once(self, key, dtype):
        with _LOCK:
            if key in self.decisions:
                return self.decisions[key]
            if key in self.deciding:
                return None
            self.deciding.add(key)
        try:
            out = self._decide(key, dtype)
        except Exception as e:
            warnings.warn(f"cs464_b200.dispatch: selection for {key[:4]} failed ({type(e).__name__}: {e}); torch")
            out = None
        with _LOCK:
            self.deciding.discard(key)
            self.decisions[key] = out
        return out

    def _decide(self, key, dtype):
        if key in self.disabled or self.cache is None:
            return None
        M, N, K, dname, _ = key
        hit = self.cache.get(M, N, K, dname, k=1)
        if hit is None and self.settings["search_on_miss"]:
            from cs464_b200.search import select_kernel
            select_kernel(None, M, N, K, dtype=dtype, cache=self.cache, extra=lambda: {"torch_us": torch_time_us(
                M, N, K, dtype)})
            hit = self.cache.get(M, N, K, dname, k=1)
        if hit is None or (hit["choice"].get("family") or "b200_sm100a_v1") != "b200_sm100a_v1":
            return None
        if not dispatch_rule(hit, self.settings):
            return None
        return parse_key(hit["choice"]["key"])

    def matmul(self, orig, a, b):
        try:
            cfg = self.route(a, b)
        except Exception:
            cfg = None
        if cfg is None:
            self.stats["torch"] += 1
            return orig(a, b)
        try:
            self.stats["routed"] += 1
            if (a.requires_grad or b.requires_grad) and torch.is_grad_enabled():
                return _Mm.apply(a, b, cfg)
            return gemm(cfg, a, b)
        except Exception as e:
            key = (a.shape[0], b.shape[1], a.shape[1], _DTYPES[a.dtype], a.device.index)
            warnings.warn(f"cs464_b200.dispatch: kernel for {key[:4]} failed ({type(e).__name__}: {e}); torch")
            self.disabled.add(key)
            self.decisions[key] = None
            return orig(a, b)


def torch_time_us(M: int, N: int, K: int, dtype=torch.float16) -> float:
    """torch.matmul's short cold time for the shape (the dispatch rule's comparator), measured like the candidates."""
    from cs464_b200.baselines import TorchMatmul
    from cs464_b200.gate import make_inputs
    from cs464_b200.timing import SHORT_COLD, measure_us
    a, b = make_inputs(M, N, K, dtype)
    mm = _ORIG.get("matmul", torch.matmul)
    run = TorchMatmul().make_runner(a, b)
    if mm is not torch.matmul:
        c = torch.empty((M, N), device=a.device, dtype=dtype)
        run = lambda: mm(a, b, out=c)  # noqa: E731  (the unpatched function while dispatch is on)
    return measure_us(run, SHORT_COLD, keep_samples=False).median_us


def enable(cache=None, **settings) -> None:
    """Patch torch's 2-D matmul entry points. `cache`: a WinnerCache (default: the default file)."""
    global _STATE
    with _LOCK:
        if _STATE is not None:
            return
        if cache is None:
            from cs464_b200.winner_cache import WinnerCache, default_enabled
            cache = WinnerCache() if default_enabled() else None
        _STATE = _Dispatcher(cache, settings)
        _ORIG.update(matmul=torch.matmul, mm=torch.mm, t_matmul=torch.Tensor.matmul,
                     t_rmatmul=torch.Tensor.__matmul__)
        st = _STATE

        def matmul(a, b, *args, **kw):
            if args or kw:
                return _ORIG["matmul"](a, b, *args, **kw)
            return st.matmul(_ORIG["matmul"], a, b)

        def mm(a, b, *args, **kw):
            if args or kw:
                return _ORIG["mm"](a, b, *args, **kw)
            return st.matmul(_ORIG["mm"], a, b)

        def t_matmul(self, other):
            return st.matmul(_ORIG["t_matmul"], self, other)

        def t_rmatmul(self, other):
            return st.matmul(_ORIG["t_rmatmul"], self, other)

        torch.matmul = matmul
        torch.mm = mm
        torch.Tensor.matmul = t_matmul
        torch.Tensor.__matmul__ = t_rmatmul


def disable() -> None:
    global _STATE
    with _LOCK:
        if _STATE is None:
            return
        torch.matmul = _ORIG["matmul"]
        torch.mm = _ORIG["mm"]
        torch.Tensor.matmul = _ORIG["t_matmul"]
        torch.Tensor.__matmul__ = _ORIG["t_rmatmul"]
        _STATE = None


def is_enabled() -> bool:
    return _STATE is not None


def stats() -> dict:
    return dict(_STATE.stats) if _STATE is not None else {}
