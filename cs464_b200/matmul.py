"""The sm_100a GEMM family behind the reference's backend protocol: C[M,N] = A[M,K] @ B[K,N], fp16/bf16 in, fp32 acc.

Mirrors kernels/triton_matmul.py (the reference's hot path) so its callers drive this family unchanged:
  * `MatmulConfig` keeps the seven tunables and their meaning (kernels/triton_matmul.py:20-35) and `key()` keeps the
    reference's format; extra knobs (PERSISTENT, CLUSTER) are appended to the key only when they differ from their
    defaults.
  * `B200Matmul(cfg).make_runner(a, b, out=None)` allocates the output, split-K workspace and launch plan once and
    returns a zero-allocation closure that enqueues on the current stream (kernels/triton_matmul.py:103-147), so
    `tune/timing.py:benchmark` can capture it in a CUDA graph.
  * `matmul`, `even_k`, `grid` as in kernels/triton_matmul.py:95-100, :150-151.

There is no Triton, no CPU path and no other backend here: the kernels are the hand-written sm_100a CUDA in
`cs464_b200/csrc` reached through the C ABI of include/b2g.h. Unsupported (config, shape) pairs raise
`Unsupported` ("unsupported: <rule>"), which the reference's gate records as an invalid candidate
(tune/correctness.py:147-149).
"""
from __future__ import annotations

import ctypes
import threading
import weakref
from collections import OrderedDict
from dataclasses import asdict, dataclass, fields

import torch

from cs464_b200 import _abi

_DTYPES = {torch.float16: _abi.DTYPE_F16, torch.bfloat16: _abi.DTYPE_BF16}

# extension knobs: key suffix letter -> (field, default)
EXTENSIONS = {"p": ("PERSISTENT", 1), "c": ("CLUSTER", 1)}


@dataclass(frozen=True)
class MatmulConfig:
    """One kernel variant. BLOCK_M x BLOCK_N output tile, BLOCK_K K step, num_warps epilogue warps (4 or 8),
    num_stages shared-memory ring depth, GROUP_M L2 tile grouping, SPLIT_K deterministic K splits. BLOCK_M <= 64 runs
    the operand-swapped skinny form. PERSISTENT=1: one CTA per SM slot walks the tiles; 0: one CTA per (tile, split),
    the reference's grid (kernels/triton_matmul.py:99-100); 2: stream-K, persistent workers split tiles x K blocks
    evenly and finish split tiles in K order (deterministic, needs SPLIT_K=1). CLUSTER=2: a pair of CTAs on two SMs
    computes each tile with M=256 tcgen05 MMAs (BLOCK_M = 256, or BLOCK_N = 256 in the skinny form), each CTA loading
    half of A and half of B."""
    BLOCK_M: int
    BLOCK_N: int
    BLOCK_K: int
    num_warps: int = 4
    num_stages: int = 4
    GROUP_M: int = 8
    SPLIT_K: int = 1
    PERSISTENT: int = 1
    CLUSTER: int = 1

    def key(self) -> str:
        k = (f"bm{self.BLOCK_M}_bn{self.BLOCK_N}_bk{self.BLOCK_K}_w{self.num_warps}_s{self.num_stages}"
             f"_g{self.GROUP_M}_sk{self.SPLIT_K}")
        for letter, (name, default) in EXTENSIONS.items():
            v = getattr(self, name)
            if v != default:
                k += f"_{letter}{v}"
        return k

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "MatmulConfig":
        names = {f.name for f in fields(cls)}
        return cls(**{k: int(v) for k, v in d.items() if k in names})

    def to_abi(self) -> _abi.Config:
        c = _abi.Config()
        c.block_m, c.block_n, c.block_k = self.BLOCK_M, self.BLOCK_N, self.BLOCK_K
        c.num_warps, c.num_stages, c.group_m, c.split_k = self.num_warps, self.num_stages, self.GROUP_M, self.SPLIT_K
        c.schedule = {0: _abi.SCHED_TILE, 1: _abi.SCHED_PERSISTENT, 2: _abi.SCHED_STREAMK}[self.PERSISTENT]
        c.cluster = self.CLUSTER
        return c


def even_k(K: int, cfg: MatmulConfig) -> bool:
    """True when K splits into whole BLOCK_K steps per split (kernels/triton_matmul.py:95-96). The sm_100a kernel
    needs no specialisation for it: TMA fills the K tail with zeros."""
    return K % (cfg.BLOCK_K * cfg.SPLIT_K) == 0


def grid(M: int, N: int, cfg: MatmulConfig) -> tuple[int, int]:
    """Work units (output tiles, splits), the reference's grid (kernels/triton_matmul.py:99-100). With PERSISTENT=1
    the launch uses min(units, SM slots) CTAs that walk these units."""
    return (-(-M // cfg.BLOCK_M)) * (-(-N // cfg.BLOCK_N)), cfg.SPLIT_K


def problem(M: int, N: int, K: int, a_strides, b_strides, c_strides, dtype: torch.dtype) -> _abi.Problem:
    p = _abi.Problem()
    p.M, p.N, p.K = M, N, K
    p.stride_am, p.stride_ak = a_strides
    p.stride_bk, p.stride_bn = b_strides
    p.stride_cm, p.stride_cn = c_strides
    p.dtype = _DTYPES[dtype]
    return p


def check_config(cfg: MatmulConfig, M: int, N: int, K: int, dtype: torch.dtype = torch.float16) -> str | None:
    """None if the family can run `cfg` on an (M, N, K) row-major problem, else the rule that rejects it (host only)."""
    lib = _abi.load()
    buf = ctypes.create_string_buffer(256)
    pr = problem(M, N, K, (K, 1), (N, 1), (N, 1), dtype)
    rc = lib.b2g_check(ctypes.byref(cfg.to_abi()), ctypes.byref(pr), buf, 256)
    return None if rc == _abi.B2G_OK else buf.value.decode()


def workspace_bytes(cfg: MatmulConfig, M: int, N: int, K: int, dtype: torch.dtype = torch.float16) -> int:
    lib = _abi.load()
    n = ctypes.c_size_t(0)
    pr = problem(M, N, K, (K, 1), (N, 1), (N, 1), dtype)
    _abi.check(lib.b2g_workspace_size(ctypes.byref(cfg.to_abi()), ctypes.byref(pr), None, None, ctypes.byref(n)),
               "b2g_workspace_size")
    return n.value


class _Runner:
    """The closure `make_runner` returns: calling it enqueues the plan on the current stream and returns C."""

    __slots__ = ("_launch", "_plan", "_device", "c", "status", "num_kernels", "grid", "_keep", "_fin", "__weakref__")

    def __init__(self, plan: ctypes.c_void_p, device: torch.device, c: torch.Tensor, status: torch.Tensor, keep):
        lib = _abi.load()
        self._launch = lib.b2g_plan_launch
        self._plan = plan
        self._device = device
        self.c = c
        self.status = status
        self.num_kernels = lib.b2g_plan_num_kernels(plan)
        self.grid = lib.b2g_plan_grid(plan)
        self._keep = keep
        self._fin = weakref.finalize(self, lib.b2g_plan_destroy, plan)

    def __call__(self) -> torch.Tensor:
        rc = self._launch(self._plan, torch.cuda.current_stream(self._device).cuda_stream)
        if rc:
            _abi.check(rc, "b2g_plan_launch")
        return self.c

    def device_status(self) -> int:
        """The kernels' device status word (0 = ok; else a bounded wait ran out). Synchronises."""
        return int(self.status.item())

    def raise_on_status(self) -> None:
        s = self.device_status()
        if s:
            raise RuntimeError(f"b200 kernel status 0x{s:x}: {_abi.status_string(s)}")


class B200Matmul:
    """Backend with the reference's protocol: `family`, `cfg`, `make_runner(a, b, out=None) -> Callable[[], Tensor]`
    (tune/runner.py:35-39). Pre-allocates output, workspace and plan so the launch closure allocates nothing."""

    family = "b200_sm100a_v1"

    def __init__(self, cfg: MatmulConfig | dict, wait_limit_us: int = 0):
        """`wait_limit_us`: limit of the kernels' bounded device waits (0: the library's default of one second);
        single-CTA configs only. Not part of the config's identity."""
        self.cfg = cfg if isinstance(cfg, MatmulConfig) else MatmulConfig.from_dict(cfg)
        self.wait_limit_us = int(wait_limit_us)

    @property
    def key(self) -> str:
        return self.cfg.key()

    def make_runner(self, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> _Runner:
        cfg = self.cfg
        assert a.ndim == 2 and b.ndim == 2 and a.shape[1] == b.shape[0], (a.shape, b.shape)
        assert a.dtype == b.dtype and a.dtype in _DTYPES, a.dtype
        if not (a.is_cuda and b.is_cuda and a.device == b.device):
            raise ValueError("B200Matmul needs both operands on the same CUDA device (there is no CPU path)")
        M, K = a.shape
        N = b.shape[1]
        dev = a.device
        c = out if out is not None else torch.empty((M, N), device=dev, dtype=a.dtype)
        if c.shape != (M, N) or c.dtype != a.dtype or c.device != dev:
            raise ValueError(f"out must be a {M}x{N} {a.dtype} tensor on {dev}")
        lib = _abi.load()
        pr = problem(M, N, K, a.stride(), b.stride(), c.stride(), a.dtype)
        acfg = cfg.to_abi()
        acfg.wait_limit_us = self.wait_limit_us
        n = ctypes.c_size_t(0)
        with torch.cuda.device(dev):
            _abi.check(lib.b2g_workspace_size(ctypes.byref(acfg), ctypes.byref(pr), a.data_ptr(), b.data_ptr(),
                                              ctypes.byref(n)), "b2g_workspace_size")
            # zeroed: the stream-K fix-up flags at its start must be 0 before the first launch
            ws = torch.zeros(n.value, dtype=torch.uint8, device=dev) if n.value else None
            status = torch.zeros(1, dtype=torch.int32, device=dev)
            plan = ctypes.c_void_p()
            _abi.check(lib.b2g_plan_create(ctypes.byref(acfg), ctypes.byref(pr), a.data_ptr(), b.data_ptr(),
                                           c.data_ptr(), ws.data_ptr() if ws is not None else None, n.value,
                                           status.data_ptr(), ctypes.byref(plan)), "b2g_plan_create")
        return _Runner(plan, dev, c, status, (a, b, ws))


def matmul(a: torch.Tensor, b: torch.Tensor, cfg: MatmulConfig) -> torch.Tensor:
    return B200Matmul(cfg).make_runner(a, b)()


_ABI_CFG: dict = {}
_STATUS: dict = {}
PLAN_CACHE_SIZE = 64  # plans kept per thread (each holds its tensor maps and, for split-K / staging, a workspace)


def status_word(device: torch.device) -> torch.Tensor:
    """A per-device int32 status word shared by one-shot launches (`gemm`); read it with `check_status`."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(key)
    if t is None:
        t = _STATUS[key] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
    return t


def check_status(device: torch.device | int | None = None) -> None:
    """Raise if a one-shot launch (`gemm`, the torch.matmul dispatcher) on `device` (default: every device used so
    far) gave up a bounded device wait since the last check, and clear the word. Synchronises with the device. A
    routed call returns without reading it (that would cost a host sync per call): call this at a sync point."""
    devs = list(_STATUS) if device is None else [torch.device("cuda", device).index if isinstance(device, int)
                                                 else (device.index if device.index is not None
                                                       else torch.cuda.current_device())]
    for d in devs:
        t = _STATUS.get(d)
        if t is None:
            continue
        code = int(t.item())
        if code:
            t.zero_()
            raise RuntimeError(f"b200 kernel status 0x{code:x} on cuda:{d}: {_abi.status_string(code)} "
                               "(results of launches since the last check may be incomplete)")


class _Plans(threading.local):
    def __init__(self):
        self.plans: OrderedDict = OrderedDict()


_PLANS = _Plans()


class _CachedPlan:
    __slots__ = ("plan", "ws", "_fin", "__weakref__")

    def __init__(self, plan: ctypes.c_void_p, ws):
        self.plan = plan
        self.ws = ws
        self._fin = weakref.finalize(self, _abi.load().b2g_plan_destroy, plan)


def gemm(cfg: MatmulConfig, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """One-shot C = A @ B on the current stream: the path of per-call dispatch. A launch plan (tensor maps, grid,
    workspace) is kept per thread for each (config, shape, strides, dtype, device, stream, pointer alignment); a
    call with new buffers re-points it (`b2g_plan_rebind`: re-encodes only the tensor maps whose operand moved) and
    launches. The output is fresh each call unless `out` is given. The device status word is not read here
    (`check_status`)."""
    M, K = a.shape
    N = b.shape[1]
    c = out if out is not None else torch.empty((M, N), device=a.device, dtype=a.dtype)
    lib = _abi.load()
    dev = a.device.index if a.device.index is not None else torch.cuda.current_device()
    stream = torch.cuda.current_stream(a.device).cuda_stream
    pa, pb, pc = a.data_ptr(), b.data_ptr(), c.data_ptr()
    key = (cfg, M, N, K, a.stride(), b.stride(), c.stride(), a.dtype, dev, stream, pa & 15, pb & 15, pc & 15)
    plans = _PLANS.plans
    ent = plans.get(key)
    if ent is not None:
        plans.move_to_end(key)
        rc = lib.b2g_plan_rebind(ent.plan, pa, pb, pc)
        if rc:
            plans.pop(key)
            ent = None
    if ent is None:
        acfg = _ABI_CFG.get(cfg)
        if acfg is None:
            acfg = _ABI_CFG[cfg] = cfg.to_abi()
        pr = problem(M, N, K, a.stride(), b.stride(), c.stride(), a.dtype)
        n = ctypes.c_size_t(0)
        _abi.check(lib.b2g_workspace_size(ctypes.byref(acfg), ctypes.byref(pr), pa, pb, ctypes.byref(n)),
                   "b2g_workspace_size")
        ws = torch.zeros(n.value, dtype=torch.uint8, device=a.device) if n.value else None
        plan = ctypes.c_void_p()
        _abi.check(lib.b2g_plan_create(ctypes.byref(acfg), ctypes.byref(pr), pa, pb, pc,
                                       ws.data_ptr() if ws is not None else None, n.value,
                                       status_word(a.device).data_ptr(), ctypes.byref(plan)), "b2g_plan_create")
        ent = plans[key] = _CachedPlan(plan, ws)
        while len(plans) > PLAN_CACHE_SIZE:
            plans.popitem(last=False)
    _abi.check(lib.b2g_plan_launch(ent.plan, stream), "b2g_plan_launch")
    return c
