"""Device timing of GEMM candidates: CUDA events around each sample, queued behind a gate the host releases.

How a measurement runs (`measure_us(fn, protocol)`):
  1. `fn()` once untimed (plan set-up, first-touch), then `protocol.warmup` untimed launches.
  2. Samples go in chunks. For each chunk the timer queues a one-thread gate kernel that spins on a flag in mapped
     host memory (`b2g_hold`, bounded), then queues every sample of the chunk: [L2 flush,] start event, `fn()` x
     burst, end event. Only then does it set the flag. The GPU finds the whole chunk queued, so the events measure
     device time whatever the host's launch rate, with no calibration of a spin loop. A gate that ran out of time
     (the host stalled for a second) marks the chunk's samples unreliable and they are dropped.
  3. mode "cold": before every sample a buffer of twice the L2 size is overwritten with a new value (outside the
     event pair); "hot": back to back. `burst` > 1 times that many launches per sample (hot only) — the way to
     resolve kernels shorter than the event clock's ~1 us granularity.
  4. Stop when the median's 95 % confidence interval (distribution-free, from order statistics: Conover,
     Practical Nonparametric Statistics, 3rd ed., sec. 3.2) is narrower than `ci_target` of the median, or at
     `max_samples` / `max_s`. The result carries the median, the mean of the middle 60 % (finer than the median
     when samples fall on the event clock's grid) and every sample.

`fn` must only enqueue work on the current stream of the timed device and allocate nothing (B200Matmul runners and
`torch.matmul(..., out=)` qualify). The short protocols of the online search: `SHORT_COLD` (10 cold samples) and,
for kernels under `SMALL_US`, `SHORT_BURST` (5 samples of 20 back-to-back launches) — the reference's
tune/online.py:47-55 counts. Kernels of `LONG_US` or more are also timed by `sustained(us)`: back-to-back launches
for `SUSTAIN_S` first, so the samples see the clock the 1000 W power cap settles at. A B200 keeps its top clock for
a few milliseconds of dense tensor work only; among long GEMMs the fastest in a short cold sample (per clock) and the
fastest under a sustained load (per joule) can differ.
"""
from __future__ import annotations

import ctypes
import math
import time
from dataclasses import dataclass, field, replace
from typing import Callable

import numpy as np
import torch

MODES = ("cold", "hot")
HOLD_TIMEOUT_NS = 2_000_000_000
SMALL_US = 50.0


@dataclass(frozen=True)
class Protocol:
    mode: str = "cold"
    samples: int = 10          # at least this many
    max_samples: int = 200
    warmup: int = 2            # untimed launches after the first call
    burst: int = 1             # launches per sample (hot mode only)
    ci_target: float = 0.01    # stop once the median's 95 % CI spans less than this fraction of it
    max_s: float = 2.0         # wall-time bound on the sampling
    chunk: int = 32            # samples queued behind one gate

    def __post_init__(self):
        if self.mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}, got {self.mode!r}")
        if self.mode == "cold" and self.burst != 1:
            raise ValueError("a cold sample flushes L2 first; launches 2..burst of a burst would run hot")
        if not (1 <= self.samples <= self.max_samples) or self.burst < 1 or self.chunk < 1:
            raise ValueError("need 1 <= samples <= max_samples, burst >= 1 and chunk >= 1")


SHORT_COLD = Protocol(mode="cold", samples=10, max_samples=10, warmup=1, ci_target=math.inf, max_s=1.0)
SHORT_BURST = Protocol(mode="hot", samples=5, max_samples=5, warmup=1, burst=20, ci_target=math.inf, max_s=1.0)
LONG_US = 1000.0
SUSTAIN_S = 0.3


def sustained(us: float) -> Protocol:
    """Protocol for a kernel of about `us` microseconds (>= LONG_US): SUSTAIN_S of untimed back-to-back launches, then
    5 samples of about 20 ms of back-to-back launches each (a kernel this long fills L2 and more by itself, so no
    flush is needed between launches)."""
    us = max(us, 1.0)
    return Protocol(mode="hot", samples=5, max_samples=5, warmup=max(1, int(SUSTAIN_S * 1e6 / us)),
                    burst=max(1, int(round(20_000.0 / us))), ci_target=math.inf, max_s=10.0)


@dataclass
class Timing:
    """Microseconds per launch (a sample's time / burst)."""
    median_us: float
    trimmed_us: float           # mean of the middle 60 % of the samples
    mean_us: float
    min_us: float
    max_us: float
    ci_rel: float               # width of the median's 95 % CI / median
    n: int
    converged: bool
    mode: str
    burst: int
    wall_s: float
    dropped: int = 0            # samples discarded because their gate timed out
    telemetry: dict = field(default_factory=dict)
    samples_us: list | None = None

    def summary(self) -> dict:
        d = dict(self.__dict__)
        d.pop("samples_us")
        return d


def median_ci(sorted_x: np.ndarray, z: float = 1.959964) -> tuple[float, float]:
    """Distribution-free CI of the median from order statistics: ranks n/2 -/+ z*sqrt(n)/2 (normal approximation of
    the binomial(n, 1/2) count below the median)."""
    n = len(sorted_x)
    if n < 6:
        return float(sorted_x[0]), float(sorted_x[-1])
    half = z * math.sqrt(n) / 2.0
    lo = max(0, int(math.floor(n / 2.0 - half)))
    hi = min(n - 1, int(math.ceil(n / 2.0 + half)) - 1)
    return float(sorted_x[lo]), float(sorted_x[hi])


def describe(samples_us) -> dict:
    x = np.sort(np.asarray(samples_us, dtype=np.float64))
    n = len(x)
    med = float(np.median(x))
    cut = n // 5
    mid = x[cut:n - cut] if n - 2 * cut > 0 else x
    lo, hi = median_ci(x)
    return {"median_us": med, "trimmed_us": float(mid.mean()), "mean_us": float(x.mean()), "min_us": float(x[0]),
            "max_us": float(x[-1]), "ci_rel": (hi - lo) / med if med > 0 else math.inf, "n": n}


def merge(results: list[Timing]) -> Timing:
    """One timing from several measurements of the same kernel (e.g. at different input placements): their samples
    pooled; converged only if every part was."""
    if len(results) == 1:
        return results[0]
    pooled = [s for r in results for s in (r.samples_us or [])]
    d = describe(pooled)
    return Timing(**d, converged=all(r.converged for r in results), mode=results[0].mode, burst=results[0].burst,
                  wall_s=sum(r.wall_s for r in results), dropped=sum(r.dropped for r in results),
                  telemetry=results[-1].telemetry, samples_us=pooled)


class _DeviceState:
    """Per-device timer state: the host-released gate flag, the gate's status word and the L2 flush buffer."""

    def __init__(self, device: int):
        from cs464_b200 import _abi
        self.lib = _abi.load()
        self.device = device
        h, d = ctypes.c_void_p(), ctypes.c_void_p()
        with torch.cuda.device(device):
            _abi.check(self.lib.b2g_host_flag_create(ctypes.byref(h), ctypes.byref(d)), "b2g_host_flag_create")
            self.status = torch.zeros(1, dtype=torch.int32, device=f"cuda:{device}")
            l2 = torch.cuda.get_device_properties(device).L2_cache_size
            self.flush_buf = torch.empty(max(2 * l2, 1 << 24) // 4, dtype=torch.int32, device=f"cuda:{device}")
        self.host_flag, self.dev_flag = h, d
        self.epoch = 0
        self.flushes = 0

    def flush(self) -> None:
        self.flushes += 1
        self.flush_buf.fill_(self.flushes & 0x7FFFFFFF)

    def gate(self, stream) -> int:
        """Queue a closed gate on `stream`; returns the value that opens it."""
        self.epoch += 1
        self.lib.b2g_host_flag_set(self.host_flag, self.epoch - 1)
        rc = self.lib.b2g_hold(self.dev_flag, self.epoch, HOLD_TIMEOUT_NS, ctypes.c_void_p(self.status.data_ptr()),
                               ctypes.c_void_p(stream.cuda_stream))
        if rc:
            from cs464_b200 import _abi
            _abi.check(rc, "b2g_hold")
        return self.epoch

    def open(self, value: int) -> None:
        self.lib.b2g_host_flag_set(self.host_flag, value)

    def gate_timed_out(self) -> bool:
        bad = int(self.status.item()) != 0
        if bad:
            self.status.zero_()
        return bad


_STATE: dict[int, _DeviceState] = {}


def _state(device: int) -> _DeviceState:
    st = _STATE.get(device)
    if st is None:
        st = _STATE[device] = _DeviceState(device)
    return st


def telemetry(device: int | None = None) -> dict:
    """SM clock (MHz), temperature (C), power (W) and the clock-event reason mask of the timed GPU through NVML,
    matched by UUID; {} when NVML is unavailable. Never raises."""
    try:
        import pynvml
        if device is None:
            device = torch.cuda.current_device()
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(device).uuid).replace("GPU-", "")
        handle = None
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            u = pynvml.nvmlDeviceGetUUID(h)
            if uuid in (u.decode() if isinstance(u, bytes) else u):
                handle = h
                break
        if handle is None:
            return {}
        return {"sm_mhz": pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM),
                "temp_c": pynvml.nvmlDeviceGetTemperature(handle, pynvml.NVML_TEMPERATURE_GPU),
                "power_w": pynvml.nvmlDeviceGetPowerUsage(handle) / 1000.0,
                "reasons": int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle))}
    except Exception:
        return {}


def measure_us(fn: Callable[[], object], protocol: Protocol = Protocol(), device: int | None = None,
               keep_samples: bool = True) -> Timing:
    """Time `fn` on `device` (default: the current device) by `protocol`."""
    if device is None:
        device = torch.cuda.current_device()
    st = _state(device)
    stream = torch.cuda.current_stream(device)
    cold = protocol.mode == "cold"
    with torch.cuda.device(device):
        fn()
        for _ in range(protocol.warmup):
            if cold:
                st.flush()
            fn()
        torch.cuda.synchronize(device)
        tel = telemetry(device)
        samples: list[float] = []
        dropped = 0
        t0 = time.perf_counter()
        converged = False
        # a closed gate holds every launch queued behind it: keep a chunk well inside the driver's queue of
        # pending launches (~1k), counting up to three kernels per call of fn, or the host would block on a full
        # queue until the gate's time limit
        chunk = max(1, min(protocol.chunk, 240 // (3 + 3 * protocol.burst)))
        while True:
            n = min(chunk, protocol.max_samples - len(samples))
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
            key = st.gate(stream)
            for s, e in ev:
                if cold:
                    st.flush()
                s.record(stream)
                for _ in range(protocol.burst):
                    fn()
                e.record(stream)
            st.open(key)
            ev[-1][1].synchronize()
            got = [s.elapsed_time(e) * 1e3 / protocol.burst for s, e in ev]
            if st.gate_timed_out():
                dropped += len(got)
            else:
                samples.extend(got)
            if len(samples) >= protocol.samples:
                d = describe(samples)
                converged = d["ci_rel"] <= protocol.ci_target
                if converged or len(samples) >= protocol.max_samples:
                    break
            if time.perf_counter() - t0 > protocol.max_s or len(samples) + dropped >= 4 * protocol.max_samples:
                break
        wall = time.perf_counter() - t0
    if not samples:
        raise RuntimeError("timing gate timed out on every chunk: the host could not queue the samples in time")
    d = describe(samples)
    return Timing(**d, converged=converged, mode=protocol.mode, burst=protocol.burst, wall_s=wall, dropped=dropped,
                  telemetry=tel, samples_us=samples if keep_samples else None)


def with_samples(protocol: Protocol, n: int) -> Protocol:
    """`protocol` with exactly n samples."""
    return replace(protocol, samples=n, max_samples=n)
