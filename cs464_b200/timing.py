"""GPU timing protocol for candidates (the same TimingConfig / TimingResult / benchmark interface as tune/timing.py).

- CUDA events around each timed sample, never host wall-clock.
- The first call is untimed; then a time-based warm-up; then repeats until the relative standard error of the mean is
  below `target_rse`, or `max_reps` / `max_time_s` is reached. Raw samples are kept; the median is the statistic.
- cache_mode "cold": a buffer of max(8 x L2, 64 MiB) is overwritten before every sample, outside the timed interval;
  "hot": no flush.
- Before each chunk of samples a device-side sleep is queued, so the host enqueues the whole chunk while the GPU is
  busy and the events measure device time, not host launch latency (tune/timing.py:151-154 describes the same need).
- batch > 1 times `batch` back-to-back launches per sample; use_graph captures them in a CUDA graph, which requires
  the timed callable to enqueue only on the current stream and allocate nothing (B200Matmul runners qualify).
"""
from __future__ import annotations

import math
import time
from dataclasses import asdict, dataclass, field
from typing import Callable

import numpy as np
import torch

CACHE_MODES = ("cold", "hot")


@dataclass
class TimingConfig:
    cache_mode: str = "cold"
    warmup_ms: float = 25.0
    min_warmup_iters: int = 3
    min_reps: int = 10
    max_reps: int = 1000
    target_rse: float = 0.01
    max_time_s: float = 2.0
    batch: int = 1
    use_graph: bool = False
    flush_bytes: int | None = None
    keep_raw: bool = True

    def __post_init__(self):
        if self.cache_mode not in CACHE_MODES:
            raise ValueError(f"cache_mode must be one of {CACHE_MODES}, got {self.cache_mode!r}")
        if self.cache_mode == "cold" and self.batch != 1:
            raise ValueError("cold mode flushes L2 before each sample; batch > 1 would make launches 2..n hot")
        if self.batch < 1 or self.min_reps < 1 or self.max_reps < self.min_reps:
            raise ValueError("need batch >= 1 and 1 <= min_reps <= max_reps")


@dataclass
class TimingResult:
    """Microseconds per launch (sample time / batch)."""
    median_us: float
    mean_us: float
    std_us: float
    min_us: float
    max_us: float
    p10_us: float
    p25_us: float
    p75_us: float
    p90_us: float
    p99_us: float
    trimmed_mean_us: float  # mean of the middle 60 % of samples: finer than the median when samples are quantised
    n_samples: int
    rse: float
    converged: bool
    cache_mode: str
    batch: int
    use_graph: bool
    wall_s: float
    telemetry_before: dict = field(default_factory=dict)
    telemetry_after: dict = field(default_factory=dict)
    samples_us: list | None = None

    @property
    def iqr_us(self) -> float:
        return self.p75_us - self.p25_us

    def summary(self) -> dict:
        d = asdict(self)
        d.pop("samples_us")
        d["iqr_us"] = self.iqr_us
        return d


def summarize(samples_us, *, rse_target: float = 0.01) -> dict:
    s = np.asarray(samples_us, dtype=np.float64)
    n = len(s)
    mean = float(s.mean())
    std = float(s.std(ddof=1)) if n > 1 else 0.0
    rse = std / math.sqrt(n) / mean if n > 1 and mean > 0 else math.inf
    q = np.percentile(s, [10, 25, 50, 75, 90, 99])
    srt = np.sort(s)
    cut = int(0.2 * n)
    mid = srt[cut:n - cut] if n - 2 * cut > 0 else srt
    return {"median_us": float(q[2]), "mean_us": mean, "std_us": std, "min_us": float(s.min()), "max_us": float(s.max()),
            "p10_us": float(q[0]), "p25_us": float(q[1]), "p75_us": float(q[3]), "p90_us": float(q[4]),
            "p99_us": float(q[5]), "trimmed_mean_us": float(mid.mean()), "n_samples": n, "rse": rse,
            "converged": rse <= rse_target}


def pool(results: list[TimingResult], rse_target: float = 0.01) -> TimingResult:
    """Merge timings of one kernel taken on different input placements (their raw samples) into one result."""
    if len(results) == 1:
        return results[0]
    samples = [s for r in results for s in (r.samples_us or [])]
    stats = summarize(samples, rse_target=rse_target)
    stats["converged"] = all(r.converged for r in results)
    first, last = results[0], results[-1]
    return TimingResult(**stats, cache_mode=first.cache_mode, batch=first.batch, use_graph=first.use_graph,
                        wall_s=sum(r.wall_s for r in results), telemetry_before=first.telemetry_before,
                        telemetry_after=last.telemetry_after, samples_us=samples)


_FLUSH: dict[tuple[int, int], torch.Tensor] = {}
_SLEEP_HZ: dict[int, float] = {}


def _flusher(nbytes: int | None, device: int) -> Callable[[], None]:
    if nbytes is None:
        l2 = torch.cuda.get_device_properties(device).L2_cache_size
        nbytes = max(8 * l2, 64 * 2**20)
    key = (device, nbytes)
    if key not in _FLUSH:
        _FLUSH[key] = torch.empty(nbytes // 4, dtype=torch.int32, device=f"cuda:{device}")
    buf = _FLUSH[key]
    return buf.zero_


def _sleep_cycles_per_s(device: int) -> float:
    """Rate of torch.cuda._sleep's spin (cycles per second), measured once per device."""
    if device not in _SLEEP_HZ:
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cycles = 10_000_000
        torch.cuda._sleep(1000)
        s.record()
        torch.cuda._sleep(cycles)
        e.record()
        e.synchronize()
        _SLEEP_HZ[device] = cycles / (s.elapsed_time(e) / 1e3)
    return _SLEEP_HZ[device]


def _backlog(seconds: float, device: int) -> None:
    if seconds > 0:
        torch.cuda._sleep(int(min(seconds, 0.2) * _sleep_cycles_per_s(device)))


def gpu_telemetry(device: int | None = None) -> dict:
    """SM clock, temperature and power via NVML when available (best effort, never raises). `device`: the torch
    device index (default: the current device)."""
    try:
        if device is None:
            device = torch.cuda.current_device()
        import pynvml
        pynvml.nvmlInit()
        idx = device
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if uuid.replace("GPU-", "") in u:
                    idx = i
                    break
        except Exception:
            pass
        h = pynvml.nvmlDeviceGetHandleByIndex(idx)
        return {"sm_mhz": pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                "temp_c": pynvml.nvmlDeviceGetTemperature(h, pynvml.NVML_TEMPERATURE_GPU),
                "power_w": pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0,
                "throttle": int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))}
    except Exception:
        return {}


def benchmark(fn: Callable[[], object], cfg: TimingConfig | None = None, device: int | None = None) -> TimingResult:
    """Time `fn`, which must only enqueue GPU work on the current stream. `device`: the torch device index to time on
    (default: the current device, so a process driving GPU r keeps working on GPU r)."""
    cfg = cfg or TimingConfig()
    if device is None:
        device = torch.cuda.current_device()
    torch.cuda.set_device(device)
    flush = _flusher(cfg.flush_bytes, device) if cfg.cache_mode == "cold" else None

    fn()  # first call: plan set-up, never timed
    torch.cuda.synchronize()
    if cfg.use_graph:
        # Capture on a stream of this device: torch's default capture stream belongs to whichever GPU was current at
        # the process's first capture, and capturing on it would switch a process that drives GPU 1 to GPU 0.
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(device).wait_stream(side)
        # Captured directly: `torch.cuda.graph` also runs a full Python garbage collection and empties the allocator
        # cache before every capture, host work that dominated the selector's step for small shapes.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            graph.capture_begin()
            try:
                for _ in range(cfg.batch):
                    fn()
            finally:
                graph.capture_end()
        run = graph.replay
    elif cfg.batch > 1:
        def run():
            for _ in range(cfg.batch):
                fn()
    else:
        run = fn

    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(cfg.min_warmup_iters):
        if flush:
            flush()
        run()
    e.record()
    e.synchronize()
    est_ms = max(s.elapsed_time(e) / cfg.min_warmup_iters, 1e-3)
    for _ in range(min(int(cfg.warmup_ms / est_ms), 10_000)):
        if flush:
            flush()
        run()
    torch.cuda.synchronize()

    t0 = time.perf_counter()
    if flush:
        flush()
    run()
    enqueue_s = time.perf_counter() - t0
    torch.cuda.synchronize()

    tel_before = gpu_telemetry(device)
    samples: list[float] = []
    t_start = time.perf_counter()
    chunk = int(min(max(50.0 / est_ms, 5), 100))
    if not cfg.use_graph:
        chunk = min(chunk, max(1, 256 // cfg.batch))  # stay below the driver's pending-launch queue
    converged = False
    while True:
        n = min(chunk, cfg.max_reps - len(samples))
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        _backlog(2.0 * enqueue_s * n, device)
        for i in range(n):
            if flush:
                flush()
            starts[i].record()
            run()
            ends[i].record()
        ends[-1].synchronize()
        samples.extend(a.elapsed_time(b) * 1e3 / cfg.batch for a, b in zip(starts, ends))
        stats = summarize(samples, rse_target=cfg.target_rse)
        converged = len(samples) >= cfg.min_reps and stats["converged"]
        if converged or len(samples) >= cfg.max_reps or time.perf_counter() - t_start > cfg.max_time_s:
            break
    wall = time.perf_counter() - t_start
    stats = summarize(samples, rse_target=cfg.target_rse)
    stats["converged"] = converged
    return TimingResult(**stats, cache_mode=cfg.cache_mode, batch=cfg.batch, use_graph=cfg.use_graph, wall_s=wall,
                        telemetry_before=tel_before, telemetry_after=gpu_telemetry(device),
                        samples_us=samples if cfg.keep_raw else None)


# The short protocol of the online search (tune/online.py:47-55, :90-97): 10 cold samples, and a CUDA-graph pass of
# 20 launches x 5 samples for kernels under 50 us, where per-launch events cannot separate candidates.
SHORT_REPS = 10
SHORT_WARMUP_MS = 2.0
GRAPH_BATCH = 20
GRAPH_REPS = 5
SMALL_US = 50.0


def short_configs() -> tuple[TimingConfig, TimingConfig]:
    cold = TimingConfig(cache_mode="cold", warmup_ms=SHORT_WARMUP_MS, min_warmup_iters=1, min_reps=SHORT_REPS,
                        max_reps=SHORT_REPS, target_rse=1.0, max_time_s=1.0, keep_raw=False)
    graph = TimingConfig(cache_mode="hot", warmup_ms=SHORT_WARMUP_MS, min_warmup_iters=1, min_reps=GRAPH_REPS,
                         max_reps=GRAPH_REPS, target_rse=1.0, max_time_s=1.0, batch=GRAPH_BATCH, use_graph=True,
                         keep_raw=False)
    return cold, graph
