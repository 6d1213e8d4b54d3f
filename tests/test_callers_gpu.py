"""GPU tests of the hot path's callers driving the sm_100a family: gate sensitivity (the reference's
tests/test_correctness.py), timer accuracy (tests/test_timing.py), first-use selection with the winner cache, the
full-space screen, one sharded-search step, and torch.matmul routing."""
from __future__ import annotations

import math
import time

import pytest
import torch

from cs464_b200 import dispatch, gate
from cs464_b200.baselines import TorchMatmul
from cs464_b200.config_space import HANDPICKED
from cs464_b200.matmul import B200Matmul, MatmulConfig
from cs464_b200.search import screen_shape, select_kernel, shape_space
from cs464_b200.timing import Protocol, measure_us
from cs464_b200.keys import parse_key as parse_key_
from cs464_b200.winner_cache import WinnerCache, environment

pytestmark = pytest.mark.gpu


class _Fn:
    def __init__(self, fn):
        self.fn = fn

    def make_runner(self, a, b, out=None):
        return lambda: self.fn(a, b, out)


def test_gate_passes_the_family_and_catches_mistakes():
    assert gate.validate(B200Matmul(HANDPICKED["medium"]), 129, 257, 1031, norm_rel=True).valid

    def bad_tile(a, b, out):
        gate.reference(a, b).to(out.dtype).clone()
        out.copy_(a @ b)
        out[64:80, 32:48] += 1.0
        return out
    r = gate.validate(_Fn(bad_tile), 128, 128, 4096)
    assert not r.valid and r.failure_reason == "tolerance_exceeded"

    def partial(a, b, out):
        out[:-1] = a[:-1] @ b
        return out
    r = gate.validate(_Fn(partial), 65, 64, 64)
    assert not r.valid and r.failure_reason.startswith("non_finite")


def test_fp16_accumulation_error_far_above_fp32_accumulation():
    M, N, K = 64, 64, 16384
    a, b = gate.make_inputs(M, N, K)
    ref = gate.reference(a, b)

    def fp16_acc(a, b):
        acc = torch.zeros(M, N, device=a.device, dtype=torch.float16)
        for k in range(0, K, 16):
            acc += a[:, k:k + 16] @ b[k:k + 16]
        return acc
    ours = B200Matmul(HANDPICKED["large_k_splitk"]).make_runner(a, b)()
    rms = lambda c: float((c.float() - ref).pow(2).mean().sqrt())  # noqa: E731
    assert rms(fp16_acc(a, b)) > 5 * rms(ours)


def test_timer_recovers_a_known_sleep():
    """A device spin of a known length (calibrated here against a long one) is measured within 25 %: the gate makes
    the events see device time, not the host's launch rate."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(1000)
    s.record()
    torch.cuda._sleep(10_000_000)
    e.record()
    e.synchronize()
    cycles_per_us = 10_000_000 / (s.elapsed_time(e) * 1e3)
    n = int(200 * cycles_per_us)
    r = measure_us(lambda: torch.cuda._sleep(n), Protocol(mode="hot", samples=20, max_samples=50))
    assert 150 <= r.median_us <= 260, r.median_us
    assert r.dropped == 0


def test_burst_hot_and_cold_modes_on_the_family():
    a, b = gate.make_inputs(1024, 1024, 1024)
    run = B200Matmul(MatmulConfig(128, 128, 64, num_stages=6)).make_runner(a, b)
    single = measure_us(run, Protocol(mode="hot", samples=20, max_samples=50)).median_us
    burst = measure_us(run, Protocol(mode="hot", burst=20, samples=10, max_samples=20)).median_us
    cold = measure_us(run, Protocol(mode="cold", samples=20, max_samples=30)).median_us
    assert burst <= single * 1.1
    assert single <= cold * 1.05


def test_gate_keeps_a_slow_host_out_of_the_samples():
    """Samples queued behind the gate measure the kernel even when the host takes far longer than the kernel to
    enqueue each one (a 200 us host delay per call around a ~10 us GEMM)."""
    a, b = gate.make_inputs(512, 512, 512)
    run = B200Matmul(MatmulConfig(128, 128, 64, num_stages=6)).make_runner(a, b)
    fast = measure_us(run, Protocol(mode="hot", samples=20, max_samples=20)).median_us

    def slow():
        t = time.perf_counter()
        while time.perf_counter() - t < 200e-6:
            pass
        return run()
    slowed = measure_us(slow, Protocol(mode="hot", samples=20, max_samples=20)).median_us
    assert slowed <= fast * 1.3 + 1.0, (fast, slowed)


def test_select_kernel_searches_then_hits_the_cache(tmp_path):
    wc = WinnerCache(tmp_path / "wc.jsonl", env=environment())
    r1 = select_kernel(None, 777, 512, 1024, cache=wc)
    # the ranker's top 3 and the zero-search rule's config (unless the ranker already proposed it)
    assert not r1["cached"] and r1["choice"]["key"] is not None and len(r1["candidates"]) in (3, 4)
    assert all(c["valid"] for c in r1["candidates"]), r1["candidates"]
    r2 = select_kernel(None, 777, 512, 1024, cache=wc)
    assert r2["cached"] and r2["choice"]["key"] == r1["choice"]["key"]
    r3 = select_kernel(None, 777, 512, 1024, cache=wc, frequent=True)  # wider search than the cached one: searched
    assert not r3["cached"] and len(r3["candidates"]) in (5, 6)


def test_screen_shape_small_pool():
    pool = shape_space(512, 512, 512)[::97][:12]
    s = screen_shape(512, 512, 512, pool)
    assert s["best_key"] is not None and s["n_configs"] == len(pool)
    assert all(r["status"] in ("ok", "slow") or r["status"].startswith("invalid") for r in s["rows"])
    assert all(not r["status"].startswith("invalid") for r in s["rows"]), s["rows"]


def test_sharded_search_units_on_the_gpu(tmp_path):
    """Two shapes, each cut into two screen slices, run through the real unit search on this GPU: every unit
    validates and times its slice plus the ranker's top 3, and the per-GPU gap combination gives each shape a best
    config and a gap >= 0; the winners reach the winner cache."""
    from cs464_b200 import shard
    shapes = [{"M": 96, "N": 640, "K": 512}, {"M": 512, "N": 256, "K": 1024}]
    units = [{"u": 2 * i + j, "i": i, "slice": j, "of": 2, "cost": 1.0} for i in range(2) for j in range(2)]
    queue = tmp_path / "queue.jsonl"
    shard.ShapeQueue.create(queue, shapes, space=12, units=units)
    st = shard.run_rank(0, str(queue), str(tmp_path), str(tmp_path / "wc.jsonl"), k=3, space=12,
                        cache_env=environment())
    assert st["units"] == 4 and st["shapes_finished"] == 2
    s = shard.summarize(str(tmp_path))
    assert s["shapes"] == 2
    for r in s["results"]:
        assert r["best_key"] is not None and r["gap"] is not None and r["gap"] >= 0.0 and r["n_screened"] >= 12
    assert len(WinnerCache(tmp_path / "wc.jsonl", env=environment())) == 2


def test_dispatch_routes_a_cached_winner(tmp_path):
    wc = WinnerCache(tmp_path / "wc.jsonl", env=environment())
    M, N, K = 384, 640, 512
    wc.put(M, N, K, "fp16", k=3, choice={"key": HANDPICKED["medium"].key(), "us": 5.0, "family": "b200_sm100a_v1"},
           extra={"torch_us": 100.0})
    a, b = gate.make_inputs(M, N, K)
    dispatch.enable(cache=wc)
    try:
        c = torch.matmul(a, b)
        assert dispatch.stats()["routed"] == 1
        assert gate.check_norm_relative(c, gate.reference(a, b), a, b).valid
        x = a.clone().requires_grad_(True)
        y = (x @ b).float().sum()
        y.backward()
        assert dispatch.stats()["routed"] == 2
        assert torch.allclose(x.grad.float(), b.float().sum(1).expand(M, K), rtol=1e-2, atol=1e-1)
        a2, b2 = gate.make_inputs(100, 100, 100)
        torch.matmul(a2, b2)                          # no cache entry: torch
        assert dispatch.stats()["torch"] >= 1
    finally:
        dispatch.disable()


def test_torch_baseline_backend():
    a, b = gate.make_inputs(64, 48, 32)
    assert gate.validate(TorchMatmul(), 64, 48, 32, inputs=(a, b)).valid


def test_cublaslt_comparator_candidates_valid():
    from cs464_b200 import cublaslt
    for M, N, K in [(1, 4096, 4096), (129, 256, 1032), (512, 512, 512)]:
        cs = cublaslt.candidates(M, N, K, n=8)
        assert cs and cs[0].cfg["heuristic_rank"] == 0
        a, b = gate.make_inputs(M, N, K)
        for c in cs:
            assert gate.validate(c, M, N, K, inputs=(a, b), norm_rel=True).valid, (M, N, K, c.key)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_timing_and_selection_stay_on_the_current_device():
    """A process that drives GPU 1 (a torchrun rank, a shard worker) times and selects on GPU 1: the timer does not
    switch the process back to GPU 0 behind the caller's back."""
    from cs464_b200.keys import parse_key
    from cs464_b200.search import FAMILY, choose, measure
    make_inputs, reference = gate.make_inputs, gate.reference
    prev = torch.cuda.current_device()
    try:
        torch.cuda.set_device(1)
        a, b = make_inputs(256, 256, 256, torch.float16)
        assert a.device.index == 1
        keys = ["bm128_bn128_bk64_w4_s4_g8_sk1", "bm128_bn64_bk64_w4_s4_g8_sk1"]
        r = measure(256, 256, 256, torch.float16, [(FAMILY, k, B200Matmul(parse_key(k))) for k in keys],
                    inputs=(a, b, reference(a, b)))
        assert choose(r["candidates"])["key"] in keys
        assert torch.cuda.current_device() == 1
    finally:
        torch.cuda.set_device(prev)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_plan_refuses_to_launch_on_another_device():
    """A runner made for GPU 1 raises instead of launching while GPU 0 is current."""
    from cs464_b200 import _abi
    prev = torch.cuda.current_device()
    try:
        torch.cuda.set_device(1)
        a, b = gate.make_inputs(128, 128, 128, torch.float16)
        run = B200Matmul(MatmulConfig(128, 128, 64)).make_runner(a, b)
        run()
        torch.cuda.synchronize()
        torch.cuda.set_device(0)
        with pytest.raises(_abi.B2GError, match="plan was made on device 1"):
            run()
    finally:
        torch.cuda.set_device(prev)


def test_dispatch_host_overhead(tmp_path):
    """Host time per torch.matmul call with routing on (the reference's tests/test_lscli_client.py:349-387): an
    undispatched call (fp32, or non-contiguous fp16) costs at most 5 us more than the unpatched function, and a
    dispatched call at most 20 us more than the family's own make_runner + call. Median of 2,000 calls, synchronising
    every 200 so the launch queue never fills."""
    wc = WinnerCache(tmp_path / "wc.jsonl", env=environment())
    key = "bm128_bn128_bk64_w4_s6_g8_sk1"
    wc.put(128, 128, 128, "fp16", k=3, choice={"key": key, "family": "b200_sm100a_v1", "us": 3.0},
           extra={"torch_us": 40.0})
    a32 = torch.randn(64, 64, device="cuda")
    h = torch.randn(128, 128, device="cuda", dtype=torch.float16)
    hn = torch.randn(64, 64, device="cuda", dtype=torch.float16).t()
    orig = torch.matmul

    def per_call(f, x, n=2000, sync_every=200):
        ts = []
        for i in range(n):
            t = time.perf_counter_ns()
            f(x, x)
            ts.append(time.perf_counter_ns() - t)
            if (i + 1) % sync_every == 0:
                torch.cuda.synchronize()
        ts.sort()
        return ts[len(ts) // 2] / 1e3
    base32, base_nc = per_call(orig, a32), per_call(orig, hn)
    dispatch.enable(cache=wc)
    try:
        patched32, patched_nc = per_call(torch.matmul, a32), per_call(torch.matmul, hn)
        be = B200Matmul(parse_key_(key))
        direct = per_call(lambda x, y: be.make_runner(x, y)(), h)
        patched_hit = per_call(torch.matmul, h)
        assert dispatch.stats()["routed"] >= 2000
        print(f"\n[overhead] undispatched +{patched32 - base32:.2f} us (torch {base32:.2f} us), late exit "
              f"+{patched_nc - base_nc:.2f} us; dispatched {patched_hit:.2f} us vs make_runner+call {direct:.2f} us")
        assert patched32 - base32 <= 5.0 and patched_nc - base_nc <= 5.0
        assert patched_hit - direct <= 20.0
        torch.cuda.synchronize()
        dispatch.check_status()
        c = torch.matmul(h, h)
        assert gate.check_norm_relative(c, gate.reference(h, h), h, h).valid
    finally:
        dispatch.disable()


def test_one_shot_plans_are_rebound_to_new_buffers():
    """The cached one-shot path: the same shape on new buffers (and a split-K config with its workspace) gives the
    oracle's answer every time; a pointer with another alignment class gets a plan of its own."""
    from cs464_b200.matmul import gemm
    for cfg in (MatmulConfig(128, 128, 64, num_stages=6), MatmulConfig(128, 128, 64, num_stages=4, SPLIT_K=4)):
        for seed in range(3):
            a, b = gate.make_inputs(200, 136, 1024, seed=seed)
            c = gemm(cfg, a, b)
            assert gate.check_norm_relative(c, gate.reference(a, b), a, b).valid, (cfg.key(), seed)
    buf = torch.empty(200 * 1024 + 8, device="cuda", dtype=torch.float16)
    a, b = gate.make_inputs(200, 136, 1024, seed=7)
    a_off = buf[8:].view(200, 1024)  # 16 bytes in: same class as a fresh tensor
    a_off.copy_(a)
    c = gemm(MatmulConfig(128, 128, 64, num_stages=6), a_off, b)
    assert gate.check_norm_relative(c, gate.reference(a, b), a, b).valid

