"""The reference's own callers drive the sm_100a family unchanged, registered the way the integration notes describe.

Runs where a checkout of the reference is available: the directory named by $CS464_REFERENCE, else a `reference`
directory next to this repository's root. Skipped elsewhere (the GPU box has no such checkout, and nothing of it is
copied here): the reference's modules are imported from their own tree.

Registration, as a maintainer would do it: the reference's `tune.sweep.parse_key`, `tune.runner`'s family class,
config table and shape rules, and `tune.winner_cache.kernel_src_hash` point at this package. Then the reference's
  * `tune.runner.candidates_for("triton:handpicked" / "triton:<key>")` builds B200Matmul candidates,
  * `tune.winner_cache.backend_for(choice)` rebuilds one from a stored key,
  * `tune.correctness.validate` runs one into its NaN-filled output and judges it (and catches a wrong one),
  * `tune.online.measure` + `choose` validate, time and pick among them.
No GPU is here, so — as in the reference's own tests/test_online_split.py — the device is faked at its edges: the C
library's plan/launch entry points compute the GEMM on the host (the C oracle, from the pointers and strides the
backend passes through the ABI), operands are host tensors that report themselves as CUDA, and the stream and
synchronise calls are no-ops; the reference's `tune.timing.benchmark` is replaced by a counter that calls the runner.
Everything between the reference's callers and the C ABI — configs, keys, output and workspace ownership, the runner
closure, the status word — is the real code. The same protocol runs on the GPU in tests/test_callers_gpu.py.
"""
from __future__ import annotations

import contextlib
import ctypes
import itertools
import os
import sys
import types
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
REF = Path(os.environ.get("CS464_REFERENCE") or ROOT.parent / "reference")
pytestmark = pytest.mark.skipif(not (REF / "tune" / "correctness.py").is_file(),
                                reason="no checkout of the reference (set CS464_REFERENCE)")

REF_PACKAGES = ("tune", "kernels", "baselines", "analysis", "lscli", "suites", "results")


class CudaLike(torch.Tensor):
    """A host tensor that answers is_cuda: the backend's device checks pass, its data stays in host memory."""

    @property
    def is_cuda(self):  # noqa: D401
        return True


def _cuda_like(t: torch.Tensor) -> torch.Tensor:
    return t.as_subclass(CudaLike)


class FakeDeviceLib:
    """The C ABI with the device half computed on the host: host-only entry points go to the real library,
    plan_create records the pointers and strides, plan_launch computes C = A @ B with the C oracle into them."""

    def __init__(self, real, corrupt: bool = False):
        self.real = real
        self.plans: dict[int, dict] = {}
        self.launches = 0
        self.corrupt = corrupt
        self._ids = itertools.count(1)

    def __getattr__(self, name):
        return getattr(self.real, name)

    def b2g_plan_create(self, cfg, prob, A, B, C, ws, ws_bytes, status, out):
        pr = prob._obj
        rc = self.real.b2g_check(cfg, prob, None, 0)  # the same rules the device path enforces
        if rc:
            return rc
        h = next(self._ids)
        self.plans[h] = {"M": pr.M, "N": pr.N, "K": pr.K, "A": A, "B": B, "C": C,
                         "sa": (pr.stride_am, pr.stride_ak), "sb": (pr.stride_bk, pr.stride_bn),
                         "sc": (pr.stride_cm, pr.stride_cn), "bf16": pr.dtype == 1}
        out._obj.value = h
        return 0

    def b2g_plan_launch(self, plan, stream):
        from oracle import oracle
        p = self.plans[plan if isinstance(plan, int) else plan.value]
        M, N, K = p["M"], p["N"], p["K"]

        def view(addr, rows, cols, strides):
            span = (rows - 1) * strides[0] + (cols - 1) * strides[1] + 1 if rows and cols else 0
            buf = np.ctypeslib.as_array((ctypes.c_uint16 * max(span, 1)).from_address(addr))
            return np.lib.stride_tricks.as_strided(buf, (rows, cols), (strides[0] * 2, strides[1] * 2))
        a = view(p["A"], M, K, p["sa"])
        b = view(p["B"], K, N, p["sb"])
        c = view(p["C"], M, N, p["sc"])
        res = oracle.round_to(oracle.gemm_f32(a, b), p["bf16"])
        if self.corrupt:
            res[: min(M, 16), : min(N, 16)] ^= 0x0400  # flip an exponent bit in one tile
        c[...] = res
        self.launches += 1
        return 0

    def b2g_plan_num_kernels(self, plan):
        return 1

    def b2g_plan_grid(self, plan):
        return 1

    def b2g_plan_destroy(self, plan):
        return 0


@pytest.fixture
def ref_env(monkeypatch):
    """The reference importable, registered with this family, and the device faked at its edges."""
    monkeypatch.syspath_prepend(str(REF))
    before = set(sys.modules)
    from cs464_b200 import _abi, config_space, keys, winner_cache
    from cs464_b200.matmul import B200Matmul
    fake = FakeDeviceLib(_abi.load())
    monkeypatch.setattr(_abi, "load", lambda: fake)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "device", lambda *a, **k: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: types.SimpleNamespace(cuda_stream=0))

    import tune.correctness
    import tune.online
    import tune.runner
    import tune.sweep
    import tune.winner_cache
    # registration: the family class, its config table and shape rules, the key codec
    # and the source hash the reference's callers look up
    import kernels.config_space
    import kernels.triton_matmul
    monkeypatch.setattr(kernels.triton_matmul, "TritonMatmul", B200Matmul)
    monkeypatch.setattr(kernels.config_space, "HANDPICKED", config_space.HANDPICKED)
    monkeypatch.setattr(kernels.config_space, "shape_violations", config_space.shape_violations)
    monkeypatch.setattr(tune.sweep, "parse_key", keys.parse_key)
    monkeypatch.setattr(tune.winner_cache, "kernel_src_hash", winner_cache.kernel_src_hash)
    yield types.SimpleNamespace(fake=fake, B200Matmul=B200Matmul, correctness=tune.correctness,
                                online=tune.online, runner=tune.runner, winner_cache=tune.winner_cache,
                                HANDPICKED=config_space.HANDPICKED)
    for name in list(sys.modules):
        if name not in before and name.split(".")[0] in REF_PACKAGES:
            del sys.modules[name]


def _inputs(M, N, K, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).half()
    b = torch.randn(K, N, generator=g).half()
    return _cuda_like(a), _cuda_like(b)


def test_reference_candidates_and_backend_for_build_b200matmul(ref_env):
    cands = ref_env.runner.candidates_for("triton:handpicked", 300, 200, 500)
    assert cands and all(isinstance(c.backend, ref_env.B200Matmul) for c in cands)
    assert all(c.family == "b200_sm100a_v1" for c in cands)
    one = ref_env.runner.candidates_for("triton:bm256_bn256_bk128_w4_s3_g8_sk1_c2", 4096, 4096, 4096)
    assert [c.config_key for c in one] == ["bm256_bn256_bk128_w4_s3_g8_sk1_c2"]
    be = ref_env.winner_cache.backend_for({"key": "bm128_bn128_bk64_w4_s6_g8_sk1", "family": "triton"}, 64, 64, 64)
    assert isinstance(be, ref_env.B200Matmul) and be.cfg.key() == "bm128_bn128_bk64_w4_s6_g8_sk1"
    from cs464_b200 import _abi
    assert ref_env.winner_cache.kernel_src_hash() == _abi.source_hash()  # stored keys name this library build


def test_reference_validate_runs_and_judges_b200matmul(ref_env):
    M, N, K = 96, 80, 256
    a, b = _inputs(M, N, K)
    ok = ref_env.correctness.validate(ref_env.B200Matmul(ref_env.HANDPICKED["medium"]), M, N, K,
                                      inputs=(a, b))
    assert ok.valid, ok
    assert ref_env.fake.launches == 1
    ref_env.fake.corrupt = True
    bad = ref_env.correctness.validate(ref_env.B200Matmul(ref_env.HANDPICKED["medium"]), M, N, K,
                                       inputs=(a, b))
    assert not bad.valid and bad.failure_reason == "tolerance_exceeded"
    # an unsupported config is an invalid candidate, as the reference's gate records compile failures
    from cs464_b200.matmul import MatmulConfig
    unsup = ref_env.correctness.validate(ref_env.B200Matmul(MatmulConfig(256, 256, 128, num_stages=8)), M, N, K,
                                         inputs=(a, b))
    assert not unsup.valid and "unsupported" in unsup.failure_reason


def test_reference_measure_and_choose_over_b200matmul(ref_env, monkeypatch):
    M, N, K = 128, 96, 512
    a, b = _inputs(M, N, K, seed=1)
    ref = ref_env.correctness.reference(a, b)
    keys = ["bm128_bn128_bk64_w4_s6_g8_sk1", "bm128_bn64_bk128_w4_s4_g4_sk1", "bm256_bn256_bk64_w4_s3_g8_sk1"]
    calls = []

    def fake_benchmark(fn, cfg=None, device=0):
        c = fn()          # the runner the reference's timer would time: it launches and returns C
        calls.append(c)
        return types.SimpleNamespace(median_us=10.0 + len(calls))
    monkeypatch.setattr("tune.timing.benchmark", fake_benchmark)
    from cs464_b200.keys import parse_key
    triton = [("triton", k, ref_env.B200Matmul(parse_key(k)), 0.0) for k in keys]
    r = ref_env.online.measure(M, N, K, torch.float16, [], triton, inputs=(a, b, ref))
    assert [c["config_key"] for c in r["candidates"]] == keys
    assert all(c["valid"] for c in r["candidates"]), r["candidates"]
    choice = ref_env.online.choose(r["candidates"], len(keys))
    assert choice["key"] in keys
    assert calls and all(tuple(c.shape) == (M, N) for c in calls)
