"""The allocation-free entry point `b2g_gemm_noalloc`, called through the C ABI.

Some callers cannot allocate device memory: a plugin host that hands a library only its input and output buffers, a
process whose HBM another allocator has already reserved, or code running while a stream is captured in global mode.
For them the library keeps its split-K partials in a fixed 32 MiB scratch array instead of a caller workspace. Here
its output is compared with the regular entry point's (`b2g_plan_create` + `b2g_plan_launch` with a torch-allocated
workspace) on several calls in a row, and each result is also checked against the CPU oracle under the tolerances
the other GPU tests use. The calls use different shapes and split counts, so stale partials left in the shared
scratch by an earlier call would show up as errors. An empty K with SPLIT_K > 1 needs no partials at all and must be
accepted.

This file sorts last so a run that stops at the first failure has already run every other test; it also passes
alone in a fresh process (the first call sets the scratch address up).
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from cs464_b200 import _abi
from cs464_b200.matmul import B200Matmul, MatmulConfig, problem
from oracle import oracle

pytestmark = pytest.mark.gpu


def _noalloc(cfg: MatmulConfig, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, status: torch.Tensor) -> int:
    lib = _abi.load()
    M, K = a.shape
    N = b.shape[1]
    pr = problem(M, N, K, a.stride(), b.stride(), c.stride(), a.dtype)
    return lib.b2g_gemm_noalloc(ctypes.byref(cfg.to_abi()), ctypes.byref(pr), a.data_ptr(), b.data_ptr(),
                                c.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)


CALLS = [  # (config, (M, N, K), seed, dtype): run in this order, back to back
    (MatmulConfig(128, 128, 64, num_stages=6, GROUP_M=1, SPLIT_K=8), (512, 384, 4096), 0, torch.float16),
    (MatmulConfig(16, 128, 128, num_stages=6, GROUP_M=1, SPLIT_K=4), (24, 1000, 2048), 1, torch.float16),
    (MatmulConfig(128, 256, 64, num_stages=4, GROUP_M=8, SPLIT_K=3), (300, 520, 1000), 2, torch.bfloat16),
    (MatmulConfig(128, 128, 64, num_stages=6, GROUP_M=1, SPLIT_K=8), (512, 384, 4096), 3, torch.float16),
    (MatmulConfig(128, 128, 64, num_stages=6, GROUP_M=1, SPLIT_K=8), (64, 96, 0), 4, torch.float16),
]


def test_noalloc_matches_regular_entry_point_on_calls_in_a_row():
    dev = torch.device("cuda:0")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    results = []
    for cfg, (M, N, K), seed, dt in CALLS:
        a_cpu, b_cpu = oracle.make_inputs(M, N, K, dtype=dt, seed=seed)
        a, b = a_cpu.to(dev), b_cpu.to(dev)
        out = torch.full((M, N), float("nan"), device=dev, dtype=dt)
        rc = _noalloc(cfg, a, b, out, status)
        assert rc == _abi.B2G_OK, _abi.last_error()
        results.append((cfg, K, a_cpu, b_cpu, a, b, out))
    torch.cuda.synchronize()
    assert int(status.item()) == 0, _abi.status_string(int(status.item()))
    for cfg, K, a_cpu, b_cpu, a, b, out in results:
        expect = B200Matmul(cfg).make_runner(a, b)()  # regular entry point, torch-allocated workspace
        torch.cuda.synchronize()
        got32 = out.float().cpu().numpy()
        ref = oracle.gemm_f32(a_cpu, b_cpu)  # the CPU oracle, independent of both entry points
        dt = "bfloat16" if out.dtype == torch.bfloat16 else "float16"
        r = oracle.check_output(got32, ref, K, dt)
        assert r.valid, (cfg.key(), r)
        ok, worst = oracle.norm_rel_check(got32, ref, a_cpu, b_cpu)
        assert ok, (cfg.key(), worst)
        # same kernels, same reduction order: the two entry points agree bit for bit
        assert torch.equal(out, expect), cfg.key()


def test_noalloc_rejects_oversized_partials_and_staging():
    dev = torch.device("cuda:0")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    a = torch.zeros(1024, 1024, device=dev, dtype=torch.float16)
    b = torch.zeros(1024, 1024, device=dev, dtype=torch.float16)
    c = torch.zeros(1024, 1024, device=dev, dtype=torch.float16)
    # 16 splits x 1024 x 1024 fp32 partials = 64 MiB > 32 MiB
    rc = _noalloc(MatmulConfig(128, 128, 64, SPLIT_K=16), a, b, c, status)
    assert rc == _abi.B2G_ERR_WORKSPACE
    msg = _abi.last_error()
    assert "67108864" in msg and "33554432" in msg, msg
    # an operand whose leading dimension is not a multiple of 8 elements would need a staged copy
    a_odd = torch.zeros(64, 65, device=dev, dtype=torch.float16)
    b_odd = torch.zeros(65, 64, device=dev, dtype=torch.float16)
    c_odd = torch.zeros(64, 64, device=dev, dtype=torch.float16)
    assert _noalloc(MatmulConfig(128, 128, 64), a_odd, b_odd, c_odd, status) == _abi.B2G_ERR_UNSUPPORTED
    assert "operand_needs_staging" in _abi.last_error()
    # stream-K's fix-up flags need a zeroed workspace of the caller's
    assert _noalloc(MatmulConfig(128, 128, 64, PERSISTENT=2), a, b, c, status) == _abi.B2G_ERR_UNSUPPORTED
    assert "streamk" in _abi.last_error()
