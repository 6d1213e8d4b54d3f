"""Failure detection on the GPU without a fault: a bounded device wait that runs out.

Every wait of the kernels (mbarrier phases, stream-K flags) gives up after a limit, records a code in the caller's
status word, tells the CTA's other roles to stop, waits for its own copies and MMAs in flight, frees tensor memory and
returns. Here the limit is set to 1 us on a GEMM whose epilogue must wait tens of microseconds for its first tile, so
a wait runs out for certain. The test checks the status code, then that the same process still runs GEMMs that
match the oracle (the context was not lost). Nothing traps, asserts on the device or touches a bad address.
"""
from __future__ import annotations

import pytest
import torch

from cs464_b200 import _abi, gate
from cs464_b200.matmul import B200Matmul, MatmulConfig
from oracle import oracle

pytestmark = pytest.mark.gpu

TIMEOUT_CODES = {0x101, 0x102, 0x103}


def test_expired_wait_reports_status_and_context_survives():
    a, b = gate.make_inputs(2048, 2048, 16384)
    cfg = MatmulConfig(128, 128, 64, num_stages=4)
    run = B200Matmul(cfg, wait_limit_us=1).make_runner(a, b)
    run()
    torch.cuda.synchronize()  # the kernel returned: no hang, no sticky error
    code = run.device_status()
    assert code in TIMEOUT_CODES, hex(code)
    assert "timed out" in _abi.status_string(code)
    with pytest.raises(RuntimeError, match="status 0x10"):
        run.raise_on_status()
    # the status word is the caller's: cleared, the same runner times out again rather than hanging
    run.status.zero_()
    run()
    torch.cuda.synchronize()
    assert run.device_status() in TIMEOUT_CODES

    # the context is intact: the default limit on the same inputs, and a fresh small problem, match
    ok = B200Matmul(cfg).make_runner(a, b)
    c = ok()
    torch.cuda.synchronize()
    ok.raise_on_status()
    assert gate.check_norm_relative(c, gate.reference(a, b), a, b).valid
    a2, b2 = oracle.make_inputs(300, 200, 500, seed=3)
    c2 = B200Matmul(cfg).make_runner(a2.cuda(), b2.cuda())()
    r = oracle.check_output(c2.float().cpu().numpy(), oracle.gemm_f32(a2, b2), 500)
    assert r.valid, r


def test_gate_verdict_names_the_timeout():
    a, b = gate.make_inputs(1024, 1024, 16384)
    r = gate.validate(B200Matmul(MatmulConfig(128, 128, 64, num_stages=4), wait_limit_us=1), 1024, 1024, 16384,
                      inputs=(a, b))
    assert not r.valid and r.failure_reason.startswith("device_wait_timeout(0x10")
    assert not gate.context_poisoned(r.failure_reason)


def test_wait_limit_is_refused_for_cta_pairs():
    a, b = gate.make_inputs(512, 512, 512)
    with pytest.raises(_abi.Unsupported, match="wait_limit_single_cta_only"):
        B200Matmul(MatmulConfig(256, 256, 64, num_stages=6, CLUSTER=2), wait_limit_us=10).make_runner(a, b)
