"""GPU parity tests: the sm_100a family, called through the C ABI, against the CPU oracle.

Ported in spirit from the reference's tests/test_kernels.py (hand-picked configs x its 8 shapes, split-K with uneven K,
bitwise split-K determinism, bf16) and tests/test_correctness.py (NaN-prefilled outputs, so unwritten elements fail).
Every result must pass both bounds, written here:
  * the reference's gate (tune/correctness.py:116-127): |C-ref| <= 1e-2*|ref| + 1e-2*sqrt(K) (bf16: 3e-2, 3e-2);
  * the north star's per-element bound: |C-ref|_ij <= 2e-3 * ||A_i,:||_2 * ||B_:,j||_2.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from cs464_b200.config_space import HANDPICKED, shape_violations
from cs464_b200.matmul import B200Matmul, MatmulConfig
from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
# the reference's kernel-test shapes (tests/test_kernels.py:10-11)
SHAPES = [(1, 1, 1), (1, 4096, 4096), (17, 33, 65), (128, 128, 128), (129, 257, 1031), (513, 255, 16),
          (2048, 2048, 8), (64, 64, 16384)]


def _run(cfg, a_cpu, b_cpu, *, a_dev=None, b_dev=None):
    """Run `cfg` on the operands (copied to the GPU unless device views are given) into a NaN-filled output."""
    a = a_dev if a_dev is not None else a_cpu.cuda()
    b = b_dev if b_dev is not None else b_cpu.cuda()
    out = torch.full((a.shape[0], b.shape[1]), float("nan"), device=a.device, dtype=a.dtype)
    run = B200Matmul(cfg).make_runner(a, b, out=out)
    c = run()
    torch.cuda.synchronize()
    run.raise_on_status()
    assert c.data_ptr() == out.data_ptr()
    return c, run


def _assert_parity(c, ref, a_cpu, b_cpu, K):
    c32 = c.float().cpu().numpy()
    dt = "bfloat16" if c.dtype == torch.bfloat16 else "float16"
    r = oracle.check_output(c32, ref, K, dt)
    assert r.valid, r
    ok, worst = oracle.norm_rel_check(c32, ref, a_cpu, b_cpu)
    assert ok, f"norm-relative error {worst:.3e} > {oracle.NORM_REL_TOL}"
    return worst


@pytest.mark.parametrize("name", list(HANDPICKED))
@pytest.mark.parametrize("shape", SHAPES)
def test_handpicked_matches_oracle(name, shape):
    cfg = HANDPICKED[name]
    M, N, K = shape
    if "split_k_workspace_too_large" in shape_violations(cfg, M, N, K):
        pytest.skip("workspace limit")
    a, b = oracle.make_inputs(M, N, K, seed=0)
    ref = oracle.gemm_f32(a, b)
    c, _ = _run(cfg, a, b)
    _assert_parity(c, ref, a, b, K)


@pytest.mark.parametrize("case", json.loads((GOLDEN / "gemm_cases.json").read_text())["cases"], ids=lambda c: c["name"])
@pytest.mark.parametrize("name", ["large_square", "skinny_m", "large_k_splitk"])
def test_golden_cases(case, name):
    """The reference's own fp32 results (tests/golden, made by running tune/correctness.py) as the oracle."""
    z = np.load(GOLDEN / "gemm_cases.npz")
    dt = torch.bfloat16 if case["dtype"] == "bfloat16" else torch.float16
    a = torch.from_numpy(z[f"{case['name']}_a"].view(np.int16)).view(dt)
    b = torch.from_numpy(z[f"{case['name']}_b"].view(np.int16)).view(dt)
    ref = z[f"{case['name']}_ref"]
    cfg = HANDPICKED[name]
    c, _ = _run(cfg, a, b)
    _assert_parity(c, ref, a, b, case["K"])


@pytest.mark.parametrize("split_k", [2, 4, 16])
@pytest.mark.parametrize("bm", [128, 16])
def test_split_k_uneven_k(split_k, bm):
    cfg = MatmulConfig(bm, 128 if bm < 128 else 64, 64, num_warps=4, num_stages=4, GROUP_M=1, SPLIT_K=split_k)
    a, b = oracle.make_inputs(100, 70, 1000, seed=0)
    c, _ = _run(cfg, a, b)
    _assert_parity(c, oracle.gemm_f32(a, b), a, b, 1000)


@pytest.mark.parametrize("split_k", [1, 3])
@pytest.mark.parametrize("cfg", [MatmulConfig(128, 128, 64, num_stages=4, GROUP_M=1),
                                 MatmulConfig(256, 256, 64, num_stages=3, GROUP_M=1),
                                 MatmulConfig(256, 128, 64, num_stages=4, GROUP_M=1, CLUSTER=2)],
                         ids=lambda c: c.key())
@pytest.mark.parametrize("shape", [(100, 72, 640), (300, 520, 700), (33, 136, 256)])
def test_staged_epilogue_edges(cfg, split_k, shape):
    """The epilogue that writes rows through shared memory, at C's edges: rows past M inside a 32-row slab, and a
    last 64-column group (32 for the fp32 split-K partials) holding only some 16-byte pieces. Every element must be
    written exactly as the oracle has it, none outside C (the output starts NaN and C is a view inside a larger
    NaN-filled buffer)."""
    M, N, K = shape
    cfg = MatmulConfig(cfg.BLOCK_M, cfg.BLOCK_N, cfg.BLOCK_K, num_warps=cfg.num_warps, num_stages=cfg.num_stages,
                       GROUP_M=cfg.GROUP_M, SPLIT_K=split_k, CLUSTER=cfg.CLUSTER)
    a_cpu, b_cpu = oracle.make_inputs(M, N, K, seed=7)
    big = torch.full((M + 3, N + 16), float("nan"), device="cuda", dtype=torch.float16)
    out = big[1:M + 1, 8:N + 8]  # 16-byte-aligned start, row stride N + 16 (a multiple of 8)
    run = B200Matmul(cfg).make_runner(a_cpu.cuda(), b_cpu.cuda(), out=out)
    c = run()
    torch.cuda.synchronize()
    run.raise_on_status()
    _assert_parity(c, oracle.gemm_f32(a_cpu, b_cpu), a_cpu, b_cpu, K)
    rest = big.clone()
    rest[1:M + 1, 8:N + 8] = 0
    assert torch.isnan(rest[0]).all() and torch.isnan(rest[M + 1:]).all()
    assert torch.isnan(rest[:, :8]).all() and torch.isnan(rest[:, N + 8:]).all()


@pytest.mark.parametrize("cfg", [MatmulConfig(256, 256, 64, num_stages=3, PERSISTENT=2),
                                 MatmulConfig(256, 256, 64, num_stages=6, CLUSTER=2, PERSISTENT=2),
                                 MatmulConfig(16, 256, 64, num_stages=6, GROUP_M=1, PERSISTENT=2)],
                         ids=lambda c: c.key())
def test_stream_k_deterministic_and_correct(cfg):
    """Few tiles, long K: every tile is split over several workers, so the owner fix-up does all the work; the
    result must match the oracle and be bitwise identical run to run (fixed K-order sums, no atomics)."""
    M, N, K = (1024, 1024, 8192) if cfg.BLOCK_M > 64 else (16, 2048, 16384)
    a, b = oracle.make_inputs(M, N, K, seed=4)
    run = B200Matmul(cfg).make_runner(a.cuda(), b.cuda())
    c1 = run().clone()
    c2 = run().clone()
    torch.cuda.synchronize()
    run.raise_on_status()
    assert torch.equal(c1, c2)
    _assert_parity(c1, oracle.reference_cpu(a, b).numpy(), a, b, K)


@pytest.mark.parametrize("cfg", [MatmulConfig(256, 256, 64, num_stages=3, PERSISTENT=2),
                                 MatmulConfig(256, 256, 128, num_stages=3, CLUSTER=2, PERSISTENT=2)],
                         ids=lambda c: c.key())
@pytest.mark.parametrize("shape", [(3328, 3328, 2048), (4096, 4096, 1024), (4096, 4096, 4096)])
def test_stream_k_schedules_at_wave_edges(cfg, shape):
    """Both stream-K cases: full data-parallel waves with the partial last wave's tiles split evenly in K (3328^2:
    169 tiles on 148 SMs; 4096^2 pairs: 256 tiles on 74 pairs), and plain data-parallel waves when the last wave is
    more than half full (4096^2 single CTAs: 256 tiles on 148 SMs). Outputs through the staged epilogue, owners adding
    their contributors' partials; bitwise stable run to run."""
    M, N, K = shape
    a, b = oracle.make_inputs(M, N, K, seed=5)
    run = B200Matmul(cfg).make_runner(a.cuda(), b.cuda())
    c1 = run().clone()
    c2 = run().clone()
    torch.cuda.synchronize()
    run.raise_on_status()
    assert torch.equal(c1, c2)
    _assert_parity(c1, oracle.reference_cpu(a, b).numpy(), a, b, K)


def test_split_k_deterministic():
    cfg = MatmulConfig(128, 128, 64, SPLIT_K=8)
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(256, 4096, device="cuda", generator=g).half()
    b = torch.randn(4096, 256, device="cuda", generator=g).half()
    run = B200Matmul(cfg).make_runner(a, b)
    c1 = run().clone()
    c2 = run().clone()
    assert torch.equal(c1, c2)


@pytest.mark.parametrize("name", ["medium", "skinny_m", "large_k_splitk"])
def test_bf16(name):
    a, b = oracle.make_inputs(300, 200, 500, dtype=torch.bfloat16, seed=0)
    c, _ = _run(HANDPICKED[name], a, b)
    _assert_parity(c, oracle.gemm_f32(a, b), a, b, 500)


@pytest.mark.parametrize("cfg", [
    MatmulConfig(128, 128, 64, num_stages=4),
    MatmulConfig(256, 128, 64, num_stages=4),
    MatmulConfig(128, 256, 128, num_stages=2, num_warps=8),
    MatmulConfig(256, 256, 64, num_stages=3, num_warps=8),
    MatmulConfig(128, 192, 64, num_stages=4),
    MatmulConfig(32, 256, 64, num_stages=4, GROUP_M=1),
    MatmulConfig(64, 128, 128, num_stages=4, GROUP_M=1),
    MatmulConfig(48, 128, 64, num_stages=4, GROUP_M=1),
    MatmulConfig(128, 128, 64, num_stages=4, PERSISTENT=0),
    MatmulConfig(128, 64, 128, num_stages=4, GROUP_M=4, SPLIT_K=3),
    MatmulConfig(256, 256, 64, num_stages=6, CLUSTER=2),
    MatmulConfig(256, 128, 64, num_stages=6, CLUSTER=2),
    MatmulConfig(256, 256, 128, num_stages=3, num_warps=8, CLUSTER=2),
    MatmulConfig(256, 192, 64, num_stages=6, CLUSTER=2),
    MatmulConfig(256, 256, 64, num_stages=6, SPLIT_K=3, GROUP_M=4, CLUSTER=2),
    MatmulConfig(256, 256, 64, num_stages=6, PERSISTENT=0, CLUSTER=2),
    MatmulConfig(32, 256, 128, num_stages=6, GROUP_M=1, CLUSTER=2),
    MatmulConfig(16, 256, 128, num_stages=6, GROUP_M=1, SPLIT_K=2, CLUSTER=2),
    MatmulConfig(256, 256, 64, num_stages=3, PERSISTENT=2),
    MatmulConfig(128, 128, 64, num_stages=6, PERSISTENT=2),
    MatmulConfig(128, 256, 64, num_stages=4, num_warps=8, PERSISTENT=2),
    MatmulConfig(256, 256, 64, num_stages=6, CLUSTER=2, PERSISTENT=2),
    MatmulConfig(16, 256, 64, num_stages=6, GROUP_M=1, PERSISTENT=2),
    MatmulConfig(32, 256, 128, num_stages=6, GROUP_M=1, CLUSTER=2, PERSISTENT=2),
], ids=lambda c: c.key())
@pytest.mark.parametrize("shape", [(300, 520, 700), (1024, 1024, 1024), (40, 1000, 3000)])
def test_knobs_match_oracle(cfg, shape):
    M, N, K = shape
    a, b = oracle.make_inputs(M, N, K, seed=1)
    c, _ = _run(cfg, a, b)
    _assert_parity(c, oracle.gemm_f32(a, b), a, b, K)


@pytest.mark.parametrize("layout", ["a_t", "b_t", "both_t", "a_offset", "b_strided"])
@pytest.mark.parametrize("name", ["medium", "skinny_m", "large_square"])
def test_layouts(layout, name):
    """Transposed views read MN-major or K-major in place; unaligned views go through the packing kernel."""
    M, N, K = 200, 256, 320
    a, b = oracle.make_inputs(M, N, K, seed=2)
    a_dev, b_dev = a.cuda(), b.cuda()
    if layout in ("a_t", "both_t"):
        a_dev = a_dev.t().contiguous().t()  # stride (1, M)
    if layout in ("b_t", "both_t"):
        b_dev = b_dev.t().contiguous().t()  # stride (1, K)
    if layout == "a_offset":
        buf = torch.empty(M * K + 1, device="cuda", dtype=a.dtype)
        a_dev = buf[1:].view(M, K)  # base 2 bytes off 16-byte alignment
        a_dev.copy_(a.cuda())
    if layout == "b_strided":
        buf = torch.empty(K, N * 2, device="cuda", dtype=b.dtype)
        b_dev = buf[:, ::2]  # stride (2N, 2)
        b_dev.copy_(b.cuda())
    c, _ = _run(HANDPICKED[name], a, b, a_dev=a_dev, b_dev=b_dev)
    _assert_parity(c, oracle.gemm_f32(a, b), a, b, K)


def test_empty_and_k_zero():
    cfg = HANDPICKED["medium"]
    a = torch.empty(0, 64, device="cuda", dtype=torch.float16)
    b = torch.empty(64, 32, device="cuda", dtype=torch.float16)
    assert B200Matmul(cfg).make_runner(a, b)().shape == (0, 32)
    a = torch.empty(5, 0, device="cuda", dtype=torch.float16)
    b = torch.empty(0, 7, device="cuda", dtype=torch.float16)
    c, _ = _run(cfg, a.cpu(), b.cpu())
    assert torch.equal(c, torch.zeros(5, 7, device="cuda", dtype=torch.float16))


@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (8192, 8192, 1024), (2048, 28672, 4096)])
def test_large_vs_cpu_reference(shape):
    """Large shapes against the reference's fp32 reference run on the host (torch CPU, all threads)."""
    M, N, K = shape
    a, b = oracle.make_inputs(M, N, K, seed=0)
    ref = oracle.reference_cpu(a, b).numpy()
    c, _ = _run(HANDPICKED["large_square"], a, b)
    _assert_parity(c, ref, a, b, K)


def test_square_16384_properties():
    """At the largest square size: every config family agrees with the fp32 GPU reference within the bound, and
    split-K is bitwise stable run to run."""
    M = N = K = 16384
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(M, K, device="cuda", generator=g).half()
    b = torch.randn(K, N, device="cuda", generator=g).half()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = a.float() @ b.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    an = a.float().norm(dim=1)
    bn = b.float().norm(dim=0)
    for cfg in (HANDPICKED["large_square"], MatmulConfig(256, 256, 64, num_stages=3, num_warps=8),
                MatmulConfig(128, 128, 64, num_stages=6, SPLIT_K=2),
                MatmulConfig(256, 256, 64, num_stages=6, SPLIT_K=2, CLUSTER=2)):
        run = B200Matmul(cfg).make_runner(a, b)
        c = run()
        torch.cuda.synchronize()
        run.raise_on_status()
        err = (c.float() - ref).abs()
        ratio = float((err / (an[:, None] * bn[None, :])).max())
        assert ratio <= oracle.NORM_REL_TOL, (cfg.key(), ratio)
        if cfg.SPLIT_K > 1:
            assert torch.equal(c, run())
        del c, err


def test_split_k_plan_replays_from_a_cuda_graph():
    """Split-K runners captured into a CUDA graph (as the timer does) give the same bits as a direct call: one launch of
    CTA clusters that sum the splits in shared memory, or (larger tiles, more than 8 splits) the GEMM and its reduce
    kernel, a programmatic dependent launch."""
    a_cpu, b_cpu = oracle.make_inputs(192, 256, 2048, seed=9)
    a, b = a_cpu.cuda(), b_cpu.cuda()
    ref = oracle.gemm_f32(a_cpu, b_cpu)
    for cfg in (MatmulConfig(128, 64, 64, num_stages=4, GROUP_M=1, SPLIT_K=4),
                MatmulConfig(128, 128, 64, num_stages=4, GROUP_M=1, SPLIT_K=4),
                MatmulConfig(128, 64, 64, num_stages=4, GROUP_M=1, SPLIT_K=12)):
        run = B200Matmul(cfg).make_runner(a, b)
        assert run.num_kernels == (1 if cfg.SPLIT_K <= 8 and cfg.BLOCK_N == 64 else 2)
        direct = run().clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            run()
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            g.capture_begin()
            run()
            g.capture_end()
        run.c.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        run.raise_on_status()
        assert torch.equal(run.c, direct)
        _assert_parity(run.c, ref, a_cpu, b_cpu, 2048)
        del g


# (config, (M, N, K), dtype, C's leading-dimension padding, B transposed in memory): split-K summed inside CTA clusters
CLUSTER_SPLITS = [
    (MatmulConfig(128, 64, 64, num_stages=4, GROUP_M=1, SPLIT_K=4), (512, 384, 2048), torch.float16, 0, False),
    (MatmulConfig(16, 128, 128, num_stages=6, GROUP_M=1, SPLIT_K=4), (24, 1000, 2048), torch.float16, 0, False),
    (MatmulConfig(32, 256, 64, num_stages=6, GROUP_M=1, SPLIT_K=8), (1, 2048, 4096), torch.float16, 0, False),
    (MatmulConfig(128, 64, 64, num_stages=6, GROUP_M=1, SPLIT_K=8), (256, 192, 256), torch.float16, 0, False),
    (MatmulConfig(128, 64, 64, num_stages=4, GROUP_M=8, SPLIT_K=3), (300, 520, 1000), torch.bfloat16, 0, False),
    (MatmulConfig(256, 32, 64, num_stages=4, GROUP_M=1, SPLIT_K=2), (512, 384, 2048), torch.float16, 0, True),
    (MatmulConfig(128, 64, 128, num_stages=3, GROUP_M=1, SPLIT_K=5), (256, 256, 2560), torch.float16, 8, False),
    (MatmulConfig(128, 64, 64, num_stages=6, GROUP_M=1, SPLIT_K=7, PERSISTENT=0), (200, 136, 3000), torch.float16,
     0, True),
    (MatmulConfig(64, 128, 64, num_stages=8, GROUP_M=1, SPLIT_K=6), (40, 264, 1536), torch.bfloat16, 16, False),
]


@pytest.mark.parametrize("case", range(len(CLUSTER_SPLITS)))
def test_split_k_cluster_sum_matches_the_reduce_kernel(case):
    """SPLIT_K <= 8 on tiles of at most 8192 outputs, with every cluster of the launch resident at once, runs as one
    launch whose CTA clusters sum the splits through shared memory, in the split order of the separate reduce kernel. Its output must equal, bit for bit, the workspace path's
    (the allocation-free entry point keeps that path: fp32 partials in its scratch, then the reduce kernel), and pass
    both bounds. Cases cover ragged tiles, splits with empty K ranges (8 splits of 4 K blocks), the skinny swapped
    form (C written along its columns), 256-row tiles, odd split counts, bf16, a padded C and a K-major B."""
    import ctypes

    from cs464_b200 import _abi
    from cs464_b200.matmul import problem
    cfg, (M, N, K), dt, pad, bt = CLUSTER_SPLITS[case]
    a_cpu, b_cpu = oracle.make_inputs(M, N, K, dtype=dt, seed=30 + case)
    a = a_cpu.cuda()
    b = b_cpu.t().contiguous().cuda().t() if bt else b_cpu.cuda()  # K-major B: a transposed view
    c_full = torch.full((M, N + pad), float("nan"), device="cuda", dtype=dt)
    c = c_full[:, :N]
    run = B200Matmul(cfg).make_runner(a, b, out=c)
    assert run.num_kernels == 1, "expected the single-launch cluster sum"
    run()
    torch.cuda.synchronize()
    run.raise_on_status()
    _assert_parity(c, oracle.gemm_f32(a_cpu, b_cpu), a_cpu, b_cpu, K)
    assert torch.isnan(c_full[:, N:]).all(), "wrote outside C"
    ref = torch.full_like(c_full, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = _abi.load()
    pr = problem(M, N, K, a.stride(), b.stride(), ref[:, :N].stride(), dt)
    rc = lib.b2g_gemm_noalloc(ctypes.byref(cfg.to_abi()), ctypes.byref(pr), a.data_ptr(), b.data_ptr(),
                              ref.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == _abi.B2G_OK, _abi.last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(c, ref[:, :N]), "cluster sum differs from the reduce kernel's bits"


def test_split_k_beyond_one_wave_of_clusters_keeps_the_reduce_kernel():
    """16 tiles x 8 splits need 16 clusters of 8 CTAs; a B200 holds 15 at once, so the plan keeps the GEMM + reduce
    kernel pair (a second wave of clusters measured slower); the result is the same either way."""
    cfg = MatmulConfig(32, 256, 64, num_stages=6, GROUP_M=1, SPLIT_K=8)
    a_cpu, b_cpu = oracle.make_inputs(1, 4096, 4096, seed=41)
    c, run = _run(cfg, a_cpu, b_cpu)
    assert run.num_kernels == 2
    _assert_parity(c, oracle.gemm_f32(a_cpu, b_cpu), a_cpu, b_cpu, 4096)
