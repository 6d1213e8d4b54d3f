"""The C-ABI library loads and exports every symbol include/b2g.h declares; host-only entry points answer without a
GPU (no compute call is made here)."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from cs464_b200 import _abi
from cs464_b200.build import LIB_PATH, source_hash
from cs464_b200.matmul import MatmulConfig, check_config, workspace_bytes

HEADER = Path(__file__).resolve().parent.parent / "include" / "b2g.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(b2g_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _abi.load()
    names = declared_functions()
    assert len(names) >= 16
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (b2g_[a-z0-9_]+)$", out, flags=re.M))
    assert set(names) <= exported, set(names) - exported
    assert set(_abi.EXPORTS) <= set(names)


def test_identity():
    lib = _abi.load()
    assert lib.b2g_abi_version() == 1
    assert lib.b2g_version().decode().startswith("b2g-sm100a")
    assert _abi.source_hash() == source_hash()
    assert lib.b2g_status_string(0) == b"ok"
    assert b"timed out" in lib.b2g_status_string(0x102)


@pytest.mark.parametrize("cfg,shape,reason", [
    (MatmulConfig(96, 64, 64), (64, 64, 64), "block_m_invalid"),
    (MatmulConfig(16, 64, 64), (16, 64, 64), "block_n_invalid"),
    (MatmulConfig(128, 136, 64), (64, 64, 64), "block_n_invalid"),
    (MatmulConfig(128, 128, 32), (64, 64, 64), "block_k_invalid"),
    (MatmulConfig(128, 128, 64, num_warps=2), (64, 64, 64), "num_warps_invalid"),
    (MatmulConfig(256, 256, 128, num_stages=4), (64, 64, 64), "smem_exceeds_limit"),
    (MatmulConfig(128, 128, 64, num_stages=1), (64, 64, 64), "num_stages_invalid"),
    (MatmulConfig(128, 128, 64, SPLIT_K=65), (64, 64, 64), "split_k_invalid"),
    (MatmulConfig(128, 128, 64, SPLIT_K=2, PERSISTENT=2), (64, 64, 64), "streamk_with_split_k"),
])
def test_check_rejects_with_named_rule(cfg, shape, reason):
    got = check_config(cfg, *shape)
    assert got is not None and got.startswith(reason), got


def test_check_accepts_handpicked():
    from cs464_b200.config_space import HANDPICKED
    for cfg in HANDPICKED.values():
        assert check_config(cfg, 1000, 1000, 1000) is None


def test_workspace_size():
    assert workspace_bytes(MatmulConfig(128, 128, 64), 512, 512, 512) == 0
    def r256(x):
        return -(-x // 256) * 256
    # SPLIT_K <= 8 on single-CTA tiles of at most 8192 outputs is summed inside a cluster of the tile's CTAs: no
    # partials, only staged operands (B here: N = 70 is not a multiple of 8, so rows of 72 elements, K = 1000 rows)
    assert workspace_bytes(MatmulConfig(128, 64, 64, SPLIT_K=4), 100, 70, 1000) == r256(1000 * 72 * 2)
    assert workspace_bytes(MatmulConfig(128, 64, 64, SPLIT_K=4), 128, 64, 1024) == 0
    assert workspace_bytes(MatmulConfig(16, 128, 128, num_stages=6, GROUP_M=1, SPLIT_K=4), 24, 1000, 2048) == 0
    assert workspace_bytes(MatmulConfig(128, 64, 64, num_stages=6, GROUP_M=1, SPLIT_K=2), 512, 256, 2048) == 0
    # otherwise the second kernel sums fp32 partials [SPLIT_K, M, N] from the workspace: larger tiles, more than 8
    # splits, CTA pairs, and launches with more clusters than fit at once
    assert workspace_bytes(MatmulConfig(128, 128, 64, SPLIT_K=4), 100, 70, 1000) == r256(4 * 100 * 70 * 4) + r256(
        1000 * 72 * 2)
    assert workspace_bytes(MatmulConfig(128, 64, 64, SPLIT_K=16), 128, 64, 1024) == r256(16 * 128 * 64 * 4)
    assert workspace_bytes(MatmulConfig(256, 128, 64, num_stages=6, SPLIT_K=2, CLUSTER=2), 512, 256, 1024) == r256(
        2 * 512 * 256 * 4)
    # the clusters of one launch must all fit on the GPU at once (33 clusters of 4 CTAs on a B200): 32 tiles do,
    # 512 tiles would need further waves of clusters and keep the reduce kernel
    assert workspace_bytes(MatmulConfig(128, 64, 64, SPLIT_K=4, PERSISTENT=0), 512, 512, 1024) == 0
    assert workspace_bytes(MatmulConfig(128, 64, 64, SPLIT_K=4, PERSISTENT=0), 2048, 2048, 1024) == r256(
        4 * 2048 * 2048 * 4)
    # 16 tiles x 8 splits: more clusters of 8 than a B200 holds at once (15)
    assert workspace_bytes(MatmulConfig(32, 256, 64, SPLIT_K=8), 1, 4096, 4096) == r256(8 * 1 * 4096 * 4)
    lib = _abi.load()
    n = ctypes.c_size_t()
    pr = _abi.Problem(M=17, N=33, K=65, stride_am=65, stride_ak=1, stride_bk=33, stride_bn=1, stride_cm=33,
                      stride_cn=1, dtype=0)
    assert lib.b2g_workspace_size(ctypes.byref(MatmulConfig(128, 128, 64).to_abi()), ctypes.byref(pr), None, None,
                                  ctypes.byref(n)) == 0
    # K = 65 and N = 33 are not multiples of 8 elements: both operands are staged (256-byte-rounded copies)
    # A: 17 rows of 72 (K = 65 rounded to 8); B stays N-major: 65 rows of 40 (N = 33 rounded to 8)
    assert n.value == r256(17 * 72 * 2) + r256(65 * 40 * 2)


def test_smem_bytes_matches_config_space():
    from cs464_b200.config_space import smem_bytes
    lib = _abi.load()
    for cfg in (MatmulConfig(128, 256, 64, num_stages=4), MatmulConfig(16, 128, 128, num_stages=6)):
        n = ctypes.c_size_t()
        pr = _abi.Problem(M=256, N=256, K=256, stride_am=256, stride_ak=1, stride_bk=256, stride_bn=1,
                          stride_cm=256, stride_cn=1, dtype=0)
        assert lib.b2g_smem_bytes(ctypes.byref(cfg.to_abi()), ctypes.byref(pr), ctypes.byref(n)) == 0
        assert n.value == smem_bytes(cfg)


def test_plan_create_without_gpu_reports_cuda_error():
    """Without a device the plan fails cleanly with B2G_ERR_CUDA (never a crash)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    lib = _abi.load()
    plan = ctypes.c_void_p()
    pr = _abi.Problem(M=64, N=64, K=64, stride_am=64, stride_ak=1, stride_bk=64, stride_bn=1, stride_cm=64,
                      stride_cn=1, dtype=0)
    rc = lib.b2g_plan_create(ctypes.byref(MatmulConfig(128, 128, 64).to_abi()), ctypes.byref(pr), 256, 256, 256,
                             None, 0, None, ctypes.byref(plan))
    assert rc == _abi.B2G_ERR_CUDA
    assert plan.value is None


def test_fast_division_method_used_by_the_tile_decode():
    """The kernel divides tile and split indices by a multiply-high and a shift (round-up reciprocal): m =
    floor(2^32 * (2^s - d) / d) + 1 with s = ceil(log2 d), q = (umulhi(n, m) + n) >> s, for 0 <= n < 2^31. This
    restates the host set-up (`make_fastdiv`) and the device step (`fdiv`) and checks them against exact division."""
    import random

    def make(d):
        s = 0
        while (1 << s) < d:
            s += 1
        return ((1 << 32) * ((1 << s) - d)) // d + 1, s

    def fdiv(n, m, s):
        return (((n * m) >> 32) + n) >> s

    rng = random.Random(0)
    divisors = [1, 2, 3, 5, 7, 8, 13, 16, 64, 127, 148, 1000, 4096, (1 << 20) + 3, (1 << 30) - 1, (1 << 31) - 1]
    divisors += [rng.randrange(1, 1 << 31) for _ in range(40)]
    for d in divisors:
        m, s = make(d)
        assert 0 < m < (1 << 32) or d == 1
        ns = [0, 1, d - 1, d, d + 1, 2 * d - 1, (1 << 31) - 1, (1 << 31) - 2] + [rng.randrange(0, 1 << 31) for _ in range(300)]
        for n in ns:
            if 0 <= n < (1 << 31):
                assert fdiv(n, m, s) == n // d, (n, d)
