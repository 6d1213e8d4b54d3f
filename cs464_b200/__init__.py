"""cs464_b200 — B200-native (sm_100a) fp16/bf16 GEMM family behind the CS464 backend protocol.

Public API (mirrors the reference's kernels/triton_matmul.py and kernels/config_space.py):
    MatmulConfig, B200Matmul, matmul, even_k, grid        cs464_b200.matmul
    SPACE, HwLimits, full_space, smem_bytes, static_violations, shape_violations, prune, HANDPICKED
                                                           cs464_b200.config_space
    parse_key                                              cs464_b200.keys
The kernels are hand-written CUDA for sm_100a in cs464_b200/csrc, reached through the C ABI of include/b2g.h.
"""
from cs464_b200.matmul import B200Matmul, MatmulConfig, even_k, grid, matmul  # noqa: F401
from cs464_b200.keys import parse_key  # noqa: F401

__all__ = ["B200Matmul", "MatmulConfig", "matmul", "even_k", "grid", "parse_key"]
