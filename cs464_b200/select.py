"""Zero-search config choice: a fixed rule from shape to config, used when no winner is cached.

The reference's zero-search fallback is a hand-picked config per regime (kernels/config_space.py:109-115) and its
learned ranker (analysis/learned.py:461-535); this module is the rule-based first stage that the measured search
(cs464_b200.search) replaces per shape once a winner exists.
"""
from __future__ import annotations

from cs464_b200.matmul import MatmulConfig

SM_COUNT = 148


def heuristic_config(M: int, N: int, K: int, sm_count: int = SM_COUNT) -> MatmulConfig:
    """A reasonable config for a row-major (M, N, K) problem without any timing."""
    if M <= 64:
        bm = 16 if M <= 16 else (32 if M <= 32 else 64)
        tiles = -(-N // 128)
        kb = -(-K // 128)
        split = 1
        while tiles * split < sm_count and split * 2 <= 16 and kb // (split * 2) >= 4:
            split *= 2
        stages = 6 if bm <= 32 else 5
        return MatmulConfig(bm, 128, 128, num_warps=4, num_stages=stages, GROUP_M=1, SPLIT_K=split)
    tiles_big = -(-M // 256) * -(-N // 256)
    if tiles_big >= sm_count // 2:
        return MatmulConfig(256, 256, 64, num_warps=4, num_stages=3, GROUP_M=8)
    tiles = -(-M // 128) * -(-N // 128)
    split = 1
    kb = -(-K // 64)
    while tiles * split < sm_count and split * 2 <= 16 and kb // (split * 2) >= 8:
        split *= 2
    return MatmulConfig(128, 128, 64, num_warps=4, num_stages=6, GROUP_M=8, SPLIT_K=split)
