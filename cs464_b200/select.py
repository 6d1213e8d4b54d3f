"""Zero-search config choice: a fixed rule from shape to config, used when no winner is cached.

The reference's zero-search fallback is a hand-picked config per regime (kernels/config_space.py:109-115) and its
learned ranker (analysis/learned.py:461-535); this module is the rule-based first stage that the measured search
(cs464_b200.search) replaces per shape once a winner exists.
"""
from __future__ import annotations

from cs464_b200.matmul import MatmulConfig

SM_COUNT = 148
SMEM_BYTES = 232448   # opt-in dynamic shared memory per block on sm_100
CTL_BYTES = 2048      # the kernel's control block and alignment slack in front of the ring


def heuristic_config(M: int, N: int, K: int, sm_count: int = SM_COUNT) -> MatmulConfig:
    """A reasonable config for a row-major (M, N, K) problem without any timing."""
    if M <= 64:
        bm = 16 if M <= 16 else (32 if M <= 32 else 64)
        tiles = -(-N // 128)
        kb = -(-K // 128)
        split = 1
        while tiles * split < sm_count and split * 2 <= 16 and kb // (split * 2) >= 4:
            split *= 2
        # the deepest ring (up to 6) whose stages of 128 B-rows + bm A-rows x 128 K fit the shared memory
        stages = min(6, (SMEM_BYTES - CTL_BYTES) // ((128 + bm) * 128 * 2))
        return MatmulConfig(bm, 128, 128, num_warps=4, num_stages=stages, GROUP_M=1, SPLIT_K=split)
    tiles_big = -(-M // 256) * -(-N // 256)
    if tiles_big >= sm_count:
        # several waves of 256 x 256 tiles: a CTA pair per tile (double-buffered accumulators), K step 128, stream-K:
        # a partial last wave that fits twice into the pairs is split in K over them (4096^3: 97 against 104 us);
        # otherwise the waves run data-parallel, as the persistent schedule would
        return MatmulConfig(256, 256, 128, num_warps=4, num_stages=3, GROUP_M=8, CLUSTER=2, PERSISTENT=2)
    if tiles_big >= sm_count // 2:
        return MatmulConfig(256, 256, 64, num_warps=4, num_stages=3, GROUP_M=8)
    tiles = -(-M // 128) * -(-N // 128)
    split = 1
    kb = -(-K // 64)
    while tiles * split < sm_count and split * 2 <= 16 and kb // (split * 2) >= 8:
        split *= 2
    return MatmulConfig(128, 128, 64, num_warps=4, num_stages=6, GROUP_M=8, SPLIT_K=split)
