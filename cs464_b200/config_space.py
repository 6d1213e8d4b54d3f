"""Config space and pruning rules of the sm_100a family (same functions and return shapes as kernels/config_space.py).

Pruning is split in two, as in the reference (kernels/config_space.py:1-6):
  * static rules - depend only on the config and the hardware limits (run once per GPU)
  * shape rules  - depend on (M, N, K) as well (run per shape when building the work list)
Each rule has a name; `prune` returns the reasons a config was dropped so the pruning is auditable.

The shape rules are the reference's rules with the same names and tests (kernels/config_space.py:69-90): a selector
that prunes by them keeps working unchanged. The static rules are new, because the limits are: tensor-memory columns,
the tcgen05 tile shapes, the 227 KB shared-memory ring, instead of mma.sync register pressure.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass

from cs464_b200.matmul import MatmulConfig

SPACE = {
    "BLOCK_M": [16, 32, 64, 128, 256],   # <= 64: operand-swapped skinny form (tensor-core N side over M)
    "BLOCK_N": [64, 128, 192, 256],
    "BLOCK_K": [64, 128],
    "num_warps": [4, 8],                 # epilogue warps
    "num_stages": [2, 3, 4, 5, 6, 8],
    "GROUP_M": [1, 4, 8, 16],
    "SPLIT_K": [1, 2, 4, 8, 16],
    "PERSISTENT": [1, 0, 2],              # 1 persistent tiles, 0 one CTA per tile, 2 stream-K
    "CLUSTER": [1, 2],                   # 2: CTA pair on two SMs, M = 256 tcgen05 MMAs
}

TMEM_COLUMNS = 512
CTL_SMEM_BYTES = 2048          # barriers + alignment slack in front of the ring (kCtlBytes + kAlignSlack)
# Little's law: ~6.5 TB/s x ~1.5 us of load latency over 148 SMs is ~66 KB in flight per SM; a ring smaller than
# 64 KB cannot cover it
MIN_RING_BYTES = 64 * 1024


@dataclass(frozen=True)
class HwLimits:
    smem_per_block_bytes: int   # opt-in max dynamic shared memory per block
    regs_per_sm: int
    sm_count: int
    tmem_columns: int = TMEM_COLUMNS

    @classmethod
    def from_device(cls, device: int | None = None) -> "HwLimits":
        import torch
        p = torch.cuda.get_device_properties(torch.cuda.current_device() if device is None else device)
        return cls(p.shared_memory_per_block_optin, p.regs_per_multiprocessor, p.multi_processor_count)

    @classmethod
    def b200(cls) -> "HwLimits":
        """The B200 limits (sm_100: 232,448 B opt-in shared memory per block, 64K registers, 148 SMs)."""
        return cls(232448, 65536, 148)


def full_space() -> list[MatmulConfig]:
    keys = list(SPACE)
    return [MatmulConfig(**dict(zip(keys, vals))) for vals in itertools.product(*SPACE.values())]


def swapped(cfg: MatmulConfig) -> bool:
    return cfg.BLOCK_M <= 64


def mma_tile(cfg: MatmulConfig) -> tuple[int, int]:
    """(rows on the tensor core's M side, columns on its N side) of one tile (of the pair, with CLUSTER=2)."""
    return (cfg.BLOCK_N, cfg.BLOCK_M) if swapped(cfg) else (cfg.BLOCK_M, cfg.BLOCK_N)


def smem_bytes(cfg: MatmulConfig, elem_bytes: int = 2) -> int:
    """Dynamic shared memory of one CTA: control block + num_stages x (A tile + B tile); a pair's CTA holds halves."""
    rows = cfg.BLOCK_M + cfg.BLOCK_N
    if cfg.CLUSTER == 2:
        rows //= 2
    return CTL_SMEM_BYTES + cfg.num_stages * rows * cfg.BLOCK_K * elem_bytes


def tmem_columns(cfg: MatmulConfig) -> int:
    """fp32 accumulator columns of one CTA (one column per output column per 128 rows it owns)."""
    tm, tn = mma_tile(cfg)
    return tn if cfg.CLUSTER == 2 else tm // 128 * tn


def static_violations(cfg: MatmulConfig, hw: HwLimits, elem_bytes: int = 2) -> list[str]:
    reasons = []
    if smem_bytes(cfg, elem_bytes) > hw.smem_per_block_bytes:
        reasons.append("smem_exceeds_limit")
    tm, tn = mma_tile(cfg)
    if swapped(cfg):
        # the tensor core's M side runs over BLOCK_N: one (128) or two (256) M=128 MMAs
        if cfg.BLOCK_N not in (128, 256):
            reasons.append("skinny_block_n_not_128_or_256")
    elif cfg.BLOCK_N % 64:
        # B (N-contiguous) is read in 64-column, 128-byte swizzle atoms
        reasons.append("block_n_not_multiple_of_64")
    if cfg.CLUSTER == 2 and tm != 256:
        # the pair splits a 256-row tensor-core tile into two 128-row halves
        reasons.append("cluster_needs_256_rows")
    if cfg.CLUSTER == 2 and not swapped(cfg) and (cfg.BLOCK_N // 2) % 64:
        # each CTA reads its half of B in 64-column swizzle atoms; other widths would stage B through a copy per call
        reasons.append("cluster_half_n_not_multiple_of_64")
    if tmem_columns(cfg) > hw.tmem_columns:
        reasons.append("tmem_exceeds_limit")
    if cfg.PERSISTENT == 2 and cfg.SPLIT_K != 1:
        reasons.append("streamk_with_split_k")
    if cfg.num_warps == 8 and tn <= 32:
        # a second epilogue warpgroup would have no 32-column chunk of its own
        reasons.append("epilogue_warps_idle")
    if smem_bytes(cfg, elem_bytes) - CTL_SMEM_BYTES < MIN_RING_BYTES:
        reasons.append("ring_too_shallow")
    return reasons


def shape_violations(cfg: MatmulConfig, M: int, N: int, K: int, *, max_workspace_bytes: int = 512 * 2**20) -> list[str]:
    """The reference's shape rules, same names and order (kernels/config_space.py:69-90)."""
    reasons = []

    def cover(x: int) -> int:
        return max(16, 1 << (x - 1).bit_length())

    if cfg.BLOCK_M > 2 * cover(M):
        reasons.append("block_m_oversized")
    if cfg.BLOCK_N > 2 * cover(N):
        reasons.append("block_n_oversized")
    if cfg.BLOCK_K > 2 * cover(K):
        reasons.append("block_k_oversized")
    if cfg.SPLIT_K > 1:
        if K < cfg.SPLIT_K * cfg.BLOCK_K:
            reasons.append("split_k_starved")
        ws_elems = cfg.SPLIT_K * M * N
        if ws_elems * 4 > max_workspace_bytes or ws_elems >= 2**31:
            reasons.append("split_k_workspace_too_large")
    if cfg.GROUP_M > 1 and -(-M // cfg.BLOCK_M) <= 1:
        reasons.append("group_m_noop")
    return reasons


def prune(configs: list[MatmulConfig], hw: HwLimits, shape: tuple[int, int, int] | None = None,
          elem_bytes: int = 2) -> tuple[list[MatmulConfig], dict[str, int]]:
    kept, dropped = [], {}
    for c in configs:
        reasons = static_violations(c, hw, elem_bytes)
        if shape is not None:
            reasons += shape_violations(c, *shape)
        if reasons:
            for r in reasons:
                dropped[r] = dropped.get(r, 0) + 1
        else:
            kept.append(c)
    return kept, dropped


# Hand-picked starting configs, one per regime (the reference's HANDPICKED, kernels/config_space.py:109-115).
HANDPICKED = {
    "large_square": MatmulConfig(256, 256, 64, num_warps=4, num_stages=6, GROUP_M=8, CLUSTER=2),
    "medium": MatmulConfig(128, 128, 64, num_warps=4, num_stages=6, GROUP_M=8),
    "small_tile": MatmulConfig(128, 64, 64, num_warps=4, num_stages=8, GROUP_M=8),
    "skinny_m": MatmulConfig(16, 128, 128, num_warps=4, num_stages=6, GROUP_M=1),
    "large_k_splitk": MatmulConfig(128, 128, 64, num_warps=4, num_stages=6, GROUP_M=1, SPLIT_K=8),
}
