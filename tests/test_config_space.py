"""Config space, pruning rules and key codec, against the reference's own verdicts (tests/golden/config_rules.json,
made by running kernels/config_space.py and tune/sweep.py of the reference)."""
from __future__ import annotations

import json
from pathlib import Path

import pytest

from cs464_b200.config_space import (HANDPICKED, SPACE, HwLimits, full_space, prune, shape_violations, smem_bytes,
                                     static_violations, tmem_columns)
from cs464_b200.keys import parse_key
from cs464_b200.matmul import MatmulConfig, check_config, even_k, grid

RULES = json.loads((Path(__file__).resolve().parent / "golden" / "config_rules.json").read_text())


def test_shape_rules_match_reference():
    """Same names, order and verdicts as the reference's shape_violations on its own configs (2,639 cases)."""
    for r in RULES["shape_rules"]:
        cfg = MatmulConfig(**r["cfg"])
        assert shape_violations(cfg, *r["shape"]) == r["reasons"], (r["key"], r["shape"])


def test_reference_keys_parse_unchanged():
    for r in RULES["shape_rules"][::13]:
        cfg = parse_key(r["key"])
        assert cfg.key() == r["key"]
        assert {k: v for k, v in cfg.to_dict().items() if k not in ("PERSISTENT", "CLUSTER")} == r["cfg"]
    for key in RULES["handpicked"].values():
        assert parse_key(key).key() == key


def test_extended_keys_round_trip():
    for cfg in full_space()[::211]:
        assert parse_key(cfg.key()) == cfg
    c = MatmulConfig(128, 256, 64, PERSISTENT=0)
    assert c.key().endswith("_p0") and parse_key(c.key()) == c
    for bad in ("bm128_bn256_bk64_w4_s4_g8_sk1_p1", "bm128_bn256_bk64_w4_s4_g8_sk1_q3", "bm128_bn256_bk64",
                "xbm128_bn256_bk64_w4_s4_g8_sk1"):
        with pytest.raises(ValueError):
            parse_key(bad)


def test_space_size_and_static_prune():
    space = full_space()
    n = 1
    for v in SPACE.values():
        n *= len(v)
    assert len(space) == n == 57600
    hw = HwLimits.b200()
    kept, dropped = prune(space, hw)
    assert 0 < len(kept) < len(space)
    assert all(smem_bytes(c) <= hw.smem_per_block_bytes for c in kept)
    assert all(tmem_columns(c) <= 512 for c in kept)
    assert "smem_exceeds_limit" in dropped and "skinny_block_n_not_128_or_256" in dropped
    assert "cluster_needs_256_rows" in dropped
    assert set(HANDPICKED.values()) <= set(kept)


def test_statically_kept_configs_are_accepted_by_the_library():
    """Every config the static rules keep is one the C ABI accepts (sampled)."""
    kept, _ = prune(full_space(), HwLimits.b200())
    for cfg in kept[::37]:
        assert check_config(cfg, 4096, 4096, 4096) is None, cfg.key()


def test_static_rules():
    hw = HwLimits.b200()
    assert "smem_exceeds_limit" in static_violations(MatmulConfig(256, 256, 128, num_stages=4), hw)
    assert "block_n_not_multiple_of_64" in static_violations(MatmulConfig(128, 192 - 64 + 32, 64), hw)
    assert "epilogue_warps_idle" in static_violations(MatmulConfig(16, 128, 128, num_warps=8), hw)
    assert "ring_too_shallow" in static_violations(MatmulConfig(16, 128, 64, num_stages=2), hw)


def test_shape_rules():
    big = MatmulConfig(256, 128, 64)
    assert "block_m_oversized" in shape_violations(big, 1, 4096, 4096)
    assert "block_m_oversized" not in shape_violations(big, 4096, 4096, 4096)
    sk = MatmulConfig(64, 64, 64, SPLIT_K=16)
    assert "split_k_starved" in shape_violations(sk, 64, 64, 512)
    assert "split_k_workspace_too_large" in shape_violations(sk, 16384, 16384, 16384)


def test_even_k_and_grid():
    cfg = MatmulConfig(128, 256, 64, SPLIT_K=2)
    assert even_k(256, cfg) and not even_k(200, cfg)
    assert grid(300, 600, cfg) == (3 * 3, 2)
