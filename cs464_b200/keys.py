"""Config-key codec: `parse_key` inverts `MatmulConfig.key()` (the reference's tune/sweep.py:355-364).

Keys of the reference's format (`bm128_bn256_bk32_w8_s3_g8_sk1`, 7 fields) parse unchanged; extension knobs follow
as `_<letter><int>` suffixes (`_p0`: PERSISTENT=0, `_c2`: CLUSTER=2) and are present only when they differ from
their defaults, so a key with no suffix means the same 7 fields it always did.
"""
from __future__ import annotations

import re

from cs464_b200.matmul import EXTENSIONS, MatmulConfig

KEY_RE = re.compile(r"bm(\d+)_bn(\d+)_bk(\d+)_w(\d+)_s(\d+)_g(\d+)_sk(\d+)((?:_[a-z]+\d+)*)")
_EXT_RE = re.compile(r"_([a-z]+)(\d+)")


def parse_key(key: str) -> MatmulConfig:
    m = KEY_RE.fullmatch(key)
    if not m:
        raise ValueError(f"bad config key {key!r}")
    base = list(map(int, m.groups()[:7]))
    ext = {}
    for letter, val in _EXT_RE.findall(m.group(8) or ""):
        if letter not in EXTENSIONS:
            raise ValueError(f"bad config key {key!r}: unknown extension {letter!r}")
        ext[EXTENSIONS[letter][0]] = int(val)
    cfg = MatmulConfig(*base, **ext)
    if cfg.key() != key:  # defaults spelled out, or suffixes out of order: one canonical key per config
        raise ValueError(f"bad config key {key!r}: canonical form is {cfg.key()!r}")
    return cfg
