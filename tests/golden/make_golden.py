"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's own Python code.

Run where a checkout of the reference exists (pass its path as argv[1], or set $CS464_REFERENCE; by default a
`reference` directory next to this repository's root):
    python tests/golden/make_golden.py /path/to/reference

It imports, from the reference:
  * tune/correctness.py: `make_inputs` (seeded inputs), `reference` (fp32 ground truth), `check_output` (the gate);
  * kernels/config_space.py: `full_space`, `shape_violations`, `prune`, `HwLimits`, `HANDPICKED`;
  * kernels/triton_matmul.py: `MatmulConfig.key`, and tune/sweep.py: `parse_key`.
and writes:
  * gemm_cases.npz + gemm_cases.json  inputs (CPU generator), the reference's fp32 result, and the gate's verdicts on
                                      the rounded result and on planted mistakes (a corrupted tile, a NaN row);
  * inputs_hash.json                  sha256 of make_inputs bytes for the BASELINE.json config-1 shape (1024^3, seed 0)
                                      and other seeds/shapes, so the CPU generator stream is pinned without 4 MB arrays;
  * config_rules.json                 the reference's shape-rule verdicts and key strings on a sample of its space,
                                      plus its static-prune counts for the RTX 3080 limits it was written for.
Nothing under tests/ reads the reference at test time: the tests read only these files.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent
REF = Path(sys.argv[1] if len(sys.argv) > 1 else
           (os.environ.get("CS464_REFERENCE") or Path(__file__).resolve().parents[3] / "reference"))
sys.path.insert(0, str(REF))

import torch  # noqa: E402
from kernels.config_space import HANDPICKED, HwLimits, full_space, prune, shape_violations  # noqa: E402
from tune.correctness import check_output, make_inputs, reference  # noqa: E402
from tune.sweep import parse_key  # noqa: E402

CASES = [  # (name, M, N, K, dtype, seed): the reference's kernel-test shapes that stay small, plus bf16
    ("t1x1x1", 1, 1, 1, "float16", 0),
    ("t17x33x65", 17, 33, 65, "float16", 0),
    ("t128x128x128", 128, 128, 128, "float16", 0),
    ("t129x257x1031", 129, 257, 1031, "float16", 0),
    ("t513x255x16", 513, 255, 16, "float16", 0),
    ("t64x64x2048", 64, 64, 2048, "float16", 0),
    ("t100x70x1000", 100, 70, 1000, "float16", 0),
    ("bf300x200x500", 300, 200, 500, "bfloat16", 0),
    ("t96x80x512s3", 96, 80, 512, "float16", 3),
]

SHAPES_FOR_RULES = [(1, 1, 1), (1, 4096, 4096), (17, 33, 65), (128, 128, 128), (129, 257, 1031), (513, 255, 16),
                    (2048, 2048, 8), (64, 64, 16384), (16384, 16384, 16384), (64, 64, 512), (8192, 28672, 4096),
                    (16, 6144, 4096), (1, 4096, 14336)]


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    arrays, meta = {}, []
    for name, M, N, K, dt, seed in CASES:
        dtype = getattr(torch, dt)
        a, b = make_inputs(M, N, K, dtype=dtype, seed=seed, device="cpu")
        ref = reference(a, b)
        rounded = ref.to(dtype)
        verdicts = {"rounded": check_output(rounded, ref, K, dtype).to_dict()}
        if M >= 16 and N >= 16:
            bad = rounded.clone()
            bad[:16, :16] += float(max(1.0, 0.05 * np.sqrt(K)) * 10)
            verdicts["corrupt_tile"] = check_output(bad, ref, K, dtype).to_dict()
        nan = rounded.clone()
        nan[-1] = float("nan")
        verdicts["nan_row"] = check_output(nan, ref, K, dtype).to_dict()
        arrays[f"{name}_a"] = bits(a)
        arrays[f"{name}_b"] = bits(b)
        arrays[f"{name}_ref"] = ref.numpy().astype(np.float32)
        meta.append({"name": name, "M": M, "N": N, "K": K, "dtype": dt, "seed": seed, "verdicts": verdicts})
    np.savez_compressed(OUT / "gemm_cases.npz", **arrays)
    (OUT / "gemm_cases.json").write_text(json.dumps({"cases": meta}, indent=1) + "\n")

    hashes = []
    for M, N, K, dt, seed in [(1024, 1024, 1024, "float16", 0), (256, 512, 128, "float16", 1),
                              (64, 64, 64, "bfloat16", 0), (16, 6144, 4096, "float16", 2)]:
        a, b = make_inputs(M, N, K, dtype=getattr(torch, dt), seed=seed, device="cpu")
        hashes.append({"M": M, "N": N, "K": K, "dtype": dt, "seed": seed,
                       "a_sha256": hashlib.sha256(bits(a).tobytes()).hexdigest(),
                       "b_sha256": hashlib.sha256(bits(b).tobytes()).hexdigest()})
    (OUT / "inputs_hash.json").write_text(json.dumps({"inputs": hashes}, indent=1) + "\n")

    space = full_space()
    sample = list(HANDPICKED.values()) + space[::97]
    rules = []
    for cfg in sample:
        key = cfg.key()
        assert parse_key(key) == cfg
        for shape in SHAPES_FOR_RULES:
            rules.append({"key": key, "cfg": cfg.to_dict(), "shape": list(shape),
                          "reasons": shape_violations(cfg, *shape)})
    kept, dropped = prune(space, HwLimits(101376, 65536, 68))
    doc = {"space_size": len(space), "handpicked": {k: v.key() for k, v in HANDPICKED.items()},
           "static_prune_rtx3080": {"kept": len(kept), "dropped": dropped}, "shape_rules": rules}
    (OUT / "config_rules.json").write_text(json.dumps(doc) + "\n")
    print(f"wrote {len(meta)} GEMM cases, {len(hashes)} input hashes, {len(rules)} rule verdicts to {OUT}")


if __name__ == "__main__":
    main()
