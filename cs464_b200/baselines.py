"""Comparator backends with the same make_runner protocol: B1 = torch.matmul (cuBLAS default heuristic).

The reference's B1 is baselines/torch_mm.py:10-18. These are measurement baselines only; nothing in the sm_100a
family dispatches to them.
"""
from __future__ import annotations

import torch


class TorchMatmul:
    family = "torch_matmul"
    cfg: dict = {}
    key = "default"

    def make_runner(self, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None):
        c = out if out is not None else torch.empty((a.shape[0], b.shape[1]), device=a.device, dtype=a.dtype)

        def run():
            return torch.matmul(a, b, out=c)
        return run
