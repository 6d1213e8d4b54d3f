"""Per-shape winner cache: an append-only JSONL file of search results, shared by processes and GPUs of one host.

Same role and guarantees as the reference's tune/winner_cache.py:
  * one line per search (shape, dtype, search width, choice, environment); the last line of a shape wins;
  * appends are serialised with flock and fsync'd; a torn last line left by a crash is terminated before the next
    append and skipped on read; `compact` rewrites the file atomically (temp file + os.replace) under the lock;
  * environment tiers: a line from another GPU model (`hw_id`) or another build of the kernels (`kernel_src`, the hash
    of the CUDA sources and flags the loaded library reports, the role of kernel_src_hash in tune/winner_cache.py:76-79)
    is hard-stale and ignored; other differences (driver, torch, CUDA runtime, declared clock lock) are soft-stale:
    served only with allow_stale;
  * `backend_for(choice)` rebuilds a runnable backend from a stored key (tune/winner_cache.py:421-441).
Many ranks of a sharded search append to one file concurrently; `merge` folds per-rank files into one.
"""
from __future__ import annotations

import fcntl
import hashlib
import json
import os
import time
from pathlib import Path

SCHEMA = 1
ENV_PATH = "B2G_WINNER_CACHE"        # a file path, or "off"
HARD_FIELDS = ("hw_id", "kernel_src")


def default_path() -> Path:
    return Path(os.environ.get(ENV_PATH) or Path.home() / ".cache" / "cs464_b200" / "winner_cache.jsonl")


def default_enabled() -> bool:
    return os.environ.get(ENV_PATH, "").strip().lower() not in ("off", "0", "none")


def kernel_src_hash() -> str:
    """Hash of the CUDA sources and build flags of the loaded library: any kernel change invalidates stored keys."""
    from cs464_b200 import _abi
    return _abi.source_hash()


def hw_id(device: int | None = None) -> str:
    import torch
    p = torch.cuda.get_device_properties(torch.cuda.current_device() if device is None else device)
    return f"{p.name}|sm{p.major}{p.minor}|{p.multi_processor_count}sm|{round(p.total_memory / 2**30)}GiB"


def clock_lock_declared(value: str | None = None) -> str | None:
    v = value if value is not None else os.environ.get("B2G_CLOCK_LOCK")
    if v is None or not str(v).strip():
        return None
    v = str(v).strip().lower()
    return "unlocked" if v in ("none", "off", "0", "unlocked") else v


def environment(device: int | None = None, clock_lock: str | None = None, extra: dict | None = None) -> dict:
    import torch
    env = {"hw_id": hw_id(device), "kernel_src": kernel_src_hash(), "torch": torch.__version__,
           "cuda_runtime": torch.version.cuda, "driver": _driver_version(), "clock_lock": clock_lock_declared(clock_lock)}
    if extra:
        env.update(extra)
    return env


def _driver_version() -> str | None:
    try:
        import pynvml
        pynvml.nvmlInit()
        v = pynvml.nvmlSystemGetDriverVersion()
        return v.decode() if isinstance(v, bytes) else v
    except Exception:
        return None


def tier(row: dict, env: dict) -> tuple[str, list[str]]:
    """("current" | "soft" | "hard", differing fields) of a stored line against `env`. Fields the current environment
    declares as None are not compared; a field the line lacks is unknown, so at most soft."""
    row_env = row.get("env") or {}
    fields = [f for f, v in env.items() if v is not None and row_env.get(f) != v]
    if any(f in HARD_FIELDS and f in row_env for f in fields):
        return "hard", fields
    return ("soft" if fields else "current"), fields


def _row_id(row: dict) -> str:
    return hashlib.sha256(json.dumps(row, sort_keys=True, default=str).encode()).hexdigest()[:16]


class WinnerCache:
    def __init__(self, path: str | os.PathLike | None = None, env: dict | None = None):
        self.path = Path(path) if path else default_path()
        self.env = env if env is not None else environment()
        self._rows: dict[tuple, dict[str, dict]] = {}
        self._stamp = None
        self.reload()

    @staticmethod
    def key(M: int, N: int, K: int, dtype: str) -> tuple:
        return (int(M), int(N), int(K), str(dtype))

    def _file_stamp(self):
        try:
            st = os.stat(self.path)
            return (st.st_ino, st.st_size, st.st_mtime_ns)
        except OSError:
            return None

    @staticmethod
    def parse_lines(lines):
        """Readable rows of this schema; torn or damaged lines are skipped."""
        for line in lines:
            try:
                r = json.loads(line)
            except ValueError:
                continue
            if (isinstance(r, dict) and r.get("schema") == SCHEMA and isinstance(r.get("dtype"), str)
                    and all(isinstance(r.get(x), int) for x in ("M", "N", "K", "k"))):
                yield r

    def reload(self) -> None:
        rows = {}
        self._stamp = self._file_stamp()
        try:
            lines = self.path.read_text(errors="replace").splitlines()
        except OSError:
            lines = []
        for r in self.parse_lines(lines):
            t, fields = tier(r, self.env)
            if t == "hard":
                continue
            r = dict(r)
            r["id"] = _row_id(r)
            r["_stale"] = fields
            rows.setdefault(self.key(r["M"], r["N"], r["K"], r["dtype"]), {})[t] = r
        self._rows = rows

    def refresh(self) -> bool:
        if self._file_stamp() == self._stamp:
            return False
        self.reload()
        return True

    def __len__(self) -> int:
        return sum(1 for v in self._rows.values() if "current" in v)

    @staticmethod
    def _out(r: dict) -> dict:
        out = {k: v for k, v in r.items() if k != "_stale"}
        out["stale"] = list(r["_stale"])
        return out

    def get(self, M: int, N: int, K: int, dtype: str = "fp16", *, k: int = 1, allow_stale: bool = False) -> dict | None:
        """The stored entry whose search timed at least `k` candidates; current preferred, soft-stale with allow_stale."""
        tiers = self._rows.get(self.key(M, N, K, dtype), {})
        for t in ("current", "soft") if allow_stale else ("current",):
            r = tiers.get(t)
            if r is not None and r["k"] >= k and (r.get("choice") or {}).get("key") is not None:
                return self._out(r)
        return None

    def entries(self, allow_stale: bool = False) -> list[dict]:
        tiers = ("current", "soft") if allow_stale else ("current",)
        return [self._out(v[t]) for v in self._rows.values() for t in tiers if t in v]

    def _locked(self, mode: str):
        self.path.parent.mkdir(parents=True, exist_ok=True)
        for _ in range(20):
            f = open(self.path, mode)
            fcntl.flock(f, fcntl.LOCK_EX)
            try:
                if os.fstat(f.fileno()).st_ino == os.stat(self.path).st_ino:
                    return f
            except FileNotFoundError:
                pass
            f.close()  # compacted (replaced) while waiting for the lock: reopen the new file
        raise OSError(f"{self.path}: kept being replaced while waiting for its lock")

    def _append(self, row: dict) -> None:
        with self._locked("a+b") as f:
            f.seek(0, os.SEEK_END)
            torn = False
            if f.tell() > 0:
                f.seek(-1, os.SEEK_END)
                torn = f.read(1) != b"\n"
            f.seek(0, os.SEEK_END)
            f.write((b"\n" if torn else b"") + (json.dumps(row, default=str) + "\n").encode())
            f.flush()
            os.fsync(f.fileno())

    def put(self, M: int, N: int, K: int, dtype: str, *, k: int, choice: dict, candidates: list | None = None,
            extra: dict | None = None) -> dict:
        row = {"schema": SCHEMA, "M": int(M), "N": int(N), "K": int(K), "dtype": str(dtype), "k": int(k),
               "choice": choice, "env": self.env, "t": time.time()}
        if candidates is not None:
            row["n_candidates"] = len(candidates)
            row["n_valid"] = sum(1 for c in candidates if c.get("valid"))
        if extra:
            row.update(extra)
        self._append(row)
        r = dict(row)
        r["id"] = _row_id(row)
        r["_stale"] = []
        self._rows.setdefault(self.key(M, N, K, dtype), {})["current"] = r
        return self._out(r)

    def compact(self) -> dict:
        """Rewrite the file keeping, per shape, the last line of each readable tier (hard-stale lines of other
        environments are kept too: they belong to other GPUs or builds sharing the file)."""
        with self._locked("r+b") as f:
            lines = f.read().decode(errors="replace").splitlines()
            last: dict[tuple, str] = {}
            order = []
            for line in lines:
                rs = list(self.parse_lines([line]))
                if not rs:
                    continue
                r = rs[0]
                k = (*self.key(r["M"], r["N"], r["K"], r["dtype"]), json.dumps(r.get("env"), sort_keys=True))
                if k not in last:
                    order.append(k)
                last[k] = line
            tmp = self.path.with_name(self.path.name + f".tmp{os.getpid()}")
            with open(tmp, "wb") as g:
                g.write("".join(last[k] + "\n" for k in order).encode())
                g.flush()
                os.fsync(g.fileno())
            os.replace(tmp, self.path)
        self.reload()
        return {"before": len(lines), "after": len(order)}

    def merge(self, paths) -> int:
        """Append every readable line of other cache files (per-rank results) to this one; returns lines merged."""
        n = 0
        for p in paths:
            try:
                lines = Path(p).read_text(errors="replace").splitlines()
            except OSError:
                continue
            for r in self.parse_lines(lines):
                self._append(r)
                n += 1
        self.reload()
        return n


def backend_for(choice: dict, M: int = 0, N: int = 0, K: int = 0, dtype=None):
    """The runnable backend a stored choice names, or None (no key)."""
    if not choice or choice.get("key") is None:
        return None
    family = choice.get("family") or "b200_sm100a_v1"
    if family == "torch_matmul":
        from cs464_b200.baselines import TorchMatmul
        return TorchMatmul()
    from cs464_b200.keys import parse_key
    from cs464_b200.matmul import B200Matmul
    return B200Matmul(parse_key(choice["key"]))
