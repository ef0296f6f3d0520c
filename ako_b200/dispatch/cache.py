"""Persistent ``kernel_cache.json`` of selection decisions.

File format of the reference (``ako/dispatcher/cache.py:1-39``), so either
package reads the other's records: schema v2 is
``{"version": 2, "entries": {gpu_key: {op: {shape_key: record}}}}`` where a
record holds ``kernel``, ``created_at`` and the metrics that justified it;
a v1 file (bare kernel names, no ``version``) is read and upgraded in memory.
The path defaults to ``~/.ako/kernel_cache.json``, overridable with
``AKO_CACHE_PATH``. An unreadable file never breaks dispatch: it is moved
aside to ``<name>.corrupt`` and the cache starts empty.

Unlike the reference, saves are safe across processes: a save takes an
exclusive ``flock`` on ``<name>.lock``, merges the records other processes
wrote since, and replaces the file atomically, so one process per GPU can
share a cache file without losing records.
"""

from __future__ import annotations

import contextlib
import json
import logging
import os
from dataclasses import dataclass
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

try:
    import fcntl
except ImportError:  # pragma: no cover - non-POSIX
    fcntl = None  # type: ignore[assignment]

CACHE_SCHEMA_VERSION = 2
DEFAULT_CACHE_PATH = Path.home() / ".ako" / "kernel_cache.json"
log = logging.getLogger(__name__)


def default_cache_path() -> Path:
    env = os.environ.get("AKO_CACHE_PATH")
    return Path(env).expanduser() if env else DEFAULT_CACHE_PATH


@dataclass(frozen=True)
class CacheStats:
    hits: int = 0
    misses: int = 0

    @property
    def total(self) -> int:
        return self.hits + self.misses

    @property
    def hit_rate(self) -> float:
        return self.hits / self.total if self.total else 0.0

    def to_dict(self) -> dict[str, Any]:
        return {"hits": self.hits, "misses": self.misses, "lookups": self.total,
                "hit_rate": round(self.hit_rate, 4)}


def _upgrade(raw: Any) -> dict[str, Any]:
    if not isinstance(raw, dict):
        return {}
    if raw.get("version") == CACHE_SCHEMA_VERSION:
        entries = raw.get("entries", {})
        return entries if isinstance(entries, dict) else {}
    return {k: v for k, v in raw.items() if k != "version" and isinstance(v, dict)}


class KernelCache:
    """JSON-backed ``(gpu, op, shape key) -> record`` store."""

    def __init__(self, path: Path | str | None = None, *, autosave: bool = True) -> None:
        self.path = Path(path) if path is not None else default_cache_path()
        self.autosave = autosave
        self._entries: dict[str, Any] = {}
        self._hits = 0
        self._misses = 0
        self.load()

    # ------------------------------------------------------------ disk
    def _read_disk(self) -> dict[str, Any] | None:
        """Entries on disk; None if the file is absent; {} after moving a corrupt one aside."""
        try:
            text = self.path.read_text()
        except FileNotFoundError:
            return None
        except OSError as exc:
            log.warning("kernel cache %s unreadable (%s); starting empty", self.path, exc)
            return {}
        try:
            return _upgrade(json.loads(text))
        except json.JSONDecodeError as exc:
            log.warning("kernel cache %s is corrupt (%s); moved aside", self.path, exc)
            with contextlib.suppress(OSError):
                os.replace(self.path, self.path.with_name(self.path.name + ".corrupt"))
            return {}

    def load(self) -> None:
        self._entries = self._read_disk() or {}

    @contextlib.contextmanager
    def _locked(self):
        self.path.parent.mkdir(parents=True, exist_ok=True)
        if fcntl is None:
            yield
            return
        with open(self.path.with_name(self.path.name + ".lock"), "a") as fh:
            fcntl.flock(fh, fcntl.LOCK_EX)
            try:
                yield
            finally:
                fcntl.flock(fh, fcntl.LOCK_UN)

    def _write(self) -> None:
        payload = {"version": CACHE_SCHEMA_VERSION, "entries": self._entries}
        tmp = self.path.with_name(f".{self.path.name}.{os.getpid()}.tmp")
        tmp.write_text(json.dumps(payload, indent=2))
        os.replace(tmp, self.path)

    def save(self) -> None:
        """Merge with what other processes saved, then write atomically."""
        with self._locked():
            disk = self._read_disk() or {}
            for gpu, ops in self._entries.items():
                for op, shapes in ops.items():
                    disk.setdefault(gpu, {}).setdefault(op, {}).update(shapes)
            self._entries = disk
            self._write()

    # --------------------------------------------------------- lookups
    def get_record(self, gpu_key: str, op_name: str, shape_key: str) -> dict[str, Any] | None:
        rec = self._entries.get(gpu_key, {}).get(op_name, {}).get(shape_key)
        if rec is None:
            self._misses += 1
            return None
        self._hits += 1
        return {"kernel": rec} if isinstance(rec, str) else dict(rec)

    def get(self, gpu_key: str, op_name: str, shape_key: str) -> str | None:
        rec = self.get_record(gpu_key, op_name, shape_key)
        return rec.get("kernel") if rec else None

    def set(self, gpu_key: str, op_name: str, shape_key: str, kernel_name: str, **metrics: Any) -> None:
        rec: dict[str, Any] = {"kernel": kernel_name, "created_at": datetime.now(timezone.utc).isoformat()}
        rec.update({k: v for k, v in metrics.items() if v is not None})
        self._entries.setdefault(gpu_key, {}).setdefault(op_name, {})[shape_key] = rec
        if self.autosave:
            self.save()

    def clear(self) -> None:
        self._entries = {}
        self._hits = self._misses = 0
        if self.autosave:
            with self._locked():
                self._write()

    # --------------------------------------------------- introspection
    def stats(self) -> CacheStats:
        return CacheStats(self._hits, self._misses)

    def to_dict(self) -> dict[str, Any]:
        return {"version": CACHE_SCHEMA_VERSION, "entries": dict(self._entries)}

    def __len__(self) -> int:
        return sum(len(shapes) for ops in self._entries.values() for shapes in ops.values())
