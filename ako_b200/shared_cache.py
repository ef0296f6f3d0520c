"""A ``kernel_cache.json`` that several processes can share.

AKO's ``KernelCache.save`` (``ako/dispatcher/cache.py:110-116``) writes the
whole document from one process's memory, so with one process per GPU on a
shared ``AKO_CACHE_PATH`` each save drops the records the other processes
wrote since it loaded. :class:`LockedKernelCache` keeps AKO's document,
lookups and records and changes only how a save reaches the file.
"""

from __future__ import annotations

import fcntl
import json
import os
import tempfile
from typing import Any

from ako_b200.reference import ako

ako()
from ako.dispatcher.cache import KernelCache  # noqa: E402


class LockedKernelCache(KernelCache):
    """AKO's ``KernelCache`` whose saves merge instead of overwrite.

    Under an exclusive ``flock`` on ``<file>.lock`` a save reads the file,
    replaces only the records this process set since its last save, writes
    the result to a temporary file in the same directory and renames it over
    the cache, then adopts the merged entries. ``clear()`` empties the file.
    """

    def __init__(self, path: Any = None, *, autosave: bool = True) -> None:
        self._dirty: set[tuple[str, str, str]] = set()
        self._cleared = False
        super().__init__(path, autosave=autosave)

    def set(self, gpu_key: str, op_name: str, shape_key: str, kernel_name: str, **metrics: Any) -> None:
        self._dirty.add((gpu_key, op_name, shape_key))
        super().set(gpu_key, op_name, shape_key, kernel_name, **metrics)

    def clear(self) -> None:
        self._dirty.clear()
        self._cleared = True
        super().clear()

    def _disk_entries(self) -> dict[str, Any]:
        try:
            raw = json.loads(self.path.read_text())
        except (OSError, json.JSONDecodeError):
            return {}
        return self._migrate(raw) if isinstance(raw, dict) else {}

    def save(self) -> None:
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with open(self.path.with_name(self.path.name + ".lock"), "a+") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            try:
                merged = {} if self._cleared else self._disk_entries()
                for gpu_key, op_name, shape_key in self._dirty:
                    rec = self._entries.get(gpu_key, {}).get(op_name, {}).get(shape_key)
                    if rec is not None:
                        merged.setdefault(gpu_key, {}).setdefault(op_name, {})[shape_key] = rec
                doc = self.to_dict()
                doc["entries"] = merged
                fd, tmp = tempfile.mkstemp(prefix=self.path.name + ".", suffix=".part", dir=self.path.parent)
                with os.fdopen(fd, "w") as f:
                    json.dump(doc, f, indent=2)
                os.replace(tmp, self.path)
                self._entries = merged
                self._dirty.clear()
                self._cleared = False
            finally:
                fcntl.flock(lock, fcntl.LOCK_UN)
