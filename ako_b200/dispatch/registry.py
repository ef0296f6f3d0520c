"""Kernel registry: op name -> candidate implementations.

Interface of the reference's ``ako/dispatcher/registry.py:13-60``: a frozen
``KernelEntry(op_name, kernel_name, fn, backend, priority)``; registering a
name again replaces the old entry; candidates are listed by descending
priority, ties in registration order; ``default`` is the first of them.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

KernelFn = Callable[..., Any]


@dataclass(frozen=True)
class KernelEntry:
    op_name: str
    kernel_name: str
    fn: KernelFn
    backend: str
    priority: int = 0


class KernelRegistry:
    def __init__(self) -> None:
        self._ops: dict[str, dict[str, KernelEntry]] = {}
        self._order = 0
        self._seq: dict[tuple[str, str], int] = {}

    def register(self, entry: KernelEntry) -> None:
        """Add ``entry``; an entry of the same op and kernel name is replaced."""
        self._ops.setdefault(entry.op_name, {})[entry.kernel_name] = entry
        self._order += 1
        self._seq[(entry.op_name, entry.kernel_name)] = self._order

    def list_ops(self) -> list[str]:
        return sorted(self._ops)

    def list_kernels(self, op_name: str) -> list[KernelEntry]:
        entries = self._ops.get(op_name, {}).values()
        return sorted(entries, key=lambda e: (-e.priority, self._seq[(e.op_name, e.kernel_name)]))

    def get(self, op_name: str, kernel_name: str) -> KernelEntry | None:
        return self._ops.get(op_name, {}).get(kernel_name)

    def default(self, op_name: str) -> KernelEntry | None:
        kernels = self.list_kernels(op_name)
        return kernels[0] if kernels else None


_registry = KernelRegistry()


def get_registry() -> KernelRegistry:
    return _registry
