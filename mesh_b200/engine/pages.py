"""KV page allocator. Uses the native runtime (``mesh_b200._runtime``) when built, else a Python
free list with identical behaviour (lowest page ids first, double-free detection)."""
from __future__ import annotations

import heapq
from typing import List, Optional


class _PyPageAllocator:
    def __init__(self, num_pages: int, reserved: int = 0):
        if num_pages <= reserved:
            raise ValueError("page pool too small")
        self.num_pages = num_pages
        self.reserved = reserved
        self._free = list(range(reserved, num_pages))
        heapq.heapify(self._free)
        self._used = set()

    def alloc(self, n: int) -> Optional[List[int]]:
        if n > len(self._free):
            return None
        out = [heapq.heappop(self._free) for _ in range(n)]
        self._used.update(out)
        return out

    def free(self, pages: List[int]) -> None:
        for p in pages:
            if p not in self._used:
                raise ValueError(f"double free or foreign page {p}")
            self._used.remove(p)
            heapq.heappush(self._free, p)

    @property
    def num_free(self) -> int:
        return len(self._free)

    @property
    def num_used(self) -> int:
        return len(self._used)


def PageAllocator(num_pages: int, reserved: int = 0):
    try:
        from .. import _runtime  # type: ignore
        return _runtime.PageAllocator(num_pages, reserved)
    except ImportError:
        return _PyPageAllocator(num_pages, reserved)
