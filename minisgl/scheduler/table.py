"""Request-row allocator over the page table (reference: python/minisgl/scheduler/table.py)."""

from __future__ import annotations

import torch


class TableManager:
    def __init__(self, max_running_reqs: int, page_table: torch.Tensor) -> None:
        self._max = max_running_reqs
        self._free = list(range(max_running_reqs - 1, -1, -1))
        self.page_table = page_table

    @property
    def available_size(self) -> int:
        return len(self._free)

    def allocate(self) -> int:
        return self._free.pop()

    def free(self, row: int) -> None:
        if row in self._free:  # at most max_running_reqs entries
            raise RuntimeError(f"page-table row {row} freed twice")
        self._free.append(row)
