"""Running-set manager for decode (reference: python/minisgl/scheduler/decode.py:9-39)."""

from __future__ import annotations

from typing import Dict, Iterable

from minisgl.core import Batch, Req


class DecodeManager:
    def __init__(self, page_size: int):
        self.page_size = page_size
        self.running: Dict[int, Req] = {}  # uid -> req, insertion-ordered

    def filter_reqs(self, reqs: Iterable[Req]) -> None:
        """Only the batch's requests changed: add those that continue, drop those that ended."""
        running = self.running
        for r in reqs:
            if r.can_decode:
                running.setdefault(r.uid, r)
            elif running.get(r.uid) is r:
                del running[r.uid]

    def remove_req(self, req: Req) -> None:
        if self.running.get(req.uid) is req:
            del self.running[req.uid]

    def abort_req(self, uid: int) -> Req | None:
        return self.running.pop(uid, None)

    @property
    def inflight_tokens(self) -> int:
        """Tokens that running requests may still claim (plus one partial page each)."""
        n = len(self.running)
        return sum(r.remain_len for r in self.running.values()) + (self.page_size - 1) * n

    def schedule_next_batch(self) -> Batch | None:
        if not self.running:
            return None
        return Batch(reqs=sorted(self.running.values(), key=lambda r: r.uid), phase="decode")

    @property
    def runnable(self) -> bool:
        return bool(self.running)
