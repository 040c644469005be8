"""Per-process traffic / launch counters read by the benchmark.

* ``h2d_bytes``: host -> device bytes of batch plans and sampling parameters;
* ``d2h_bytes``: device -> host bytes of sampled tokens;
* ``launches``: kernels of this engine's native library launched (eager calls are counted as they
  happen; a CUDA-graph replay adds the number of native launches recorded at capture).
"""

from __future__ import annotations


class Counters:
    def __init__(self) -> None:
        self.reset()

    def reset(self) -> None:
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.launches = 0

    def snapshot(self) -> dict:
        return {"h2d_bytes": self.h2d_bytes, "d2h_bytes": self.d2h_bytes, "launches": self.launches}


COUNTERS = Counters()
