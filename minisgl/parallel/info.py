"""Process-global tensor-parallel identity (reference: python/minisgl/distributed/info.py)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class DistributedInfo:
    rank: int
    size: int

    def __post_init__(self):
        if not (0 <= self.rank < self.size):
            raise ValueError(f"invalid rank {self.rank} for world size {self.size}")

    def is_primary(self) -> bool:
        return self.rank == 0


_TP_INFO: DistributedInfo | None = None


def set_tp_info(rank: int, size: int) -> DistributedInfo:
    global _TP_INFO
    if _TP_INFO is not None and (_TP_INFO.rank, _TP_INFO.size) != (rank, size):
        raise RuntimeError(f"TP info already set to {_TP_INFO}")
    _TP_INFO = DistributedInfo(rank, size)
    return _TP_INFO


def get_tp_info() -> DistributedInfo:
    if _TP_INFO is None:
        raise RuntimeError("TP info is not set")
    return _TP_INFO


def try_get_tp_info() -> DistributedInfo | None:
    return _TP_INFO


def reset_tp_info() -> None:
    global _TP_INFO
    _TP_INFO = None
