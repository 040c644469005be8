"""Colored per-module loggers tagged with time, optional pid and the TP rank, plus ``*_rank0``
variants that only print on the primary rank (reference: python/minisgl/utils/logger.py:9-128).

Environment: ``LOG_LEVEL`` (DEBUG/INFO/WARNING/ERROR/CRITICAL), ``LOG_PID`` (1 adds the pid).
"""

from __future__ import annotations

import logging
import os
import sys

_COLORS = {
    "DEBUG": "\033[36m",
    "INFO": "\033[32m",
    "WARNING": "\033[33m",
    "ERROR": "\033[31m",
    "CRITICAL": "\033[35m",
}
_RESET, _BOLD = "\033[0m", "\033[1m"


def _level_from_env() -> int:
    return getattr(logging, os.getenv("LOG_LEVEL", "INFO").upper(), logging.INFO)


class _Formatter(logging.Formatter):
    def __init__(self, tag: str, show_rank: bool):
        super().__init__()
        self.tag = tag
        self.show_rank = show_rank

    def format(self, record: logging.LogRecord) -> str:
        from minisgl.parallel.info import try_get_tp_info

        tag = self.tag
        info = try_get_tp_info()
        if info is not None and self.show_rank:
            tag += f"|core|rank={info.rank}"
        stamp = self.formatTime(record, "%Y-%m-%d|%H:%M:%S")
        color = _COLORS.get(record.levelname, "")
        level = f"{color}{record.levelname:<8}{_RESET}"
        return f"{_BOLD}[{stamp}{tag}]{_RESET} {level} {record.getMessage()}"


class MiniLogger(logging.Logger):
    """Logger with rank-0-only helpers."""

    def _rank0(self, level: int, msg, *args, **kwargs) -> None:
        from minisgl.parallel.info import try_get_tp_info

        info = try_get_tp_info()
        if info is None or info.is_primary():
            self.log(level, msg, *args, **kwargs)

    def info_rank0(self, msg, *args, **kwargs):
        self._rank0(logging.INFO, msg, *args, **kwargs)

    def debug_rank0(self, msg, *args, **kwargs):
        self._rank0(logging.DEBUG, msg, *args, **kwargs)

    def warning_rank0(self, msg, *args, **kwargs):
        self._rank0(logging.WARNING, msg, *args, **kwargs)

    def critical_rank0(self, msg, *args, **kwargs):
        self._rank0(logging.CRITICAL, msg, *args, **kwargs)


def init_logger(
    name: str,
    suffix: str = "",
    *,
    level: str | None = None,
    use_pid: bool | None = None,
    use_tp_rank: bool | None = None,
) -> MiniLogger:
    old_cls = logging.getLoggerClass()
    logging.setLoggerClass(MiniLogger)
    try:
        logger = logging.getLogger(f"minisgl::{name}")
    finally:
        logging.setLoggerClass(old_cls)
    assert isinstance(logger, MiniLogger)
    logger.setLevel(getattr(logging, level.upper()) if level else _level_from_env())
    if use_pid is None:
        use_pid = os.getenv("LOG_PID", "0").lower() in ("1", "true", "yes")
    tag = ""
    if use_pid:
        tag += f"|pid={os.getpid()}"
    if suffix:
        tag += f"|{os.path.basename(suffix)}"
    logger.handlers.clear()
    handler = logging.StreamHandler(sys.stdout)
    handler.setFormatter(_Formatter(tag, use_tp_rank is not False))
    logger.addHandler(handler)
    logger.propagate = False
    return logger
