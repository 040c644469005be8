"""Small integer helpers (reference: python/minisgl/utils/misc.py:4-48)."""

from __future__ import annotations

from typing import Callable


def call_if_main(name: str = "__main__"):
    """Decorator: run the function immediately when the defining module is ``__main__``."""

    def wrap(fn: Callable):
        if name == "__main__":
            fn()
        return fn

    return wrap


def div_even(a: int, b: int, allow_replicate: bool = False) -> int:
    """``a / b`` that must divide evenly.

    With ``allow_replicate`` and ``b > a`` (e.g. more TP ranks than KV heads) each rank keeps one
    replicated unit, which requires ``b % a == 0``.
    """
    if allow_replicate and b > a:
        if b % a != 0:
            raise ValueError(f"{b} ranks cannot replicate {a} units evenly")
        return 1
    if a % b != 0:
        raise ValueError(f"{a} is not divisible by {b}")
    return a // b


def div_ceil(a: int, b: int) -> int:
    return -(-a // b)


def align_ceil(a: int, b: int) -> int:
    return div_ceil(a, b) * b


def align_down(a: int, b: int) -> int:
    return a - a % b


class Unset:
    def __repr__(self) -> str:
        return "UNSET"


UNSET = Unset()
