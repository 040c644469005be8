"""Named factory registry that raises argparse-friendly errors
(reference: python/minisgl/utils/registry.py:6-38)."""

from __future__ import annotations

from typing import Callable, Dict, Generic, Iterable, List, TypeVar

T = TypeVar("T")


class Registry(Generic[T]):
    def __init__(self, kind: str):
        self._kind = kind
        self._items: Dict[str, T] = {}

    def register(self, name: str) -> Callable[[T], T]:
        if name in self._items:
            raise KeyError(f"{self._kind} '{name}' registered twice")

        def deco(item: T) -> T:
            self._items[name] = item
            return item

        return deco

    def __getitem__(self, name: str) -> T:
        try:
            return self._items[name]
        except KeyError:
            raise KeyError(f"Unsupported {self._kind}: {name}") from None

    def __contains__(self, name: str) -> bool:
        return name in self._items

    def supported_names(self) -> List[str]:
        return list(self._items)

    def assert_supported(self, names: str | Iterable[str]) -> None:
        from argparse import ArgumentTypeError

        for n in [names] if isinstance(names, str) else names:
            if n not in self._items:
                raise ArgumentTypeError(
                    f"Unsupported {self._kind}: {n}. Supported: {self.supported_names()}"
                )
