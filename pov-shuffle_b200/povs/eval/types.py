"""N-gram specification of the bias metrics (reference: src/povs/eval/types.py)."""

from __future__ import annotations

from typing import Iterable, NamedTuple, Union


class NgramSpec(NamedTuple):
    """An n-gram degree ``n`` and the number of positions ``skip`` between its elements."""

    n: int
    skip: int = 0

    @classmethod
    def parse(cls, x: Union[int, "NgramSpec", Iterable[int]]) -> "NgramSpec":
        """An ``NgramSpec`` from itself, a degree, or an ``(n, skip)`` iterable."""
        if isinstance(x, cls):
            return x
        if isinstance(x, int):
            return cls(n=x)
        return cls(*x)

    @property
    def title(self) -> str:
        """Display name, e.g. ``"2-gram"`` or ``"3-gram (skip 1)"``."""
        return f"{self.n}-gram" + (f" (skip {self.skip})" if self.skip else "")
