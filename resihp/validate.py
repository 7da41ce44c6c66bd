"""Argument checks shared by every planning entry point.

Mirrors the reference's argument contract (``resihp/validate.py:16-41`` in
ksqbxm/resihp-reproduction): ``bool`` never counts as an integer, because ``True``
would otherwise plan degree 1 or rank 1 silently, and rank sets come back sorted so
that a planner's answer cannot depend on the order its caller discovered the ranks in.
"""

from numbers import Integral
from typing import Iterable


def _as_int(name: str, value: object, floor: int, word: str) -> int:
    ok = isinstance(value, Integral) and not isinstance(value, bool) and value >= floor
    if not ok:
        raise ValueError(f"{name} must be a {word} integer")
    return int(value)


def positive_int(name: str, value: object) -> int:
    """``value`` as ``int`` if it is an integer ``>= 1``; ``ValueError`` otherwise."""
    return _as_int(name, value, 1, "positive")


def non_negative_int(name: str, value: object) -> int:
    """``value`` as ``int`` if it is an integer ``>= 0``; ``ValueError`` otherwise."""
    return _as_int(name, value, 0, "non-negative")


def unique_ranks(name: str, values: Iterable[int]) -> tuple[int, ...]:
    """Sorted tuple of distinct non-negative ranks; repeats or non-integers raise."""
    ranks = [non_negative_int(name, v) for v in values]
    if len(set(ranks)) != len(ranks):
        raise ValueError(f"{name} must not contain duplicate ranks")
    return tuple(sorted(ranks))
