"""Small integer helpers (behaviour of src/povs/utils.py:4-14 in the reference)."""

import math


def is_power_of_2(x: int) -> bool:
    return x > 0 and x & (x - 1) == 0


def round_down_to_power_of_2(x: int) -> int:
    """Largest power of two not above ``x`` (x >= 1)."""
    return 1 << (int(x).bit_length() - 1)


def least_factor_to_make_multiple(x: int, y: int) -> int:
    """Smallest k >= 1 such that k * x is a multiple of y."""
    return y // math.gcd(x, y)
