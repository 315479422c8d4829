"""``tutti.common.utils``: small config helpers with Tutti's names and rules.

``parse_capacity`` needs a unit (``"64 GiB"``; GB counts 1000s, GiB 1024s) and an
exact positive number of bytes.
"""
import re
from fractions import Fraction


def is_int(value) -> bool:
    """A real int (bools are ints in Python, but not here)."""
    return isinstance(value, int) and not isinstance(value, bool)


def positive_int(config: dict, key: str) -> int:
    value = config.get(key)
    if not is_int(value) or value <= 0:
        raise ValueError(f"{key} must be a positive integer, got {value!r}")
    return value


def parse_capacity(value: str) -> int:
    m = re.fullmatch(r"\s*(\d+(?:\.\d+)?)\s*([KMGT]?i?B)\s*", value, flags=re.IGNORECASE) if isinstance(value, str) else None
    if m is None:
        raise ValueError(f"capacity needs a unit, e.g. '64 GiB', got {value!r}")
    unit = m[2].upper()
    power = "BKMGT".index(unit[0]) if unit != "B" else 0
    amount = Fraction(m[1]) * (1024 if "I" in unit else 1000) ** power
    if amount <= 0 or amount.denominator != 1:
        raise ValueError(f"capacity must be a whole positive number of bytes, got {value!r}")
    return int(amount)


def flatten_block_ids(block_tables) -> tuple[int, ...]:
    """Block tables (nested sequences of ints) as one flat tuple."""
    out = []
    for row in block_tables:
        if is_int(row):
            out.append(row)
        else:
            out.extend(flatten_block_ids(row))
    return tuple(int(x) for x in out)
