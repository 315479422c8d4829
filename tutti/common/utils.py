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


def _block_id(value):
    """An integer block id (int or NumPy integer, not bool), else None."""
    if isinstance(value, bool):
        return None
    if isinstance(value, int):
        return value
    try:
        import numpy as np
    except ImportError:  # pragma: no cover - numpy is a dependency of torch
        return None
    return int(value) if isinstance(value, np.integer) else None


def flatten_block_ids(block_tables) -> tuple[int, ...]:
    """Block ids of a wave's block tables as one flat tuple, for error reports.

    Used on failure paths, so it never raises: ``None``, strings and bytes give
    ``()``; a lone integer gives a 1-tuple; rows that are lists, tuples or sets
    contribute their integer items (one level deep) and every other value is
    skipped. Parity: tutti/common/utils.py:46-62 of the reference.
    """
    if block_tables is None or isinstance(block_tables, (str, bytes, bytearray)):
        return ()
    one = _block_id(block_tables)
    if one is not None:
        return (one,)
    try:
        rows = list(block_tables)
    except TypeError:
        return ()
    out: list[int] = []
    for row in rows:
        if isinstance(row, (list, tuple, set)):
            out.extend(b for b in map(_block_id, row) if b is not None)
        else:
            b = _block_id(row)
            if b is not None:
                out.append(b)
    return tuple(out)
