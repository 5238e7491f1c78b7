"""BLAS flag arguments (`uplo`, `side`, `diag`, `trans*`), same semantics as the
reference's trnblas/_flags.py:1-51: the documented words and the single BLAS
letters are accepted, case-insensitively; anything else is a ValueError; a
non-string transpose flag keeps its truth value; 'C' is rejected (no conjugate
transpose)."""

from __future__ import annotations

_WORDS = {
    "uplo": {"upper": "upper", "u": "upper", "lower": "lower", "l": "lower"},
    "side": {"left": "left", "l": "left", "right": "right", "r": "right"},
    "diag": {
        "unit": "unit",
        "u": "unit",
        "nonunit": "nonunit",
        "non-unit": "nonunit",
        "n": "nonunit",
    },
}


def _word(kind: str, value) -> str:
    table = _WORDS[kind]
    if isinstance(value, str) and value.strip().lower() in table:
        return table[value.strip().lower()]
    choices = sorted(set(table.values()))
    raise ValueError(f"{kind} must be one of {choices} (or the BLAS letter); got {value!r}")


def uplo_flag(value) -> str:
    """'upper' or 'lower'."""
    return _word("uplo", value)


def side_flag(value) -> str:
    """'left' or 'right'."""
    return _word("side", value)


def diag_flag(value) -> str:
    """'unit' or 'nonunit'."""
    return _word("diag", value)


def trans_flag(value, name: str = "trans") -> bool:
    """A bool transpose flag; 'N' / 'T' (any case) mean no-transpose / transpose."""
    if isinstance(value, str):
        key = value.strip().lower()
        if key == "n":
            return False
        if key == "t":
            return True
        raise ValueError(f"{name} must be a bool or 'N' / 'T'; got {value!r}")
    return bool(value)
