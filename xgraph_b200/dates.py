"""Dates of a KG index's date entities, as date comparisons read them (the reference's
xgraph.expressions.Date, src/xgraph/expressions.py:139-201, and its packed date keys,
src/xgraph/index.py:600-662).

A date states a year and, by its precision, a month and a day; it covers the interval from
its first to its last day (a year covers 1 January to 31 December, a month its 1st to a
bound of 31).  One date is before another when its interval ends before the other's
starts.  A key packs a date into an int32 (year in the top 21 bits, signed; month 4 bits,
0 if unstated; day 5 bits, 0 if unstated; precision 2 bits), so that keys sort by year,
month, day and precision, and equal keys are equal stored dates.  The interval bounds pack
the same way with precision bits 0, so that bounds compare as plain integers.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass

import numpy as np

PRECISIONS = ("year", "month", "day")
YEAR_BITS = 21
YEARS = (-(1 << (YEAR_BITS - 1)), (1 << (YEAR_BITS - 1)) - 1)  # the years a key holds

VERDICTS = {"no": "Q1499999998", "yes": "Q1499999999"}
"""A value comparison's verdicts as entities, each labelled with its verdict, which an index
built with verdicts appends to the KG's entities (src/xgraph/index.py:657-662)."""


@dataclass(frozen=True)
class Date:
    year: int
    month: int | None = None
    day: int | None = None
    precision: str = ""

    def __post_init__(self) -> None:
        if not self.precision:
            object.__setattr__(self, "precision", "day" if self.day else "month" if self.month else "year")
        if self.precision not in PRECISIONS:
            raise ValueError(f"unknown date precision {self.precision!r}")

    @property
    def lo(self) -> tuple[int, int, int]:
        """The first day the date covers."""
        if self.precision == "year":
            return (self.year, 1, 1)
        return (self.year, self.month or 1, self.day if self.precision == "day" else 1)

    @property
    def hi(self) -> tuple[int, int, int]:
        """The last day the date covers (31 for a month's last day)."""
        if self.precision == "year":
            return (self.year, 12, 31)
        return (self.year, self.month or 12, self.day if self.precision == "day" else 31)

    def before(self, other: Date) -> bool:
        return self.hi < other.lo


def pack_date(date: Date) -> int:
    if not YEARS[0] <= date.year <= YEARS[1]:
        raise ValueError(f"the year of {date} does not fit a date key {YEARS}")
    month, day = date.month or 0, date.day or 0
    if not (0 <= month <= 12 and 0 <= day <= 31):
        raise ValueError(f"{date!r} has no valid month and day for a date key")
    return (date.year << 11) | (month << 7) | (day << 2) | PRECISIONS.index(date.precision)


def unpack_date(key: int) -> Date:
    key = int(key)
    month, day = (key >> 7) & 15, (key >> 2) & 31
    return Date(key >> 11, month or None, day or None, PRECISIONS[key & 3])


def _bounds(keys, first: bool) -> np.ndarray:
    keys = np.asarray(keys, dtype=np.int64)
    year, month, day, precision = keys >> 11, (keys >> 7) & 15, (keys >> 2) & 31, keys & 3
    month = np.where((precision == 0) | (month == 0), 1 if first else 12, month)
    day = np.where(precision == 2, day, 1 if first else 31)
    return ((year << 11) | (month << 7) | (day << 2)).astype(np.int32)


def date_lo(keys) -> np.ndarray:
    """Each key's first day, packed with precision bits 0 (Date.lo as an integer)."""
    return _bounds(keys, True)


def date_hi(keys) -> np.ndarray:
    """Each key's last day, packed as date_lo (Date.hi); a before b iff hi(a) < lo(b)."""
    return _bounds(keys, False)


def date_table(dates: Mapping[int, Date]) -> tuple[np.ndarray, np.ndarray]:
    """The date table of dates by entity position: the positions, sorted, and their keys;
    a date whose year a key cannot hold is left out."""
    kept = sorted((e, d) for e, d in dates.items() if YEARS[0] <= d.year <= YEARS[1])
    return (np.array([e for e, _ in kept], dtype=np.int32),
            np.array([pack_date(d) for _, d in kept], dtype=np.int32))
