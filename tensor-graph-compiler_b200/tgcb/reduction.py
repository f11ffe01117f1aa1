"""How the backend splits column reductions, in tgc's split-reduction terms.

tgc/passes/reduction.py:33-121 splits a reduction of ``length`` terms into ``parts`` partial
chains of ceil(length / parts) consecutive terms, each added left to right, and then adds the
partials left to right (``split_sum``); ``SplitPlan`` reports the chain lengths. A column
reduction on the GPU (one thread per column and row block, then one per column over the
blocks, tgcb/codegen.py) runs exactly that order with the part count ``col_split`` picks, so its
results are tgc's ``split_sum`` of each column bit for bit (tests/golden/models.json holds
tgc's values).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from tgcb.codegen import col_split
from tgcb.errors import ConfigError


@dataclass
class SplitPlan:
    """A reduction of ``length`` terms in ``parts`` partial chains (reduction.py:33-81)."""

    length: int
    parts: int

    def __post_init__(self) -> None:
        if self.length < 1:
            raise ConfigError(f"a reduction needs at least one term, got {self.length}")
        if not 1 <= self.parts <= self.length:
            raise ConfigError(f"the parts must number from one to the length ({self.length}), got {self.parts}")

    @property
    def per_part(self) -> int:
        return math.ceil(self.length / self.parts)

    @property
    def serial_depth(self) -> int:
        """Dependent additions on the longest path: one part, then the partials."""
        return self.per_part + self.parts - 1

    @property
    def speedup(self) -> float:
        return self.length / self.serial_depth

    def as_dict(self) -> dict:
        return {"length": self.length, "parts": self.parts, "per_part": self.per_part,
                "serial_depth": self.serial_depth, "speedup": round(self.speedup, 3)}


def column_plan(rows: int, cols: int) -> SplitPlan:
    """The split the backend's column kernel uses for a reduction over axis 0 of [rows, cols]."""
    parts, per = col_split(rows, cols)
    plan = SplitPlan(rows, parts)
    if plan.per_part != per:
        raise ConfigError(f"the column kernel's {per} rows per part are not split_sum's {plan.per_part}")
    return plan
