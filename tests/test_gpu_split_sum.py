"""Column reductions on the GPU are tgc's split_sum of each column, bit for bit.

The backend lowers a sum over axis 0 to its column kernels (row blocks of ``L`` rows added in
order, then the partials in order; tgcb/codegen.py ``col_split``). tgc's
tgc/passes/reduction.py:105-121 ``split_sum(column, parts)`` adds ceil(rows / parts) terms per
part and then the partials: the same additions in the same order. tests/golden/models.json
holds tgc's values for seeded columns at the shapes of the training step's bias gradients and
two ragged shapes; the GPU's columns must equal them exactly. The error against the float64
sum is reported beside the zero error against the declared order.
"""

from __future__ import annotations

import json
import os

import pytest
import torch
from conftest import GOLDEN

from tgcb import ir
from tgcb.codegen import col_split
from tgcb.runtime import compile_graph

pytestmark = pytest.mark.gpu


def _cases():
    with open(os.path.join(GOLDEN, "models.json")) as f:
        return json.load(f)["split_sum"]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: f"{c['rows']}x{c['cols']}")
def test_column_sum_is_tgcs_split_sum(cuda, case):
    rows, cols = case["rows"], case["cols"]
    b = ir.Builder()
    x = b.input([rows, cols], name="x")
    g = b.finish(b.sum(x, [0]))
    compiled = compile_graph(g)
    step = [s for s in compiled.module.steps if s.kind == "colreduce"]
    assert len(step) == 1, "a sum over axis 0 lowers to the column kernels"
    parts, per = col_split(rows, cols)
    assert f"{parts} row blocks of {per}" in step[0].bracketing
    gen = torch.Generator().manual_seed(rows * 31 + cols)
    xs = torch.randn(rows, cols, generator=gen)
    out = compiled({"x": xs.to(cuda)})[0].cpu()
    compiled.check_status()
    k = len(case["split_sum"])
    got = out[:k].tolist()
    assert got == case["split_sum"]  # zero error against the declared bracketing
    for c, (g_, exact) in enumerate(zip(got, case["exact"], strict=True)):
        # and the error against float64 stays inside the bound of the split: at most
        # per + parts - 1 dependent roundings, each within 2^-24 of the magnitudes summed
        bound = (per + parts) * 2.0**-24 * float(xs[:, c].double().abs().sum())
        assert abs(g_ - exact) <= bound
