"""Reverse mode restated from tgc, pinned to the gradient graphs tgc itself printed."""

from __future__ import annotations

import os

import pytest
from conftest import GOLDEN

from tgcb import grad, ir, passes, serialize, workloads
from tgcb.errors import ConfigError, PassError


def golden_text(name: str) -> str:
    with open(os.path.join(GOLDEN, "graphs", f"{name}.tgc")) as f:
        return f.read()


def test_raw_gradient_graph_is_tgcs():
    g = workloads.mlp_graph(ir.Builder, rows=96, d=64, f=256, loss=True)
    res = grad.gradient(g, ["w1", "b1", "w2", "b2"], seed_is_input=False)
    assert serialize.dumps(res.graph) == golden_text("train_grad_small_raw")


@pytest.mark.parametrize("rows", [8192, 16384, 32768, 65536])
def test_optimised_gradient_graphs_are_tgcs(rows):
    g = workloads.mlp_graph(ir.Builder, rows=rows, loss=True)
    res = grad.gradient(g, ["w1", "b1", "w2", "b2"], seed_is_input=False)
    opt, _ = passes.default_pipeline().run(res.graph)
    assert serialize.dumps(opt) == golden_text(f"train_grad_{rows}")


def test_every_rule_builds_a_valid_graph():
    b = ir.Builder()
    x = b.input([4, 6], name="x")
    y = b.input([6], name="y")
    h = b.add(b.mul(x, y), b.div(x, b.exp(y)))
    h = b.maximum(b.tanh(h), b.minimum(b.sigmoid(h), b.relu(h)))
    h = b.sub(b.sqrt(b.abs(h)), b.reciprocal(b.add(b.log(b.abs(h)), b.constant(3.0))))
    h = b.concat(b.slice(h, 1, 1, 3), b.transpose(b.reshape(h, [6, 4]), [1, 0]), axis=1)
    out = b.sum(b.max(b.mean(h, [1], keepdims=True), [0]), [0])
    g = b.finish(out)
    res = grad.gradient(g, ["x", "y"])
    ir.validate(res.graph)
    assert [res.graph.value(o).shape.ints() for o in res.graph.outputs] == [(4, 6), (6,)]


def test_refusals():
    b = ir.Builder()
    x = b.input([3], name="x")
    g = b.finish(b.exp(x), b.neg(x))
    with pytest.raises(ConfigError):
        grad.gradient(g)
    b = ir.Builder()
    x = b.input([3], name="x")
    g = b.finish(b.cast(x, ir.INT32))
    with pytest.raises(ConfigError):
        grad.gradient(g)
    b = ir.Builder()
    x = b.input([3], name="x")
    y = b.input([3], name="y")
    g = b.finish(b.exp(x))
    with pytest.raises(PassError):
        grad.gradient(g, ["y"])
