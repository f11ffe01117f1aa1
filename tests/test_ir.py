"""The IR mirror, text format and exact pass pipeline, pinned to tgc's own printed graphs.

tests/golden/graphs/*.tgc were printed by tgc (tgc.ir.serialize.dumps) from graphs built with
tgc's Builder, and, for the gradient graphs, produced by tgc.grad.reverse.gradient and tgc's
default pipeline. tgcb must build, print, parse and optimise them identically.
"""

from __future__ import annotations

import os

import pytest
from conftest import GOLDEN

from tgcb import ir, memory, passes, serialize, workloads
from tgcb.errors import ConfigError, GraphError, PassError, TypeInferenceError

GRAPHS = os.path.join(GOLDEN, "graphs")


def golden_text(name: str) -> str:
    with open(os.path.join(GRAPHS, f"{name}.tgc")) as f:
        return f.read()


@pytest.mark.parametrize(
    "name,build",
    [
        ("cone", lambda: workloads.cone_graph(ir.Builder)),
        ("mlp", lambda: workloads.mlp_graph(ir.Builder)),
        ("mlp_loss_64", lambda: workloads.mlp_graph(ir.Builder, rows=64, loss=True)),
        ("int8_linear", lambda: workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32)),
        ("sum", lambda: workloads.sum_graph(ir.Builder)),
    ],
)
def test_builder_prints_like_tgc(name, build):
    assert serialize.dumps(build()) == golden_text(name)


@pytest.mark.parametrize("name", sorted(f[:-4] for f in os.listdir(GRAPHS) if f.endswith(".tgc")))
def test_text_round_trip(name):
    text = golden_text(name)
    g = serialize.loads(text)
    ir.validate(g)
    assert serialize.dumps(g) == text


def test_pipeline_matches_tgc_on_gradient_graph():
    """tgc's default pipeline turned the raw gradient graph into train_grad_small; so must ours."""
    raw = serialize.loads(golden_text("train_grad_small_raw"))
    opt, report = passes.default_pipeline().run(raw)
    assert serialize.dumps(opt) == golden_text("train_grad_small")
    assert report.rounds >= 1


def test_pipeline_is_a_fixed_point_on_optimised_graphs():
    for name in ("train_grad_8192", "mlp", "cone"):
        g = serialize.loads(golden_text(name))
        opt, _ = passes.default_pipeline().run(g)
        if name.startswith("train"):
            assert serialize.dumps(opt) == golden_text(name)


def test_exact_rules_only():
    b = ir.Builder()
    x = b.input([4, 4], name="x")
    one = b.constant(1.0)
    zero = b.constant(0.0)
    y = b.add(b.mul(x, one), zero)
    z = b.mul(b.sub(x, x), zero)  # x*0 is not exact (inf*0 = nan): must stay
    g = b.finish(y, z)
    opt, _ = passes.default_pipeline().run(g)
    ops = [n.op.name for n in opt.nodes]
    assert opt.outputs[0] == "x"
    assert "mul" in ops and "sub" in ops


def test_constant_folding_in_declared_type():
    b = ir.Builder()
    x = b.input([2], name="x")
    c = b.add(b.constant(0.1), b.constant(0.2))
    g = b.finish(b.mul(x, c))
    opt, _ = passes.default_pipeline().run(g)
    consts = [n for n in opt.nodes if n.op.name == "constant"]
    assert len(consts) == 1
    assert consts[0].attrs["value"] == passes.round_to(0.1 + 0.2, ir.FLOAT32)


def test_transposes_cancel():
    b = ir.Builder()
    x = b.input([3, 5], name="x")
    g = b.finish(b.relu(b.transpose(b.transpose(x, [1, 0]), [1, 0])))
    opt, _ = passes.default_pipeline().run(g)
    assert [n.op.name for n in opt.nodes] == ["relu"]


def test_builder_errors_match_tgc():
    b = ir.Builder()
    b.input([2, 3], name="x")
    with pytest.raises(GraphError):
        b.input([2, 3], name="x")
    with pytest.raises(GraphError):
        b.exp("nope")
    x2 = b.input([4, 4], name="y")
    with pytest.raises(TypeInferenceError):
        b.matmul("x", x2)
    with pytest.raises(ConfigError):
        b.sum("x", [2])
    with pytest.raises(TypeInferenceError):
        ir.promote(ir.FLOAT16, ir.BFLOAT16)
    with pytest.raises(GraphError):
        b.finish()


def test_accumulator_widening():
    b = ir.Builder()
    h = b.input([8], ir.FLOAT16, name="h")
    q = b.input([8], ir.INT8, name="q")
    g = b.finish(b.sum(h, [0]), b.sum(q, [0]), b.max(q, [0]))
    assert [g.value(o).dtype for o in g.outputs] == [ir.FLOAT32, ir.INT32, ir.INT8]


def test_pipeline_refuses_a_pass_that_never_settles():
    counter = {"n": 0}

    def retag(graph):
        counter["n"] += 1
        n = graph.nodes[0]
        return ir.Graph([ir.Node(n.op, n.inputs, n.output, {"tag": counter["n"]})], list(graph.inputs), list(graph.outputs))

    b = ir.Builder()
    x = b.input([2], name="x")
    g = b.finish(b.exp(x))
    with pytest.raises(PassError):
        passes.Pipeline([passes.Pass("retag", retag)], max_rounds=3).run(g)


def test_depth_first_order_and_plan():
    g = serialize.loads(golden_text("fixture_branching_graph"))
    order = memory.depth_first_order(g)
    assert len(order) == len(g.nodes)
    seen = {v.name for v in g.inputs}
    for n in order:
        assert all(i in seen for i in n.inputs)
        seen.add(n.name)
    sizes = {v.name: v.bytes for v in g.inputs} | {n.name: n.output.bytes for n in g.nodes}
    steps = [(list(n.inputs), [n.name]) for n in order]
    iv = memory.intervals_for_steps([v.name for v in g.inputs], steps, g.outputs, sizes)
    plan = memory.plan_largest_first(iv)
    memory.validate_plan(iv, plan)
    assert plan.arena_bytes >= memory.peak_bytes(iv)
    assert all(a.offset % memory.ALIGNMENT == 0 for a in plan.allocations)
