"""tgc's models restated by tgcb, pinned to the numbers tgc itself printed (tests/golden/
models.json, made by tests/golden/make_model_golden.py): fusion_search's plans and costs
(tgc/schedule/fusion_search.py), the roofline estimate (tgc/analysis/cost.py), the all-reduce
model (tgc/parallel/collective.py), and split_sum (tgc/passes/reduction.py) against the
column kernel's declared order in the oracle.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch
from conftest import GOLDEN

from oracle import bracketing
from tgcb import collective, cost, fusion_search, ir, reduction, workloads
from tgcb.codegen import col_split


@pytest.fixture(scope="module")
def gold():
    with open(os.path.join(GOLDEN, "models.json")) as f:
        return json.load(f)


DAGS = {
    "chain": lambda: fusion_search.chain_dag(),
    "cone_3_4": lambda: fusion_search.cone_dag(readers=3, depth=4),
    "cone_3_4_x8": lambda: fusion_search.cone_dag(readers=3, depth=4, intensity=8),
    "cone_3_4_x16": lambda: fusion_search.cone_dag(readers=3, depth=4, intensity=16),
    "cone_3_4_x64": lambda: fusion_search.cone_dag(readers=3, depth=4, intensity=64),
    "cone_5_2": lambda: fusion_search.cone_dag(readers=5, depth=2),
}


@pytest.mark.parametrize("name", sorted(DAGS))
def test_fusion_search_plans_are_tgcs(gold, name):
    fs = gold["fusion_search"]
    dag = DAGS[name]()
    want = fs["dags"][name]
    assert [list(p) for p in dag.producers] == want["producers"]
    assert list(dag.sizes) == want["sizes"] and list(dag.flops) == want["flops"]
    assert list(dag.outputs) == want["outputs"] and list(dag.barriers) == want["barriers"]
    assert list(dag.interior) == want["interior"]
    rows = {r["strategy"]: r for r in fusion_search.compare(dag)}
    for strategy, expected in fs["plans"][name].items():
        got = rows[strategy]
        assert got["materialised"] == expected["materialised"], strategy
        for key in ("groups", "flops", "traffic", "cost"):
            assert got[key] == expected[key], (strategy, key)
    assert fusion_search.duplication_factor(dag, ()) == pytest.approx(fs["duplication"][name], rel=1e-15)


def test_fusion_search_details_are_tgcs(gold):
    fs = gold["fusion_search"]
    cone = fusion_search.cone_dag(readers=3, depth=4)
    assert sorted(fusion_search.group_for(cone, 5, fusion_search.normalise(cone, ()))) == fs["tip_group_outputs_only"]
    assert fusion_search.times_computed(cone, (), 4) == fs["tip_computed"]
    assert fusion_search.times_computed(cone, [4], 4) == fs["tip_computed_reused"]
    x8 = fusion_search.cone_dag(readers=3, depth=4, intensity=8)
    for w, expected in fs["weights"].items():
        got = fusion_search.exhaustive(x8, float(w)).as_dict()
        assert got["materialised"] == expected["materialised"] and got["cost"] == expected["cost"]
    for row in fs["intensity_sweep"]:
        dag = fusion_search.cone_dag(intensity=row["intensity"])
        rule, best = fusion_search.materialise_reused(dag), fusion_search.exhaustive(dag)
        assert round(rule.cost, 2) == row["rule"] and round(best.cost, 2) == row["best"]
        assert round(rule.cost / best.cost, 4) == row["regret"]


def test_one_pass_plan_beats_every_tgc_plan_on_the_cone():
    """The multi-output row kernel computes the cone once and reads x once: under tgc's own cost
    rules it is cheaper than the best plan tgc's search can find, at every intensity."""
    for intensity in (1, 8, 16, 64):
        dag = fusion_search.cone_dag(readers=3, depth=4, intensity=intensity)
        one = fusion_search.one_pass(dag)
        best = fusion_search.exhaustive(dag)
        assert one.cost < best.cost
        assert one.flops == fusion_search.materialise_reused(dag).flops  # no operation recomputed
        assert one.traffic < best.traffic


def test_dag_of_the_cone_workload():
    g = workloads.cone_graph(ir.Builder)
    dag, names = fusion_search.dag_of(g)
    assert len(dag.barriers) == 3 and len(dag.outputs) == 3
    one = fusion_search.one_pass(dag)
    # x read once (4 Mi elements) plus three 4096-element outputs written, in bytes
    assert one.traffic == (4096 * 1024 + 2 + 3 * 4096) * 4  # the two scalar constants are read too
    assert one.groups == 1
    assert one.cost < fusion_search.exhaustive(dag).cost


@pytest.mark.parametrize("name", ["cone", "mlp", "int8", "sum", "train_8192"])
def test_cost_estimates_are_tgcs(gold, name):
    from tgcb import grad

    graphs = {
        "cone": lambda: workloads.cone_graph(ir.Builder),
        "mlp": lambda: workloads.mlp_graph(ir.Builder),
        "int8": lambda: workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32),
        "sum": lambda: workloads.sum_graph(ir.Builder),
        "train_8192": lambda: grad.gradient(workloads.mlp_graph(ir.Builder, rows=8192, loss=True),
                                            ["w1", "b1", "w2", "b2"], seed_is_input=False).graph,
    }
    g = graphs[name]()
    want = gold["cost"][name]
    assert cost.graph_flops(g) == want["flops"]
    assert cost.fused_bytes(g) == want["fused_bytes"]
    assert cost.unfused_bytes(g) == want["unfused_bytes"]
    for m in cost.MACHINES.values():
        got = cost.estimate(g, m).as_dict()
        assert got["seconds"] == pytest.approx(want[m.name]["seconds"], rel=1e-12)
        assert got["memory_bound"] == want[m.name]["memory_bound"]


def test_b200_machine_from_measured_peaks():
    m = cost.b200({"hbm_gbs": 6544.0, "bf16_tflops": 1646.1, "bf16_tflops_sustained": 1404.4}, "tf32")
    assert m.bytes_per_second == 6544e9 and m.flops_per_second == pytest.approx(823.05e12)
    assert cost.b200({"hbm_gbs": 1, "bf16_tflops": 2, "bf16_tflops_sustained": 1}, "int8", sustained=True).flops_per_second == 2e12


def test_collective_model_is_tgcs(gold):
    c = gold["collective"]
    for n in (1, 2, 4, 8):
        assert collective.ring_time(33574912, n) == pytest.approx(c["ring_time"][str(n)], rel=1e-14)
        assert collective.tree_time(33574912, n) == pytest.approx(c["tree_time"][str(n)], rel=1e-14)
        assert collective.ring_volume(33574912, n) == c["ring_volume"][str(n)]
        assert collective.tree_volume(33574912, n) == c["tree_volume"][str(n)]
    link = collective.Link("given", 770e9, 20e-6)
    for n in (2, 4, 8):
        assert collective.ring_time(33574912, n, link) == pytest.approx(c["given_link_ring_time"][str(n)], rel=1e-14)
    sizes = collective.gradient_sizes()
    for row in c["bucket_sweep"]:
        assert collective.bucket_time(sizes, 8, bucket_bytes=row["bucket_bytes"]) == pytest.approx(row["seconds"], rel=1e-12)
    payload = [1024 * 4096 * 4, 4096 * 4, 4096 * 1024 * 4, 1024 * 4]
    for b, t in c["train_buckets"].items():
        assert collective.bucket_time(payload, 8, link, int(b)) == pytest.approx(t, rel=1e-12)
    for key, got in (("exposed_default", collective.exposed_time()),
                     ("exposed_given", collective.exposed_time(layers=12, width=512, devices=4, link=link,
                                                               backward_seconds=0.002))):
        for k, v in c[key].items():
            assert got[k] == pytest.approx(v, rel=1e-12), (key, k)


def test_column_kernel_order_is_tgcs_split_sum(gold):
    """The column kernel's declared order (oracle_col_parts with the kernel's rows per part)
    gives tgc's split_sum of each column bit for bit, at the backend's own part counts."""
    for case in gold["split_sum"]:
        rows, cols = case["rows"], case["cols"]
        parts, per = col_split(rows, cols)
        assert parts == case["parts"]
        assert reduction.column_plan(rows, cols).as_dict() == case["plan"]
        g = torch.Generator().manual_seed(rows * 31 + cols)
        x = torch.randn(rows, cols, generator=g)
        k = len(case["split_sum"])
        got = bracketing.col_parts(x[:, :k].contiguous().numpy(), per)
        np.testing.assert_array_equal(got, np.array(case["split_sum"], dtype=np.float32))
