"""Golden numbers of tgc's models and reduction splits, made by running tgc itself.

    TGC_REFERENCE=<path to tgc's source tree> python tests/golden/make_model_golden.py

Writes models.json:
  fusion_search   tgc.schedule.fusion_search on chain_dag, cone_dag (the cone workload's shape,
                  several intensities, readers and memory weights): every strategy's plan and
                  cost, group_for and times_computed of the tip, duplication factors
  cost            tgc.analysis.cost.estimate (flops, fused and unfused bytes) of the workload
                  graphs built with tgc's Builder, on tgc's machines
  collective      tgc.parallel.collective ring/tree times and volumes, bucket_time over tgc's
                  gradient stack and over the training step's four gradients, exposed_time
  split_sum       tgc.passes.reduction.split_sum of seeded columns at the row counts and part
                  counts the backend's column kernels use, and SplitPlan.as_dict for each
"""

from __future__ import annotations

import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "tensor-graph-compiler_b200"))
REFERENCE = os.environ.get("TGC_REFERENCE")
if not REFERENCE:
    sys.exit("set TGC_REFERENCE to the root of tgc's source tree")
sys.path.insert(0, REFERENCE)

from tgc.analysis import cost as tc  # noqa: E402
from tgc.grad.reverse import gradient  # noqa: E402
from tgc.ir import builder as tb  # noqa: E402
from tgc.ir.dtype import FLOAT32, INT8, INT32  # noqa: E402
from tgc.parallel import collective as tcol  # noqa: E402
from tgc.passes import reduction as tr  # noqa: E402
from tgc.schedule import fusion_search as fs  # noqa: E402

from tgcb import workloads as W  # noqa: E402
from tgcb.codegen import col_split  # noqa: E402

# (rows, columns) of column reductions the backend emits: the bias gradients of the training
# step at 65536 and 8192 rows per GPU (4096 and 1024 columns), and two ragged shapes; the part
# count is the one the backend's column kernel picks for the shape (tgcb.codegen.col_split)
SPLITS = [(65536, 4096), (65536, 1024), (8192, 4096), (8192, 1024), (1000, 7), (37, 3)]
SPLIT_COLUMNS = 3


def plans(dag) -> dict:
    return {row["strategy"]: row for row in fs.compare_strategies(dag)}


def main() -> None:
    out: dict = {}
    dags = {
        "chain": fs.chain_dag(),
        "cone_3_4": fs.cone_dag(readers=3, depth=4),
        "cone_3_4_x8": fs.cone_dag(readers=3, depth=4, intensity=8),
        "cone_3_4_x16": fs.cone_dag(readers=3, depth=4, intensity=16),
        "cone_3_4_x64": fs.cone_dag(readers=3, depth=4, intensity=64),
        "cone_5_2": fs.cone_dag(readers=5, depth=2),
    }
    out["fusion_search"] = {
        "dags": {k: {"producers": d.producers, "sizes": d.sizes, "flops": d.flops, "outputs": d.outputs,
                     "barriers": d.barriers, "interior": d.interior} for k, d in dags.items()},
        "plans": {k: plans(d) for k, d in dags.items()},
        "weights": {str(w): fs.exhaustive(dags["cone_3_4_x8"], w).as_dict() for w in (0.0, 0.1, 1.0, 10.0, 100.0)},
        "tip_group_outputs_only": sorted(fs.group_for(dags["cone_3_4"], 5, fs.normalise(dags["cone_3_4"], ()))),
        "tip_computed": fs.times_computed(dags["cone_3_4"], (), 4),
        "tip_computed_reused": fs.times_computed(dags["cone_3_4"], [4], 4),
        "duplication": {k: fs.duplication_factor(d, ()) for k, d in dags.items()},
        "intensity_sweep": fs.intensity_sweep(),
        "crossover": fs.the_crossover_is_a_property_of_the_machine(),
    }
    graphs = {
        "cone": W.cone_graph(tb.Builder),
        "mlp": W.mlp_graph(tb.Builder),
        "int8": W.int8_linear_graph(tb.Builder, INT8, INT32, FLOAT32),
        "sum": W.sum_graph(tb.Builder),
        "train_8192": gradient(W.mlp_graph(tb.Builder, rows=8192, loss=True), ["w1", "b1", "w2", "b2"],
                               seed_is_input=False).graph,
    }
    cost = {}
    for name, g in graphs.items():
        row = {"flops": tc.graph_flops(g), "fused_bytes": tc.fused_bytes(g), "unfused_bytes": tc.unfused_bytes(g)}
        for m in tc.MACHINES.values():
            row[m.name] = tc.estimate(g, m).as_dict()
        cost[name] = row
    out["cost"] = cost
    payload = [1024 * 4096 * 4, 4096 * 4, 4096 * 1024 * 4, 1024 * 4]
    link = tcol.Link(name="given", bytes_per_second=770e9, latency_seconds=20e-6)
    out["collective"] = {
        "ring_time": {str(n): tcol.ring_time(33574912, n) for n in (1, 2, 4, 8)},
        "tree_time": {str(n): tcol.tree_time(33574912, n) for n in (1, 2, 4, 8)},
        "ring_volume": {str(n): tcol.ring_volume(33574912, n) for n in (1, 2, 4, 8)},
        "tree_volume": {str(n): tcol.tree_volume(33574912, n) for n in (1, 2, 4, 8)},
        "given_link_ring_time": {str(n): tcol.ring_time(33574912, n, link) for n in (2, 4, 8)},
        "bucket_sweep": tcol.bucket_sweep(),
        "train_buckets": {str(b): tcol.bucket_time(payload, 8, link, b) for b in (0, 1 << 20, 1 << 26)},
        "exposed_default": tcol.exposed_time(),
        "exposed_given": tcol.exposed_time(layers=12, width=512, devices=4, link=link, backward_seconds=0.002),
    }
    splits = []
    for rows, cols in SPLITS:
        parts, _ = col_split(rows, cols)
        g = torch.Generator().manual_seed(rows * 31 + cols)
        x = torch.randn(rows, cols, generator=g)
        values = [tr.split_sum(x[:, c].contiguous(), parts) for c in range(min(cols, SPLIT_COLUMNS))]
        splits.append({"rows": rows, "cols": cols, "parts": parts, "split_sum": values,
                       "plan": tr.SplitPlan(rows, parts).as_dict(), "exact": [tr.exact_sum(x[:, c]) for c in range(min(cols, SPLIT_COLUMNS))]})
    out["split_sum"] = splits
    with open(os.path.join(HERE, "models.json"), "w") as f:
        json.dump(out, f, indent=1, default=list)
    print("wrote models.json")


if __name__ == "__main__":
    main()
