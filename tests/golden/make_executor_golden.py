"""Graphs of tgc's executor tests, printed by tgc itself. Run once where tgc's source tree is
available (it is not on the GPU hosts):

    TGC_REFERENCE=<path to tgc's source tree> python tests/golden/make_executor_golden.py

Writes graphs/exec_<name>.tgc for the graphs tgc's tests/test_executor.py runs through
compile_graph (its GRAPHS table, plus the transpose pair and chain of tgc/passes/layout.py).
"""

from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
if not os.environ.get("TGC_REFERENCE"):
    sys.exit("set TGC_REFERENCE to the root of tgc's source tree")
sys.path.insert(0, os.environ["TGC_REFERENCE"])

from tgc.ir.builder import branching_graph, diamond_graph, elementwise_chain, layernorm_graph, mlp_graph, softmax_graph  # noqa: E402
from tgc.ir.serialize import dumps  # noqa: E402
from tgc.passes.layout import transposed_chain_graph, transposed_pair_graph  # noqa: E402

GRAPHS = {
    "chain": elementwise_chain(8, sizes=(8, 8)),
    "softmax": softmax_graph(),
    "layernorm": layernorm_graph(),
    "mlp": mlp_graph(),
    "diamond": diamond_graph(sizes=(8, 8)),
    "branching": branching_graph(4, 2, width=8),
    "transposed_pair": transposed_pair_graph(width=8),
    "transposed_chain": transposed_chain_graph(width=8),
}


def main() -> None:
    os.makedirs(os.path.join(HERE, "graphs"), exist_ok=True)
    for name, g in GRAPHS.items():
        with open(os.path.join(HERE, "graphs", f"exec_{name}.tgc"), "w") as f:
            f.write(dumps(g))
    print(f"{len(GRAPHS)} executor graphs written")


if __name__ == "__main__":
    main()
