"""tgc's compiler fuzzer pointed at the B200 backend: generated graphs (the ones tgc's own
generator makes for the same seeds) compiled by tgcb, run on the GPU and compared with the
oracle's restatement of tgc's interpreter. Tolerance: atol = rtol = 1e-5 (CUDA's tanhf,
expf and the row kernels' declared summation order against ATen's). A failure is shrunk
before it is reported."""

from __future__ import annotations

import pytest

from oracle import interp
from tgcb import fuzz

pytestmark = pytest.mark.gpu

WIDE = fuzz.GeneratorConfig(nodes=16, inputs=3, rows=48, columns=200, reduction_chance=0.25)
BIG = fuzz.GeneratorConfig(nodes=24, inputs=3, rows=300, columns=1500, reduction_chance=0.25)


def _explain(report, config):
    lines = []
    for f in report.failures[:3]:
        small = fuzz.shrink(f.graph, lambda g, s=f.seed: bool(fuzz.check_one(g, s, interp.run, fuzz.DEFAULT_TOLERANCE)))
        lines.append(f"seed {f.seed}: {f.detail}; shrunk to {len(small.nodes)} nodes: "
                     + ", ".join(f"{n.name}={n.op.name}({', '.join(n.inputs)})" for n in small.nodes))
    return "\n".join(lines)


@pytest.mark.parametrize("config,count", [(None, 60), (WIDE, 30), (BIG, 12)], ids=["default", "wide", "big"])
def test_fuzz_compiler_against_the_interpreter(cuda, config, count):
    report = fuzz.fuzz_compiler(count, config, reference=interp.run)
    assert report.checked == count
    assert report.clean, _explain(report, config)
