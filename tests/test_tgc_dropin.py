"""The drop-in on tgc's own objects (tgc/runtime/executor.py:91-122).

With tgc's source tree importable (``TGC_REFERENCE`` names it; skipped otherwise), each
workload graph is built with tgc's own Builder (and the training graph with tgc's own
``gradient``) and handed to the backend: it must reach the same kernels, launches and
generated source as the graph built with tgcb's Builder. The ``backend="b200"`` binding
(tgcb.tgc_backend) is exercised on a stand-in executor module here, and on tgc's real
``tgc.runtime.executor`` when tgc is importable. Without a GPU the compile stops at the device
check (there is no CPU path), which is asserted too.
"""

from __future__ import annotations

import importlib
import os
import sys
import types

import pytest

from tgcb import grad, ir, runtime, tgc_backend, workloads
from tgcb.errors import ConfigError, DeviceError


def _tgc():
    root = os.environ.get("TGC_REFERENCE")
    if not root:
        pytest.skip("TGC_REFERENCE does not name tgc's source tree")
    if root not in sys.path:
        sys.path.insert(0, root)
    try:
        return importlib.import_module("tgc.ir.builder"), importlib.import_module("tgc.ir.dtype")
    except ImportError as e:
        pytest.skip(f"tgc is not importable from TGC_REFERENCE: {e}")


def _pairs(tb, td):
    grads = ["w1", "b1", "w2", "b2"]
    tgc_grad = importlib.import_module("tgc.grad.reverse").gradient
    return {
        "cone": (workloads.cone_graph(tb.Builder), workloads.cone_graph(ir.Builder)),
        "mlp": (workloads.mlp_graph(tb.Builder), workloads.mlp_graph(ir.Builder)),
        "int8": (workloads.int8_linear_graph(tb.Builder, td.INT8, td.INT32, td.FLOAT32),
                 workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32)),
        "sum": (workloads.sum_graph(tb.Builder), workloads.sum_graph(ir.Builder)),
        "train": (tgc_grad(workloads.mlp_graph(tb.Builder, rows=8192, loss=True), grads, seed_is_input=False).graph,
                  grad.gradient(workloads.mlp_graph(ir.Builder, rows=8192, loss=True), grads, seed_is_input=False).graph),
        "softmax": (tb.softmax_graph(), None),
    }


def test_tgc_graphs_reach_the_same_kernels():
    tb, td = _tgc()
    for name, (theirs, ours) in _pairs(tb, td).items():
        assert type(theirs).__module__.startswith("tgc."), name
        opt_t, _, _, mod_t, _ = runtime.generate(theirs)
        if ours is None:
            assert mod_t.launches, name
            continue
        opt_o, _, _, mod_o, _ = runtime.generate(ours)
        assert str(opt_t) == str(opt_o), name
        assert mod_t.source == mod_o.source, name
        assert [(s.kind, s.label, s.bracketing) for s in mod_t.steps] == [(s.kind, s.label, s.bracketing) for s in mod_o.steps]
        assert mod_t.arena_bytes == mod_o.arena_bytes


def test_backend_keyword_on_a_stand_in_executor():
    calls = []

    def original(graph, *, pipeline=None, optimise=True):
        calls.append((graph, pipeline, optimise))
        return "cpu-compiled"

    executor = types.SimpleNamespace(compile_graph=original)
    tgc_backend.install(executor)
    tgc_backend.install(executor)  # idempotent
    g = workloads.cone_graph(ir.Builder, rows=8, cols=32)
    assert executor.compile_graph(g) == "cpu-compiled" and calls[-1] == (g, None, True)
    assert executor.compile_graph(g, optimise=False, backend="cpu") == "cpu-compiled" and calls[-1][2] is False
    with pytest.raises(ConfigError):
        executor.compile_graph(g, backend="tpu")
    import torch

    if not torch.cuda.is_available():
        with pytest.raises(DeviceError):  # the b200 path was taken, and it has no CPU fallback
            executor.compile_graph(g, backend="b200")
    tgc_backend.uninstall(executor)
    assert executor.compile_graph is original


def test_backend_keyword_on_tgcs_executor():
    tb, _ = _tgc()
    executor = importlib.import_module("tgc.runtime.executor")
    original = executor.compile_graph
    tgc_backend.install(executor)
    try:
        g = tb.softmax_graph()
        assert type(executor.compile_graph(g)).__module__ == "tgc.runtime.executor"  # tgc's own path still works
        import torch

        if not torch.cuda.is_available():
            with pytest.raises(DeviceError):
                executor.compile_graph(g, backend="b200")
        else:
            compiled = executor.compile_graph(g, backend="b200")
            assert type(compiled).__module__ == "tgcb.runtime"
    finally:
        tgc_backend.uninstall(executor)
    assert executor.compile_graph is original
