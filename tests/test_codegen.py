"""Lowering: how graphs are partitioned into kernels, planned, and compiled (no GPU needed:
NVRTC compiles sm_100a code on any host)."""

from __future__ import annotations

import os

import pytest
from conftest import GOLDEN

from tgcb import codegen, ir, memory, runtime, serialize, workloads
from tgcb.codegen import row_threads
from tgcb.errors import CodegenError


def kinds(graph):
    return [s.kind for s in runtime.generate(graph)[3].steps]


def load_graph(name):
    with open(os.path.join(GOLDEN, "graphs", f"{name}.tgc")) as f:
        return serialize.loads(f.read())


def test_cone_is_one_row_kernel():
    _, _, plan, mod, low = runtime.generate(workloads.cone_graph(ir.Builder))
    assert [s.kind for s in mod.steps] == ["row"]
    # only x and the three row results touch memory: 16 MiB + 3 x 16 KiB
    assert mod.arena_bytes == 4096 * 1024 * 4 + 3 * 4096 * 4
    assert set(mod.steps[0].writes) == set(low.outputs)


def test_row_kernel_issues_its_loads_before_the_arithmetic(monkeypatch):
    """The cone's thread loads its 16 columns first; the additions keep their column order."""
    (step,) = runtime.generate(workloads.cone_graph(ir.Builder))[3].steps
    body = step.source[step.source.index("float acc_2"):]
    loads = [i for i, ln in enumerate(body.splitlines()) if "__ldg(" in ln]
    first_exp = next(i for i, ln in enumerate(body.splitlines()) if "expf(" in ln)
    assert len(loads) == 16 and max(loads) < first_exp
    offsets = [f"(long long)tid + {64 * k}LL" for k in range(16)]
    assert [body.index(o) for o in offsets] == sorted(body.index(o) for o in offsets)
    monkeypatch.setattr(codegen, "ROW_HOIST_LOADS", False)
    (inline,) = runtime.generate(workloads.cone_graph(ir.Builder))[3].steps
    lines = inline.source.splitlines()
    assert sorted(lines) == sorted(step.source.splitlines())  # the same statements, reordered
    assert lines != step.source.splitlines()


def test_row_prologue_body_keeps_loads_inline():
    """Inside the GEMM chain the layernorm body is left in its inline order (register budget)."""
    _, _, _, mod, _ = runtime.generate(workloads.mlp_graph(ir.Builder))
    src = mod.steps[0].source
    body = src[src.index("struct Rows_"):]
    first_add = body.index("acc_0 = acc_0 +")
    assert body.index("__ldg(") < first_add < body.rindex("__ldg(")


def test_mlp_is_layernorm_then_two_gemms(monkeypatch):
    monkeypatch.setattr(codegen, "CHAIN_GEMM", False)
    _, _, plan, mod, low = runtime.generate(workloads.mlp_graph(ir.Builder))
    assert [s.kind for s in mod.steps] == ["row", "gemm", "gemm"]
    ln, g1, g2 = mod.steps
    assert len(ln.writes) == 1  # the normalised x, read by the first GEMM
    assert "tgcb_tanh_approx" in g1.source  # GELU fused into the first GEMM's epilogue
    # whole 256 x 256 tiles: both GEMMs run on SM pairs
    assert "tgcb_gemm::gemm_body_pair<8192, 4096, 1024, false, false, true" in g1.source
    assert "tgcb_gemm::gemm_body_pair<8192, 1024, 4096, false, false, true" in g2.source
    assert all(ln.pair and ln.grid[0] % 2 == 0 for ln in g1.launches + g2.launches)


def test_mlp_is_one_launch_with_the_layernorm_as_row_prologue():
    _, _, plan, mod, low = runtime.generate(workloads.mlp_graph(ir.Builder))
    assert [s.kind for s in mod.steps] == ["gemm"]
    (ch,) = mod.steps
    (launch,) = ch.launches
    assert launch.gemm2 is not None and launch.block == (codegen.CHAIN_THREADS, 1, 1)
    # the layernorm body runs one row per epilogue warp: 8192 rows in groups of 16
    assert "struct Rows_tgcb_chain_4" in ch.source and "GROUPS = 512;" in ch.source
    assert ", Rows_tgcb_chain_4>(args" in ch.source and "tgcb_row_1(" not in ch.source
    # the normalised x is written and read inside the launch; counters for both GEMMs' waits
    assert launch.gemm[0].value in ch.writes
    assert launch.counter_bytes == 2 * (8192 // 256) * 4
    assert "layernorm" in ch.bracketing or "row tree: 32 threads per row" in ch.bracketing


def test_mlp_gemms_share_one_chain_launch(monkeypatch):
    monkeypatch.setattr(codegen, "ROW_PROLOGUE", False)
    _, _, plan, mod, low = runtime.generate(workloads.mlp_graph(ir.Builder))
    assert [s.kind for s in mod.steps] == ["row", "gemm"]
    ln, ch = mod.steps
    (launch,) = ch.launches
    assert launch.pair and launch.gemm2 is not None and launch.grid == (2 * codegen.NUM_SMS // 2, 1, 1)
    assert "tgcb_tanh_approx" in ch.source
    assert ("gemm_chain_pair<false, tgcb_gemm::PairGemm<8192, 4096, 1024, false, true, Epi_tgcb_gemm_2>, "
            "tgcb_gemm::PairGemm<8192, 1024, 4096, false, true, Epi_tgcb_gemm_3>") in ch.source
    # the hidden activation is the second GEMM's A operand; the counters (one per 256-row
    # block) get an arena slot of their own, zeroed by the runtime before each launch
    assert launch.gemm2[0].value in ch.writes and not launch.gemm2[0].mn_major
    assert launch.counters in ch.writes and launch.counter_bytes == 8192 // 256 * 4
    assert launch.counters in mod.offsets
    desc = mod.launches[-1]
    assert desc.is_gemm == 3 and desc.counter_bytes == 128 and desc.counter_offset % 4 == 0


def test_int8_linear_is_one_int8_gemm_with_fused_dequant():
    mod = runtime.generate(workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32))[3]
    assert [s.kind for s in mod.steps] == ["gemm"]
    # int8 operands read directly, both K-major (the weight arrives transposed)
    assert "gemm_body_pair<8192, 4096, 4096, true, false, false" in mod.steps[0].source
    assert len(mod.steps[0].writes) == 2  # the int32 accumulator and the dequantised output


def test_gradient_graph_lowers():
    g = load_graph("train_grad_8192")
    mod = runtime.generate(g)[3]
    ks = [s.kind for s in mod.steps]
    # five GEMMs; the forward pair (x1 @ W1 then h @ W2) shares one chain launch
    assert sum(2 if ln.gemm2 is not None else 1 for s in mod.steps for ln in s.launches if ln.gemm) == 5
    assert ks.count("gemm") == 4
    assert ks.count("colreduce") == 2
    # transposes are absorbed as operand majors, never materialised
    assert all("transpose" not in s.kind for s in mod.steps)


@pytest.mark.parametrize("cols,expect", [(1, 32), (1024, 32), (1025, 64), (4096, 128), (8192, 256), (20000, 256)])
def test_row_threads(cols, expect):
    assert row_threads(cols) == expect


@pytest.mark.parametrize("rows,cols,expect", [(8192, 1024, 32), (4096, 1024, 64), (64, 1024, 128), (64, 256, 32), (4, 70, 32)])
def test_row_threads_spread_few_rows(rows, cols, expect):
    """Few rows get more threads each (never below 8 columns per thread)."""
    assert row_threads(cols, rows) == expect


def test_plans_keep_live_values_apart():
    for g in (workloads.mlp_graph(ir.Builder, rows=512), load_graph("train_grad_small"), load_graph("fixture_softmax_graph")):
        og, order, plan, mod, low = runtime.generate(g)
        sizes = {v.name: v.bytes for v in og.inputs}
        for s in mod.steps:
            for w in s.writes:
                sizes[w] = low.scratch.get(w, low.values[w].bytes if w in low.values else 0)
        iv = memory.intervals_for_steps(low.inputs, [(s.reads, s.writes) for s in mod.steps], low.outputs, sizes)
        memory.validate_plan(iv, plan)


@pytest.mark.parametrize(
    "name",
    ["cone", "mlp", "int8", "grad_small", "fixture_softmax_graph", "fixture_layernorm_graph", "fixture_diamond_graph",
     "fixture_branching_graph", "fixture_mlp_graph", "sum"],
)
def test_generated_source_compiles_for_sm100a(name, tmp_path, monkeypatch):
    monkeypatch.setenv("TGCB_CACHE_DIR", str(tmp_path))
    build = {
        "cone": lambda: workloads.cone_graph(ir.Builder),
        "mlp": lambda: workloads.mlp_graph(ir.Builder, rows=1024),
        "int8": lambda: workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32, rows=256),
        "grad_small": lambda: load_graph("train_grad_small"),
        "sum": lambda: workloads.sum_graph(ir.Builder, n=1 << 20),
    }
    g = build[name]() if name in build else load_graph(name)
    cubin = runtime.compile_source(runtime.source_of(g))
    assert cubin[:4] == b"\x7fELF"


def test_refusals():
    b = ir.Builder()
    x = b.input(["n", 4], name="x")
    g = b.finish(b.exp(x))
    with pytest.raises(CodegenError):
        runtime.generate(g)
    b = ir.Builder()
    x = b.input([4, 4], ir.FLOAT64, name="x")
    g = b.finish(b.matmul(x, x))
    with pytest.raises(CodegenError):
        runtime.generate(g)
    b = ir.Builder()
    x = b.input([4, 4], ir.INT32, name="x")
    g = b.finish(b.matmul(x, x))
    with pytest.raises(CodegenError, match="int8"):
        runtime.generate(g)


def test_odd_gemm_rows_use_the_simt_fallback():
    b = ir.Builder()
    a = b.input([5, 3], name="a")
    w = b.input([3, 7], name="w")
    mod = runtime.generate(b.finish(b.matmul(a, w)))[3]
    assert mod.steps[0].kind == "gemm" and "SIMT" in mod.steps[0].bracketing


def test_compile_error_is_a_codegen_error():
    with pytest.raises(CodegenError):
        runtime.compile_source('extern "C" __global__ void k() { this is not cuda; }')


def test_fma_contraction_only_fuses_single_use_products():
    from tgcb.expr import contract_fma

    lines = [
        "    const float e_1 = (((float)a) * ((float)b));",
        "    const float e_2 = (((float)e_1) + ((float)c));",
        "    const float e_3 = (((float)a) * ((float)c));",
        "    const float e_4 = (((float)d) - ((float)e_3));",
        "    const float e_5 = (((float)a) * ((float)d));",
        "    const float e_6 = (((float)e_5) + ((float)e_5));",
    ]
    out = contract_fma(lines, ["e_2", "e_4", "e_6"])
    assert out[0] == "    const float e_2 = __fmaf_rn((float)a, (float)b, ((float)c));"
    assert out[1] == "    const float e_4 = __fmaf_rn((float)(-((float)a)), (float)c, ((float)d));"
    assert out[2:] == lines[4:]  # e_5 is read twice: left alone


def test_tf32_epilogues_approximate_int8_epilogues_exact():
    mlp = runtime.generate(workloads.mlp_graph(ir.Builder, rows=1024))[3]
    assert "tgcb_tanh_approx" in mlp.steps[1].source and "tanhf" not in mlp.steps[1].source
    int8 = runtime.generate(workloads.int8_linear_graph(ir.Builder, ir.INT8, ir.INT32, ir.FLOAT32, rows=256))[3]
    assert "__fmaf_rn" not in int8.steps[0].source and "approx" not in int8.steps[0].source
    cone = runtime.generate(workloads.cone_graph(ir.Builder))[3]
    assert "expf(" in cone.steps[0].source and "__expf" not in cone.steps[0].source


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K,kind", [(512, 512, 256, "f32"), (200, 300, 160, "f32"), (256, 96, 64, "f32"),
                                        (8192, 4096, 1024, "f32"), (256, 512, 256, "i8")])
def test_chunked_operand_maps_agree_with_the_kernels(ta, tb, M, N, K, kind):
    """The runtime encodes a 3-D (chunked) tensor map for exactly the operands the GEMM kernels
    load through one: tf32, MN-major, contiguous extent (the GEMM's M for A, N for B) a multiple
    of 32 (tgcb_gemm::chunked_mn), with tile_rows / 32 chunks per box."""
    import re

    b = ir.Builder()
    dt = ir.FLOAT32 if kind == "f32" else ir.INT8
    a = b.input([K, M] if ta else [M, K], dt, name="a")
    w = b.input([N, K] if tb else [K, N], dt, name="w")
    if kind == "i8":
        a, w = b.cast(a, ir.INT32), b.cast(w, ir.INT32)
    g = b.finish(b.matmul(b.transpose(a, [1, 0]) if ta else a, b.transpose(w, [1, 0]) if tb else w))
    _, _, _, module, _ = runtime.generate(g)
    gemms = [d for d in module.launches if d.is_gemm]
    if not gemms:
        return  # the SIMT fallback (rows TMA cannot tile) has no tensor maps
    d = gemms[0]
    m = re.search(r"gemm_(?:body_pair|body|split_pair)<(\d+), (\d+), (\d+), (true|false), (true|false), (true|false)",
                  module.source)
    assert m, "one tensor-core GEMM instantiation"
    gm, gn, _, is_int, a_mn, b_mn = m.groups()
    for op, mn, extent, tile in ((d.a, a_mn == "true", int(gm), 128), (d.b, b_mn == "true", int(gn), 128 if d.is_gemm == 2 else 256)):
        kernel_chunked = is_int == "false" and mn and extent % 32 == 0
        assert (op.chunks > 0) == kernel_chunked
        if kernel_chunked:
            assert op.cols == extent and op.swizzle == 1 and op.chunks == tile // 32


def test_column_reductions_store_their_reshaped_results_themselves():
    """A request that is the column sum element for element (the bias gradients' reshapes)
    is stored by the reduction's final kernel: no copy kernel follows it."""
    from tgcb import parallel

    mod = runtime.generate(parallel.train_graph(512))[3]
    kinds = [s.kind for s in mod.steps]
    assert "map" not in kinds and kinds.count("colreduce") == 2
    for s in mod.steps:
        if s.kind == "colreduce":
            assert len(s.writes) == 3 and len(s.launches) == 2


def test_requests_not_aligned_with_the_columns_keep_their_own_kernel():
    b = ir.Builder()
    x = b.input((4096, 1024), ir.FLOAT32, "x")
    total = b.sum(x, [0, 1])
    cols = b.sum(x, [0])
    mod = runtime.generate(b.finish(total, b.reshape(cols, (32, 32))))[3]
    assert [s.kind for s in mod.steps] == ["fullreduce", "colreduce", "map"]
