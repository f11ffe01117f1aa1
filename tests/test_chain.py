"""The work lists of a two-GEMM chain (tgcb/chain.py) and when codegen fuses two GEMMs into one launch."""

from __future__ import annotations

import pytest

from tgcb import chain, codegen, ir, runtime, workloads
from tgcb.errors import CodegenError

SHAPES = [
    # (row blocks, first GEMM tiles per row, its k-blocks, second GEMM tiles per row, its k-blocks)
    (32, 16, 32, 4, 128),   # the MLP block, 8192 rows
    (256, 16, 32, 4, 128),  # its 65536-row forward pass in the training step
    (2, 2, 8, 1, 16),       # fewer tiles than SM pairs
    (1, 1, 1, 1, 1),
    (5, 3, 7, 2, 3),
]


@pytest.mark.parametrize("rows,tn1,kb1,tn2,kb2", SHAPES)
def test_every_tile_once_and_no_wait_cycle(rows, tn1, kb1, tn2, kb2):
    lists, span = chain.schedule(rows * tn1, tn1, kb1, rows * tn2, tn2, kb2, 74)
    assert len(lists) == 74
    chain.check(lists, rows * tn1, tn1, rows * tn2, tn2)
    # never worse than the two GEMMs as separate round-robin launches under the same costs
    assert span <= chain.two_launch_makespan(rows * tn1, kb1, rows * tn2, kb2, 74)


def test_the_mlp_block_schedule_beats_two_launches():
    lists, span = chain.schedule(512, 16, 32, 128, 4, 128, 74)
    assert span < 0.98 * chain.two_launch_makespan(512, 32, 128, 128, 74)
    # first-GEMM tiles are taken in row-major order, so row blocks complete in order
    firsts = sorted((lst.index(t), t) for lst in lists for t in lst if t < 512)
    assert firsts[0][1] == 0


def test_balanced_lists_end_sooner_for_the_mlp_block(monkeypatch):
    monkeypatch.setattr(chain, "BALANCED", False)
    greedy, greedy_span = chain.schedule(512, 16, 32, 128, 4, 128, 74)
    monkeypatch.setattr(chain, "BALANCED", True)
    lists, span = chain.schedule(512, 16, 32, 128, 4, 128, 74)
    assert span < greedy_span
    assert chain.simulate(lists, 512, 16, chain.tile_cost(32), 128, 4, chain.tile_cost(128)) == span
    # pairs with fewer second-GEMM tiles take more first-GEMM tiles
    by_second = {}
    for lst in lists:
        n2 = sum(1 for t in lst if t >= 512)
        by_second.setdefault(n2, set()).add(len(lst) - n2)
    counts = sorted(by_second)
    assert len(counts) > 1 and min(by_second[counts[0]]) > max(by_second[counts[-1]])


def test_every_split_gives_lists_without_wait_cycles():
    c1, c2 = chain.tile_cost(32), chain.tile_cost(128)
    for counts in chain._splits(128, 74):
        assert sum(counts) == 128 and len(counts) == 74
        lists = chain._balanced(512, c1, 128, c2, counts)
        chain.check(lists, 512, 16, 128, 4)


def test_check_refuses_a_missing_or_repeated_tile():
    with pytest.raises(CodegenError, match="exactly once"):
        chain.check([[0, 1], [3]], 2, 1, 2, 1)  # second-GEMM tile 0 (item 2) missing
    with pytest.raises(CodegenError, match="exactly once"):
        chain.check([[0, 1, 2], [2]], 2, 1, 1, 1)  # item 2 twice


def test_check_refuses_waits_that_form_a_cycle():
    # one first-GEMM tile per row block: item 2 (second GEMM, row 0) waits for item 0 and item 3
    # (row 1) for item 1. Pair 0 runs 2 before 1 and pair 1 runs 3 before 0: each waits on the other.
    lists = [[2, 1], [3, 0]]
    with pytest.raises(CodegenError, match="cycle"):
        chain.check(lists, 2, 1, 2, 1)
    chain.check([[0, 2], [1, 3]], 2, 1, 2, 1)  # the same tiles in a feasible order


def test_chain_needs_matching_row_blocks():
    with pytest.raises(CodegenError):
        chain.schedule(32, 16, 4, 12, 4, 4, 74)


def _linear_pair(rows, k, n1, n2, second_b_from_first=False):
    b = ir.Builder()
    x = b.input((rows, k), ir.FLOAT32, "x")
    w1 = b.input((k, n1), ir.FLOAT32, "w1")
    h = b.relu(b.matmul(x, w1))
    if second_b_from_first:
        # the second GEMM's B operand is the first one's output: not a chain
        y = b.matmul(b.input((n2, rows), ir.FLOAT32, "z"), h)
    else:
        y = b.matmul(h, b.input((n1, n2), ir.FLOAT32, "w2"))
    return b.finish(y)


def test_two_linears_fuse_into_one_launch():
    mod = runtime.generate(_linear_pair(512, 256, 512, 256))[3]
    gemms = [s for s in mod.steps if s.kind == "gemm"]
    assert len(gemms) == 1 and gemms[0].launches[0].gemm2 is not None


def test_no_chain_when_the_second_gemm_reads_the_first_as_b():
    mod = runtime.generate(_linear_pair(512, 256, 512, 256, second_b_from_first=True))[3]
    assert all(ln.gemm2 is None for s in mod.steps for ln in s.launches)


def test_no_chain_when_disabled(monkeypatch):
    monkeypatch.setattr(codegen, "CHAIN_GEMM", False)
    mod = runtime.generate(workloads.mlp_graph(ir.Builder))[3]
    assert [s.kind for s in mod.steps] == ["row", "gemm", "gemm"]


def test_layernorm_becomes_the_chains_row_prologue_only_for_few_rows():
    # 8192 rows: 512 groups of 16 rows, 4 per CTA -> inside the chain launch
    mod = runtime.generate(workloads.mlp_graph(ir.Builder, rows=8192))[3]
    assert [s.kind for s in mod.steps] == ["gemm"]
    assert "Rows_" in mod.steps[0].source
    # 65536 rows: 28 groups per CTA would hold the epilogue warps back -> its own launch
    mod = runtime.generate(workloads.mlp_graph(ir.Builder, rows=65536))[3]
    assert [s.kind for s in mod.steps] == ["row", "gemm"]
    # 64 threads per row (2048 rows of 1024): shared-memory partials, never a prologue
    mod = runtime.generate(workloads.mlp_graph(ir.Builder, rows=2048))[3]
    assert [s.kind for s in mod.steps] == ["row", "gemm"]


@pytest.mark.parametrize(
    "m,n,k,split",
    [
        (1024, 1024, 65536, 4),   # 16 tiles: 4 slices fill 64 of 74 pairs
        (512, 1024, 65536, 8),    # 8 tiles
        (256, 256, 4096, 8),      # 1 tile, 128 k-blocks: 8 slices of 16
        (256, 256, 1024, 2),      # 32 k-blocks: 2 slices of 16
        (256, 256, 256, 1),       # 8 k-blocks: too short to split
        (1024, 4096, 65536, 1),   # 64 tiles: slices would run in different rounds
        (2048, 2048, 65536, 1),   # 64 tiles
    ],
)
def test_k_split_only_when_every_slice_runs_at_once(m, n, k, split):
    b = ir.Builder()
    x = b.input((k, m), ir.FLOAT32, "x")
    dy = b.input((k, n), ir.FLOAT32, "dy")
    mod = runtime.generate(b.finish(b.matmul(b.transpose(x, [1, 0]), dy)))[3]
    (step,) = mod.steps
    (launch,) = step.launches
    tiles = (m // 256) * (n // 256)
    if split == 1:
        assert launch.counters is None and "slices" not in step.bracketing
        return
    assert f"K cut into {split} equal slices" in step.bracketing
    assert f"gemm_split_pair<{m}, {n}, {k}, false, true, true, Epi_tgcb_gemm_1, {split}>" in step.source
    assert launch.grid[0] == 2 * tiles * split and tiles * split <= codegen.NUM_SMS // 2
    assert launch.counter_bytes == tiles * 32 * 4
    # the workspace holds every slice's partial
    ws = [w for w in step.writes if w.endswith("_partials")]
    assert len(ws) == 1 and mod.offsets[ws[0]] % 256 == 0
