"""CPU oracle for the B200 backend. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may
import anything here, and only as the checker or as the timed CPU baseline; the backend
(tensor-graph-compiler_b200/tgcb) never imports it and has no CPU path.

Contents, each restating a reference function (file:line in tgc's tree):
  interp.py      tgc/verify/reference.py:32-248  the torch-CPU interpreter tgc checks
                 everything against (evaluate_node, _reduce, interpret, run,
                 random_feeds, outputs_agree, relative_difference), and
                 tgc/codegen/emit.py:165-209 + tgc/runtime/executor.py:52-88 as
                 ``ArenaProgram``: the generated-Python path (one torch statement per
                 node into views of one arena), which is what the CPU baseline times.
  quantize.py    tgc/analysis/quantize.py:42-136, 229-240  symmetric per-row int8 schemes.
  bracketing.c   tgc/analysis/summation.py:47-131 (sequential, pairwise, partitioned, exact)
                 and the declared bracketing of every reduction kernel the backend emits,
                 so GPU reductions over exact summands can be checked bit for bit.

Pinning: tests/golden/make_golden.py ran tgc itself (this container, tgc importable) and
committed its outputs under tests/golden/; tests/test_oracle.py checks every function here
against those fixtures and against tgc's own known-answer assertions
(tests/test_summation.py:45,51,119; tests/test_reference.py:83-92; tests/test_quantize.py:95-110).
"""
