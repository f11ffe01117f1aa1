"""tgcb: a B200 (sm_100a) execution backend for tgc's compiled graphs.

Public surface, mirroring tgc's names:
  tgcb.ir            Builder, Graph, Node, Value, dtypes, the op table (tgc/ir/*)
  tgcb.passes        default_pipeline and the five exact passes (tgc/passes/*)
  tgcb.memory        depth_first_order, liveness, largest-first plan (tgc/schedule, tgc/analysis, tgc/memory)
  tgcb.serialize     dumps / loads of tgc's text format (tgc/ir/serialize.py)
  tgcb.runtime       compile_graph, CompiledGraph (tgc/runtime/executor.py)
  tgcb.summation     pairwise / sequential float32 sums on the GPU (tgc/analysis/summation.py)
  tgcb.quantize      per-row symmetric int8 quantisation on the GPU (tgc/analysis/quantize.py)
  tgcb.parallel      batch sharding across GPUs with NCCL (tgc/parallel/shard.py, collective.py)
"""

__version__ = "0.1.0"
