"""Generate the golden fixtures by running tgc itself. Run once, where tgc's source tree is
available (it is not on the GPU hosts); the outputs are committed next to this script.

    TGC_REFERENCE=<path to tgc's source tree> python tests/golden/make_golden.py

What it writes (all from tgc's own code paths on seeded inputs):
  graphs/*.tgc          tgc.ir.serialize.dumps of every workload graph, built with tgc's
                        Builder; the gradient graphs come from tgc.grad.reverse.gradient
                        followed by tgc's default pipeline. tgcb must print identical text.
  cone.npz              tgc.verify.reference.run of the cone at full size [4096,1024]
  mlp.npz               run() of the MLP block at 8192 rows: 48 sampled output rows plus
                        per-row float64 sums of every row; and the full output at 64 rows
  fixtures.npz          run() on tgc's builder fixtures (softmax, layernorm, diamond,
                        branching, mlp) with random_feeds(seed=0, positive=True), and the
                        executor's compiled outputs, which tgc holds bit-identical
  summation.json        tgc.analysis.summation orders on seeded vectors, incl. the 2^26 long
                        sum of the long-sum workload (sequential, pairwise, exact)
  quantize.npz          tgc.analysis.quantize per_row_schemes + quantise on seeded matrices
  int8.json / int8.npz  the int8 workload at full size: sha256 of qa, qwt, the int32
                        accumulator and the float32 output, the scale vectors, sampled rows
  train.npz             run() of the reverse-mode graph of the MLP at a small size
"""

from __future__ import annotations

import hashlib
import json
import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "tensor-graph-compiler_b200"))
REFERENCE = os.environ.get("TGC_REFERENCE")
if not REFERENCE:
    sys.exit("set TGC_REFERENCE to the root of tgc's source tree")
sys.path.insert(0, REFERENCE)

from tgc.analysis import quantize as tq  # noqa: E402
from tgc.analysis import summation as ts  # noqa: E402
from tgc.grad.reverse import gradient  # noqa: E402
from tgc.ir import builder as tb  # noqa: E402
from tgc.ir.dtype import FLOAT32, INT8, INT32  # noqa: E402
from tgc.ir.serialize import dumps  # noqa: E402
from tgc.runtime.executor import compile_graph, default_pipeline  # noqa: E402
from tgc.verify.reference import random_feeds, run  # noqa: E402

from tgcb import workloads as W  # noqa: E402

torch.set_num_threads(os.cpu_count() or 1)


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def write_graph(name: str, graph) -> None:
    os.makedirs(os.path.join(HERE, "graphs"), exist_ok=True)
    with open(os.path.join(HERE, "graphs", f"{name}.tgc"), "w") as f:
        f.write(dumps(graph))


def gradient_graph(rows: int, d: int, f: int):
    g = W.mlp_graph(tb.Builder, rows=rows, d=d, f=f, loss=True)
    res = gradient(g, ["w1", "b1", "w2", "b2"], seed_is_input=False)
    opt, _ = default_pipeline().run(res.graph)
    return g, res.graph, opt


def main() -> None:
    t0 = time.time()
    # ---- graphs as tgc prints them
    write_graph("cone", W.cone_graph(tb.Builder))
    write_graph("mlp", W.mlp_graph(tb.Builder))
    write_graph("mlp_loss_64", W.mlp_graph(tb.Builder, rows=64, loss=True))
    write_graph("int8_linear", W.int8_linear_graph(tb.Builder, INT8, INT32, FLOAT32))
    write_graph("sum", W.sum_graph(tb.Builder))
    for rows in (8192, 16384, 32768, 65536):
        _, raw, opt = gradient_graph(rows, 1024, 4096)
        write_graph(f"train_grad_{rows}", opt)
    _, raw_small, opt_small = gradient_graph(96, 64, 256)
    write_graph("train_grad_small", opt_small)
    write_graph("train_grad_small_raw", raw_small)
    for fx in ("softmax_graph", "layernorm_graph", "diamond_graph", "branching_graph", "mlp_graph"):
        write_graph(f"fixture_{fx}", getattr(tb, fx)())

    # ---- cone, full size
    g = W.cone_graph(tb.Builder)
    feeds = W.cone_inputs()
    outs = run(g, feeds)
    np.savez_compressed(
        os.path.join(HERE, "cone.npz"),
        row_sum=outs[0].numpy(), row_max=outs[1].numpy(), row_sum_tx=outs[2].numpy(),
        x_sha=np.frombuffer(sha(feeds["x"]).encode(), dtype=np.uint8),
    )

    # ---- mlp, full size (sampled rows + per-row sums) and a small full copy
    g = W.mlp_graph(tb.Builder)
    feeds = W.mlp_inputs()
    y = run(g, feeds)[0]
    rows = np.r_[0:16, 4096:4112, 8176:8192]
    gs = W.mlp_graph(tb.Builder, rows=64)
    fs = W.mlp_inputs(rows=64)
    ys = run(gs, fs)[0]
    np.savez_compressed(
        os.path.join(HERE, "mlp.npz"),
        rows=rows, y_rows=y[rows].numpy(), y_row_sums=y.double().sum(dim=1).numpy(),
        y64=ys.numpy(), x_sha=np.frombuffer(sha(feeds["x"]).encode(), dtype=np.uint8),
    )

    # ---- tgc's builder fixtures: interpreter and tgc's compiled path
    fx = {}
    for name in ("softmax_graph", "layernorm_graph", "diamond_graph", "branching_graph", "mlp_graph"):
        graph = getattr(tb, name)()
        feeds = random_feeds(graph, seed=0, positive=True)
        out = run(graph, feeds)
        compiled = compile_graph(graph)(feeds)
        assert all(torch.equal(a, b) for a, b in zip(out, compiled, strict=True))
        for k, t in feeds.items():
            fx[f"{name}/in/{k}"] = t.numpy()
        for i, t in enumerate(out):
            fx[f"{name}/out/{i}"] = t.numpy()
    np.savez_compressed(os.path.join(HERE, "fixtures.npz"), **fx)

    # ---- summation orders
    summ: dict = {"known": {}, "vectors": []}
    summ["known"]["mixed_4096_sequential"] = ts.sequential(ts.mixed_magnitudes(4096))
    summ["known"]["exact_0.1_0.2_0.3"] = ts.exact(np.asarray([0.1, 0.2, 0.3], dtype=np.float32))
    summ["known"]["tree_beats_loop"] = ts.the_tree_beats_the_loop()
    summ["known"]["best_split"] = ts.the_best_split_is_the_square_root()
    for count, seed, kind in ((1000, 1, "uniform"), (4096, 0, "mixed"), (65536, 0, "mixed"), (12345, 3, "alternating"), (1 << 20, 7, "uniform")):
        v = {"uniform": ts.uniform, "mixed": ts.mixed_magnitudes, "alternating": ts.alternating}[kind](count, seed=seed)
        summ["vectors"].append(
            {
                "kind": kind, "count": count, "seed": seed,
                "sequential": ts.sequential(v), "pairwise": ts.pairwise(v),
                "pairwise_block_3": ts.pairwise(v, block=3), "compensated": ts.compensated(v),
                "partitioned_64": ts.partitioned(v, 64) if count >= 64 else None, "exact": ts.exact(v),
            }
        )
    v, idx = W.longsum_input()
    vn = v.numpy()
    t1 = time.time()
    summ["longsum"] = {
        "n": int(v.numel()), "leader_index": idx, "x_sha": sha(v),
        "pairwise": ts.pairwise(vn), "sequential": ts.sequential(vn), "exact": math.fsum(vn.astype(np.float64).tolist()),
        "torch_sum": float(run(W.sum_graph(tb.Builder), {"x": v})[0]),
        "seconds_python_orders": None,
    }
    summ["longsum"]["seconds_python_orders"] = round(time.time() - t1, 1)
    with open(os.path.join(HERE, "summation.json"), "w") as f:
        json.dump(summ, f, indent=1)

    # ---- quantisation on seeded matrices (incl. a zero row and ties)
    gq = torch.Generator().manual_seed(11)
    mats = {
        "randn": torch.randn(64, 300, generator=gq),
        "weights_t": (torch.randn(512, 96, generator=gq) * 0.02).T.contiguous(),
        "edge": torch.cat([torch.zeros(1, 40), torch.arange(-20, 20, dtype=torch.float32).reshape(1, 40) * 0.5, torch.randn(2, 40, generator=gq)]),
    }
    qz = {}
    for name, m in mats.items():
        schemes = tq.per_row_schemes(m)
        q = torch.stack([tq.quantise(r, s) for r, s in zip(m, schemes, strict=True)])
        qz[f"{name}/x"] = m.numpy()
        qz[f"{name}/q"] = q.numpy()
        qz[f"{name}/scale"] = np.asarray([s.scale for s in schemes], dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, "quantize.npz"), **qz)

    # ---- int8 linear at full size: quantise with tgc, run the graph with tgc's interpreter
    ins = W.int8_inputs()
    a, w = ins["a"], ins["w"]
    sa_s = tq.per_row_schemes(a)
    qa = torch.stack([tq.quantise(r, s) for r, s in zip(a, sa_s, strict=True)]).to(torch.int8)
    wt = w.T.contiguous()
    sw_s = tq.per_row_schemes(wt)
    qwt = torch.stack([tq.quantise(r, s) for r, s in zip(wt, sw_s, strict=True)]).to(torch.int8)
    sa = torch.tensor([s.scale for s in sa_s], dtype=torch.float32).reshape(-1, 1)
    sw = torch.tensor([s.scale for s in sw_s], dtype=torch.float32).reshape(1, -1)
    gi = W.int8_linear_graph(tb.Builder, INT8, INT32, FLOAT32)
    t2 = time.time()
    acc, y = run(gi, {"qa": qa, "qwt": qwt, "sa": sa, "sw": sw})
    int8_secs = time.time() - t2
    srows = np.r_[0:8, 4000:4008, 8184:8192]
    np.savez_compressed(
        os.path.join(HERE, "int8.npz"), sa=sa.numpy(), sw=sw.numpy(), rows=srows,
        acc_rows=acc[srows].numpy(), y_rows=y[srows].numpy(),
    )
    with open(os.path.join(HERE, "int8.json"), "w") as f:
        json.dump(
            {"a_sha": sha(a), "qa_sha": sha(qa), "qwt_sha": sha(qwt), "acc_sha": sha(acc), "y_sha": sha(y),
             "interpreter_seconds": round(int8_secs, 1)}, f, indent=1,
        )

    # ---- reverse-mode graph at a small size
    gl, raw, opt = gradient_graph(96, 64, 256)
    feeds = W.mlp_inputs(rows=96, d=64, f=256, target=True)
    grads = run(raw, feeds)
    grads_opt = run(opt, feeds)
    np.savez_compressed(
        os.path.join(HERE, "train.npz"),
        **{f"in/{k}": t.numpy() for k, t in feeds.items()},
        **{f"grad/{i}": t.numpy() for i, t in enumerate(grads)},
        **{f"grad_opt/{i}": t.numpy() for i, t in enumerate(grads_opt)},
    )
    print(f"golden fixtures written in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
