"""The five workloads the backend is measured on, as graphs and seeded inputs.

Each graph builder takes a ``Builder`` class so the same function builds the graph with
tgcb's IR (on any host) or with tgc's own ``Builder`` (where tgc is installed); the golden
fixtures check the two print identically. Inputs come from one seeded
``torch.Generator().manual_seed(seed)`` in a fixed order, so every host regenerates the same
tensors.

1. cone     x [4096,1024] ~ N(0,1); t = exp(0.5*x - 1); row-sum(t), row-max(t), row-sum(t*x)
2. mlp      layernorm (gamma=1, beta=0, eps=1e-5) -> x@W1+b1 -> tanh-form GELU -> @W2+b2;
            x [8192,1024] ~ N(0,1), W1 [1024,4096], W2 [4096,1024] ~ N(0,0.02), zero biases
3. longsum  2^26 values ~ U(0,1) with one seeded entry set to 1e8
4. int8     A [8192,4096] ~ N(0,1) per-token, W [4096,4096] ~ N(0,0.02) per-output-channel
            symmetric int8; int32 GEMM; dequantised by the two scale vectors
5. train    mean((mlp(x) - target)^2) over a batch shard, gradients for W1, b1, W2, b2
"""

from __future__ import annotations

import torch

GELU_K = 0.7978845608028654  # sqrt(2 / pi)
GELU_C = 0.044715
LN_EPS = 1e-5


def cone_graph(B, rows: int = 4096, cols: int = 1024):
    b = B()
    x = b.input([rows, cols], name="x")
    a = b.constant(0.5)
    c = b.constant(-1.0)
    t = b.exp(b.add(b.mul(x, a), c))
    return b.finish(b.sum(t, [1]), b.max(t, [1]), b.sum(b.mul(t, x), [1]))


def row_sum_graph(B, rows: int = 4096, cols: int = 1024):
    """The cone's input read once and summed per row, nothing else: the same row kernel launch
    shape as the cone with no arithmetic to hide, the ceiling a launch over these bytes reaches."""
    b = B()
    x = b.input([rows, cols], name="x")
    return b.finish(b.sum(x, [1]))


def _gelu_tanh(b, h):
    k = b.constant(GELU_K)
    c = b.constant(GELU_C)
    half = b.constant(0.5)
    one = b.constant(1.0)
    cube = b.mul(b.mul(h, h), h)
    inner = b.mul(b.add(h, b.mul(cube, c)), k)
    return b.mul(b.mul(h, half), b.add(one, b.tanh(inner)))


def mlp_graph(B, rows: int = 8192, d: int = 1024, f: int = 4096, loss: bool = False):
    """Layernorm -> GEMM+bias -> GELU (tanh form, composed from mul/add/tanh) -> GEMM+bias.

    tgc has no GELU or erf op (tgc/ir/op.py:84-161), so GELU is the composition a frontend
    would trace; layernorm is tgc's own pattern (tgc/ir/builder.py:267-278) with gamma=1 and
    beta=0 left out; the bias add follows tgc/frontend/module.py:106-112.
    """
    b = B()
    x = b.input([rows, d], name="x")
    w1 = b.input([d, f], name="w1")
    b1 = b.input([f], name="b1")
    w2 = b.input([f, d], name="w2")
    b2 = b.input([d], name="b2")
    mean = b.mean(x, [1], keepdims=True)
    cen = b.sub(x, mean)
    var = b.mean(b.mul(cen, cen), [1], keepdims=True)
    ln = b.div(cen, b.sqrt(b.add(var, b.constant(LN_EPS))))
    h = b.add(b.matmul(ln, w1), b.broadcast_to(b1, [rows, f]))
    y = b.add(b.matmul(_gelu_tanh(b, h), w2), b.broadcast_to(b2, [rows, d]))
    if not loss:
        return b.finish(y)
    t = b.input([rows, d], name="target")
    e = b.sub(y, t)
    return b.finish(b.mean(b.mul(e, e), [0, 1]))


def sum_graph(B, n: int = 1 << 26):
    b = B()
    x = b.input([n], name="x")
    return b.finish(b.sum(x, [0]))


def int8_linear_graph(B, I8, I32, F32, rows: int = 8192, k: int = 4096, n: int = 4096):
    """cast(int8 -> int32) x2, int32 matmul, cast to float32, per-token then per-channel scale.

    The weight comes in as its per-output-channel rows qwt [n, k] (the layout per_row_schemes
    quantises) and is transposed in the graph, so the GEMM reads it K-major.
    """
    b = B()
    qa = b.input([rows, k], I8, name="qa")
    qwt = b.input([n, k], I8, name="qwt")
    sa = b.input([rows, 1], F32, name="sa")
    sw = b.input([1, n], F32, name="sw")
    acc = b.matmul(b.cast(qa, I32), b.transpose(b.cast(qwt, I32), [1, 0]))
    y = b.mul(b.mul(b.cast(acc, F32), sa), sw)
    return b.finish(acc, y)


# ----------------------------------------------------------------------------- inputs


def cone_inputs(rows: int = 4096, cols: int = 1024, seed: int = 0) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    return {"x": torch.randn(rows, cols, generator=g)}


def mlp_inputs(rows: int = 8192, d: int = 1024, f: int = 4096, seed: int = 0, target: bool = False) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    feeds = {
        "x": torch.randn(rows, d, generator=g),
        "w1": torch.randn(d, f, generator=g) * 0.02,
        "w2": torch.randn(f, d, generator=g) * 0.02,
        "b1": torch.zeros(f),
        "b2": torch.zeros(d),
    }
    if target:
        feeds["target"] = torch.randn(rows, d, generator=g)
    return feeds


def longsum_input(n: int = 1 << 26, seed: int = 0) -> tuple[torch.Tensor, int]:
    g = torch.Generator().manual_seed(seed)
    v = torch.rand(n, generator=g)
    idx = int(torch.randint(0, n, (1,), generator=g))
    v[idx] = 1e8
    return v, idx


def int8_inputs(rows: int = 8192, k: int = 4096, n: int = 4096, seed: int = 0) -> dict[str, torch.Tensor]:
    """Float activations A [rows,k] and weights W [k,n] (before quantisation)."""
    g = torch.Generator().manual_seed(seed)
    return {"a": torch.randn(rows, k, generator=g), "w": torch.randn(k, n, generator=g) * 0.02}
