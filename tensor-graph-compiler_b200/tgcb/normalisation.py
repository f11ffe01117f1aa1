"""Row and batch normalisations as fused GPU kernels (tgc/analysis/normalisation.py).

Each function writes tgc's arithmetic as a graph with the same operations in the same order
(normalisation.py:51-101: ``values.pow(2)`` is ``x * x``, a mean keeps its dimension, the
epsilon is added before the square root, the gain multiplies after the division) and runs it
through ``tgcb.runtime.compile_graph``: ``rms_norm`` and ``layer_norm`` lower to one row
kernel (both reductions and the elementwise tail in one pass over each row), ``batch_norm`` to
column reductions plus one elementwise kernel, or, with stored statistics, to one elementwise
kernel. Compiled plans are kept by shape signature (``tgcb.cache.PlanCache``). The input checks
and their ``ConfigError`` messages follow tgc's ``_check`` (normalisation.py:104-109).
Results are fresh CUDA tensors.
"""

from __future__ import annotations

import torch

from tgcb import ir
from tgcb.cache import PlanCache
from tgcb.errors import ConfigError

_plans = PlanCache(capacity=64)


def _check(values: torch.Tensor, epsilon: float) -> None:
    if values.dim() != 2:
        raise ConfigError(f"a normalisation takes a matrix, got rank {values.dim()}")
    if epsilon <= 0:
        raise ConfigError(f"the epsilon has to be positive, got {epsilon}")
    if not values.is_cuda or values.dtype != torch.float32:
        raise ConfigError("the GPU normalisations take a float32 CUDA matrix")


def layer_norm_graph(rows: int, width: int, epsilon: float = 1e-5) -> ir.Graph:
    """centred / sqrt(mean(centred^2) + eps) * gain + offset (normalisation.py:51-58)."""
    b = ir.Builder()
    x = b.input([rows, width], name="values")
    gain = b.input([width], name="gain")
    offset = b.input([width], name="offset")
    centred = b.sub(x, b.mean(x, [1], keepdims=True))
    variance = b.mean(b.mul(centred, centred), [1], keepdims=True)
    scaled = b.div(centred, b.sqrt(b.add(variance, b.constant(epsilon))))
    return b.finish(b.add(b.mul(scaled, gain), offset))


def rms_norm_graph(rows: int, width: int, epsilon: float = 1e-5) -> ir.Graph:
    """values / sqrt(mean(values^2) + eps) * gain (normalisation.py:61-70)."""
    b = ir.Builder()
    x = b.input([rows, width], name="values")
    gain = b.input([width], name="gain")
    scale = b.mean(b.mul(x, x), [1], keepdims=True)
    return b.finish(b.mul(b.div(x, b.sqrt(b.add(scale, b.constant(epsilon)))), gain))


def batch_norm_graph(rows: int, width: int, epsilon: float = 1e-5, *, running: bool = False) -> ir.Graph:
    """(values - mean) / sqrt(variance + eps) * gain + offset over the batch (normalisation.py:73-101).

    Batch statistics: mean over rows, variance = mean of squared deviations (``var(unbiased=
    False)``). With ``running`` the mean and variance are inputs (stored statistics).
    """
    b = ir.Builder()
    x = b.input([rows, width], name="values")
    gain = b.input([width], name="gain")
    offset = b.input([width], name="offset")
    if running:
        mean = b.input([width], name="mean")
        variance = b.input([width], name="variance")
        centred = b.sub(x, mean)
    else:
        mean = b.mean(x, [0], keepdims=True)
        centred = b.sub(x, mean)
        variance = b.mean(b.mul(centred, centred), [0], keepdims=True)
    scaled = b.div(centred, b.sqrt(b.add(variance, b.constant(epsilon))))
    return b.finish(b.add(b.mul(scaled, gain), offset))


def _run(graph: ir.Graph, feeds: dict, device: int) -> torch.Tensor:
    compiled = _plans.get(graph, device=device)
    (out,) = compiled({k: v.contiguous() for k, v in feeds.items()})
    return out.clone()


def layer_norm(values: torch.Tensor, gain: torch.Tensor, offset: torch.Tensor, epsilon: float = 1e-5) -> torch.Tensor:
    _check(values, epsilon)
    rows, width = values.shape
    g = layer_norm_graph(rows, width, epsilon)
    return _run(g, {"values": values, "gain": gain, "offset": offset}, values.device.index)


def rms_norm(values: torch.Tensor, gain: torch.Tensor, epsilon: float = 1e-5) -> torch.Tensor:
    _check(values, epsilon)
    rows, width = values.shape
    g = rms_norm_graph(rows, width, epsilon)
    return _run(g, {"values": values, "gain": gain}, values.device.index)


def batch_norm(values: torch.Tensor, gain: torch.Tensor, offset: torch.Tensor, epsilon: float = 1e-5, *,
               running: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    _check(values, epsilon)
    rows, width = values.shape
    g = batch_norm_graph(rows, width, epsilon, running=running is not None)
    feeds = {"values": values, "gain": gain, "offset": offset}
    if running is not None:
        feeds["mean"], feeds["variance"] = (t.reshape(width) for t in running)
    return _run(g, feeds, values.device.index)
