"""The binding that lets tgc's own ``compile_graph`` hand a graph to this backend.

tgc compiles with ``tgc.runtime.executor.compile_graph(graph, *, pipeline=None,
optimise=True)`` (executor.py:91-122). A maintainer adds one keyword: ``backend="b200"``
sends the graph, tgc's own ``Graph`` object, to ``tgcb.runtime.compile_graph`` (which rebuilds
it in tgcb's IR and runs the same pipeline, order and plan); any other value keeps tgc's
emit-and-exec path. ``install`` does exactly that to an executor module in place (idempotent),
and ``uninstall`` puts the original back; ``with_backend`` builds the wrapper around any
``compile_graph`` with tgc's signature.
"""

from __future__ import annotations

from collections.abc import Callable

from tgcb.errors import ConfigError

BACKENDS = ("cpu", "b200")


def with_backend(original: Callable) -> Callable:
    """``original`` (tgc's compile_graph) extended by ``backend="cpu" | "b200"``."""

    def compile_graph(graph, *, pipeline=None, optimise: bool = True, backend: str = "cpu"):
        if backend == "b200":
            from tgcb import runtime

            return runtime.compile_graph(graph, pipeline=pipeline, optimise=optimise)
        if backend != "cpu":
            raise ConfigError(f"unknown backend {backend!r}, expected one of {list(BACKENDS)}")
        return original(graph, pipeline=pipeline, optimise=optimise)

    compile_graph.__wrapped__ = original
    compile_graph.__doc__ = (original.__doc__ or "") + "\n\nbackend: 'cpu' (generated Python) or 'b200' (tgcb)."
    return compile_graph


def install(executor) -> None:
    """Give ``executor.compile_graph`` (tgc.runtime.executor, or a stand-in) the backend keyword."""
    current = executor.compile_graph
    if getattr(current, "__wrapped__", None) is not None:
        return
    executor.compile_graph = with_backend(current)


def uninstall(executor) -> None:
    original = getattr(executor.compile_graph, "__wrapped__", None)
    if original is not None:
        executor.compile_graph = original
