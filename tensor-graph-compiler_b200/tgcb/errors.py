"""Exception hierarchy of the host side.

The class names and their parent/child relations are the ones tgc's callers already catch
(tgc/errors.py:4-41), so code written against tgc's executor handles a B200 failure with the
except clauses it already has. Two additions sit under ``CompilerError``: ``DeviceError`` for
a CUDA/NVRTC failure or a device-side timeout reported by the library, and ``ParseError`` for
the text format.
"""

from __future__ import annotations


class CompilerError(Exception):
    """Base of everything the backend raises (tgc/errors.py:4)."""


class ConfigError(CompilerError):
    """A caller asked for something that does not make sense (tgc/errors.py:8)."""


class GraphError(CompilerError):
    """A malformed graph (tgc/errors.py:12)."""


class TypeInferenceError(CompilerError):
    """A node's output type cannot be derived (tgc/errors.py:16)."""


class PassError(CompilerError):
    """A transformation could not be applied (tgc/errors.py:20)."""


class ScheduleError(CompilerError):
    """A graph cannot be scheduled as asked (tgc/errors.py:24)."""


class AllocationError(CompilerError):
    """Buffers cannot be placed, or a launch would touch bytes outside its slot (tgc/errors.py:28)."""


class CodegenError(CompilerError):
    """A scheduled graph cannot be lowered to kernels (tgc/errors.py:36)."""


class VerificationError(CompilerError):
    """Device output disagrees with the reference interpreter (tgc/errors.py:40)."""


class DeviceError(CompilerError):
    """The CUDA library returned a failure status; the message is its last-error text."""


class ParseError(GraphError):
    """Text that does not describe a graph (tgc/ir/serialize.py ParseError)."""
