"""The names a PIton/Triton kernel module touches at definition time.

Kernels launched on the B200 backend are never traced: their bodies are not
executed, only their signatures are bound (piton/runtime/launcher.py:42-63).
So this module provides ``constexpr`` (used in parameter annotations and by
``bind``) and stand-ins for the ``tl.*`` builtins that raise if a kernel body is
ever called directly, as ``JITFunction.__call__`` does in the reference
(piton/jit.py:26-27).
"""

from __future__ import annotations


class constexpr:
    """Annotation for compile-time parameters (piton/language/core.py's constexpr)."""

    def __init__(self, value=None):
        self.value = value.value if isinstance(value, constexpr) else value

    def __repr__(self):
        return f"constexpr[{self.value!r}]"


class dtype:
    def __init__(self, name: str):
        self.name = name

    def __repr__(self):
        return self.name


float32 = dtype("fp32")
int32 = dtype("i32")
uint32 = dtype("u32")
int1 = dtype("i1")


def _device_only(name):
    def f(*_args, **_kwargs):
        raise RuntimeError(f"tl.{name} is only meaningful inside a kernel launched with kernel[grid](...)")
    f.__name__ = name
    return f


for _name in ("program_id", "num_programs", "arange", "zeros", "full", "load", "store", "dot", "max", "min", "sum",
              "maximum", "minimum", "where", "exp", "exp2", "log", "log2", "sqrt", "rsqrt", "sigmoid", "cdiv",
              "abs", "fma", "softmax", "static_range", "multiple_of", "max_contiguous"):
    globals()[_name] = _device_only(_name)

del _name
