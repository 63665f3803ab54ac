"""``kernel[grid](*args, device="b200", ...)``: binding and device dispatch.

Mirrors the reference launch path (piton/runtime/launcher.py:217-245):

* ``bind`` splits the call into (signature, constants, runtime values) with the
  reference's rules (launcher.py:42-63): ``tl.constexpr`` parameters and
  defaults are constants, integers equal to 1 are specialised into constants
  like Triton does, numpy arrays must be float32 / int32 / uint32
  (``TypeError`` otherwise).  B200 launches additionally accept CUDA torch
  tensors (used in place, no copies) and :func:`offset_ptr` views;
* the grid may be a tuple or ``callable(meta)``;
* ``num_warps`` / ``num_ctas`` are accepted and ignored; ``qpu_rounding=True``
  (or ``PITON_B200_QPU_ROUNDING=1``) selects the bit-exact QPU float mode;
* ``device="b200"`` (or ``"b200:<index>"``) runs the operator through the
  ctypes C-ABI (``piton_b200.runtime.cuda``); any other device raises
  ``ValueError`` as the reference does for unknown devices — the emulator and
  the Raspberry Pi stay with the reference.

The call returns a handle whose ``last_stats`` holds the launch's device time
(``time_us``), its algorithmic ``bytes`` and ``flops`` and the kernel ``path``.
"""

from __future__ import annotations

import inspect
import os

import numpy as np

from ..language import constexpr

_DTYPE_SIG = {np.dtype(np.float32): "*fp32", np.dtype(np.int32): "*i32", np.dtype(np.uint32): "*u32"}
_TORCH_SIG = {"torch.float32": "*fp32", "torch.int32": "*i32", "torch.uint32": "*u32"}


class offset_ptr:
    """A pointer argument ``elements`` past the start of ``base`` (numpy array or
    CUDA tensor).  The whole buffer is copied in and out as for a plain array;
    the kernel indexes from the offset, so negative strides may address the
    elements before it (the explicit-base idiom of tests/test_hw.py:185-199)."""

    def __init__(self, base, elements: int):
        self.base = base
        self.elements = int(elements)

    def __repr__(self):
        return f"offset_ptr({type(self.base).__name__}{list(self.base.shape)}, {self.elements})"


def _is_torch_tensor(v) -> bool:
    return type(v).__module__.startswith("torch") and hasattr(v, "data_ptr")


def _sig_of(value):
    if isinstance(value, offset_ptr):
        return _sig_of(value.base)
    if isinstance(value, np.ndarray):
        if value.dtype not in _DTYPE_SIG:
            raise TypeError(f"unsupported array dtype {value.dtype} (use float32/int32)")
        return _DTYPE_SIG[value.dtype]
    if _is_torch_tensor(value):
        sig = _TORCH_SIG.get(str(value.dtype))
        if sig is None:
            raise TypeError(f"unsupported tensor dtype {value.dtype} (use float32/int32)")
        return sig
    if isinstance(value, bool):
        return "i1"
    if isinstance(value, (int, np.integer)):
        return "i32"
    if isinstance(value, (float, np.floating)):
        return "fp32"
    raise TypeError(f"unsupported kernel argument {type(value).__name__}")


def bind(fn, args, kwargs, do_not_specialize=()):
    """Split launch arguments into (signature, constants, runtime values)."""
    sig = inspect.signature(fn)
    bound = sig.bind_partial(*args, **kwargs)
    signature, constants, values = {}, {}, {}
    for p in sig.parameters.values():
        if p.name not in bound.arguments:
            if p.default is inspect.Parameter.empty:
                raise TypeError(f"missing kernel argument '{p.name}'")
            constants[p.name] = p.default.value if isinstance(p.default, constexpr) else p.default
            continue
        v = bound.arguments[p.name]
        ann = p.annotation
        if _is_constexpr_annotation(ann):
            constants[p.name] = v
        elif isinstance(v, (int, np.integer)) and not isinstance(v, bool) and v == 1 \
                and p.name not in do_not_specialize:
            constants[p.name] = 1
        else:
            signature[p.name] = _sig_of(v)
            values[p.name] = v
    return signature, constants, values


def _is_constexpr_annotation(ann) -> bool:
    if ann is constexpr:
        return True
    if isinstance(ann, str):
        return "constexpr" in ann
    # the reference's own constexpr class (piton.language.core.constexpr)
    return isinstance(ann, type) and ann.__name__ == "constexpr"


def parse_device(device: str):
    """'b200' -> 0 (the current torch device is used), 'b200:3' -> 3."""
    if not isinstance(device, str) or not (device == "b200" or device.startswith("b200:")):
        raise ValueError(f"unknown device {device!r} (this backend runs device='b200'; "
                         f"the emulator and the Pi are the reference's)")
    if device == "b200":
        return None
    try:
        return int(device.split(":", 1)[1])
    except ValueError:
        raise ValueError(f"unknown device {device!r}") from None


class B200Launch:
    """What ``kernel[grid](...)`` returns: the bound launch and its last stats
    (the counterpart of the reference's CompiledKernel with ``last_stats``)."""

    def __init__(self, name, signature, constants):
        self.name = name
        self.signature = dict(signature)
        self.constants = dict(constants)
        self.last_stats = None

    def __repr__(self):
        return f"B200Launch({self.name}, {self.last_stats})"


class Launcher:
    def __init__(self, jitfn, grid, extra_constants=None):
        self.jitfn = jitfn
        self.grid = grid
        self.extra_constants = dict(extra_constants or {})

    def __call__(self, *args, device: str = "b200", num_stages: int = 2, **kwargs):
        fn = self.jitfn.fn
        launch_opts = {k: kwargs.pop(k) for k in list(kwargs) if k in ("num_warps", "num_ctas", "qpu_rounding")}
        dev_index = parse_device(device)
        signature, constants, values = bind(fn, args, kwargs, getattr(self.jitfn, "do_not_specialize", ()))
        constants.update(self.extra_constants)
        grid = self.grid(dict(constants, **values)) if callable(self.grid) else self.grid
        grid = tuple(int(g) for g in grid) if isinstance(grid, (tuple, list)) else (int(grid),)
        if not 1 <= len(grid) <= 3 or any(g < 0 for g in grid):
            raise ValueError(f"bad grid {grid}")
        key = (tuple(sorted(signature.items())), tuple(sorted((k, repr(v)) for k, v in constants.items())))
        cache = getattr(self.jitfn, "_cache", None)
        if cache is None:
            cache = {}
        handle = cache.get(("b200",) + key)
        if handle is None:
            handle = B200Launch(self.jitfn.__name__, signature, constants)
            cache[("b200",) + key] = handle
        qpu = launch_opts.get("qpu_rounding")
        if qpu is None:
            qpu = os.environ.get("PITON_B200_QPU_ROUNDING", "0") not in ("", "0")
        from .cuda import run_on_b200
        handle.last_stats = run_on_b200(self.jitfn, grid, constants, values, dev_index, bool(qpu))
        return handle
