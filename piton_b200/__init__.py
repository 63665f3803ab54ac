"""piton_b200: the B200 (sm_100a) backend of PIton's ``kernel[grid](...)`` launch.

    import piton_b200 as triton
    from piton_b200.kernels import add_kernel
    add_kernel[(triton.cdiv(n, 256),)](x, y, out, n, BLOCK_SIZE=256, device="b200")

The launch surface mirrors piton/__init__.py and piton/jit.py; operators run
as hand-written CUDA kernels in libpiton_b200.so through a ctypes C-ABI
(include/piton_b200.h).
"""

from . import language
from .jit import JITFunction, jit, cdiv, next_power_of_2
from .runtime.launcher import offset_ptr

__all__ = ["jit", "JITFunction", "language", "cdiv", "next_power_of_2", "offset_ptr"]
