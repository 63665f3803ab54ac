"""The allocation-free matmul entry point, piton_b200_matmul_f32_noalloc.

Callers that cannot allocate device memory (fixed-budget hosts, plugin hosts
that own every allocation) get the tensor-core matmul with its scratch taken
from a static device array inside the library.  This test calls it through
the C-ABI and checks it against the ordinary entry point (which takes a
caller-provided workspace) on three calls in a row (the last smaller than
the one before it, so leftovers in the shared array would show), within the
tolerance the matmul tests use; both run the same kernels, so the results are
expected to be identical bit for bit.  It also runs the CUDA-core branch
(which needs no scratch) through the same entry point, and checks that
problems too large for the static array are refused with an error instead of
running.

The file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""

import ctypes as C
import math

import pytest

pytestmark = pytest.mark.gpu


def _args(lib_mod, A, B, Cout, M, N, K, ws=None):
    a = lib_mod.MatmulArgs(A.data_ptr(), B.data_ptr(), Cout.data_ptr(), M, N, K, K, 1, N, 1, N, 1, 8, 64, 8, 8,
                           ((M + 7) // 8) * ((N + 63) // 64), 0, 0, 0, 0)
    if ws is not None:
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    return a


def _status(lib):
    s = C.c_int(-1)
    assert lib.piton_b200_device_status(C.byref(s)) == 0
    return s.value


def test_noalloc_matches_workspace_entry_point(cuda):
    torch = cuda
    from piton_b200.runtime.cuda import _lib
    lib = _lib.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the third call is smaller than the second: bytes the larger call left in the shared array
    # must never reach C
    for call, (M, N, K) in enumerate([(1024, 768, 1000), (1100, 1300, 1024), (256, 384, 512)]):
        g = torch.Generator(device="cuda").manual_seed(77 + call)
        A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
        B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
        ref_c = torch.empty(M, N, device="cuda")
        probe = _args(_lib, A, B, ref_c, M, N, K)
        need = lib.piton_b200_matmul_workspace_size(C.byref(probe))
        assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        _lib.check(lib.piton_b200_matmul_f32(C.byref(_args(_lib, A, B, ref_c, M, N, K, ws)), stream))
        out = torch.full((M, N), float("nan"), device="cuda")
        _lib.check(lib.piton_b200_matmul_f32_noalloc(C.byref(_args(_lib, A, B, out, M, N, K)), stream))
        torch.cuda.synchronize()
        assert _status(lib) == 0
        exact = A.double() @ B.double()
        scale = float(exact.abs().max())
        bound = max(4e-6, 1e-7 * math.sqrt(K))          # the fp32-level bound of test_gpu_matmul.py
        assert float((out.double() - exact).abs().max()) / scale <= bound
        assert float((out.double() - ref_c.double()).abs().max()) / scale <= bound
        assert torch.equal(out, ref_c)                    # same kernels, same bits


def test_noalloc_refuses_problems_beyond_its_scratch(cuda):
    torch = cuda
    from piton_b200.runtime.cuda import _lib
    lib = _lib.lib()
    M = N = K = 4096                                      # needs 256 MiB of scratch
    A = torch.zeros(M, K, device="cuda")
    B = torch.zeros(K, N, device="cuda")
    out = torch.full((M, N), 5.0, device="cuda")
    rc = lib.piton_b200_matmul_f32_noalloc(C.byref(_args(_lib, A, B, out, M, N, K)), C.c_void_p(0))
    assert rc == _lib.EINVAL
    assert b"scratch" in lib.piton_b200_last_error()
    torch.cuda.synchronize()
    assert bool((out == 5.0).all())


@pytest.mark.parametrize("shape,flags", [((40, 70, 36), 0), ((256, 256, 256), "FORCE_SIMT")])
def test_noalloc_cuda_core_branch_matches(cuda, shape, flags):
    """Shapes under 128 and the FORCE_SIMT flag take the CUDA-core path, which uses no scratch: the
    no-alloc entry point hands them to the ordinary one with the workspace cleared, so a garbage
    workspace pointer in the caller's args is never used and the result is the same bits."""
    torch = cuda
    from piton_b200.runtime.cuda import _lib
    lib = _lib.lib()
    M, N, K = shape
    fl = getattr(_lib, flags) if flags else 0
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    ref_c = torch.empty(M, N, device="cuda")
    ra = _args(_lib, A, B, ref_c, M, N, K)
    ra.flags = fl
    assert lib.piton_b200_matmul_workspace_size(C.byref(ra)) == 0
    _lib.check(lib.piton_b200_matmul_f32(C.byref(ra), stream))
    out = torch.full((M, N), float("nan"), device="cuda")
    na = _args(_lib, A, B, out, M, N, K)
    na.flags = fl
    na.workspace, na.workspace_bytes = 0xDEAD0000, 1 << 40     # never dereferenced
    _lib.check(lib.piton_b200_matmul_f32_noalloc(C.byref(na), stream))
    torch.cuda.synchronize()
    assert _status(lib) == 0
    assert torch.equal(out, ref_c)
