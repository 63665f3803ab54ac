"""Which host-buffer launches take the chunked copy/launch overlap (runtime/cuda
``_pipelined_on_host``), checked on the CPU: every rule that sends a launch back to the generic
path (copy everything in, launch, copy everything back) is decided from the numpy arrays alone,
before any CUDA call.  A launch that passes every rule goes on to create the copy streams, which
on a machine without a GPU raises; that is how the test sees it was accepted."""

import types

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from piton_b200.runtime.cuda import PIPE_MIN_BYTES, _pipelined_on_host

N = PIPE_MIN_BYTES // 8          # elements: two float32 arrays of this size reach the threshold


def fake_launch():
    return types.SimpleNamespace(capturing=False, device=torch.device("cpu"), host_h2d=0, host_d2h=0)


def never(*_):
    raise AssertionError("no chunk may be launched")


@pytest.fixture
def pinned(monkeypatch):
    """Every tensor reports page-locked memory, so the other rules decide."""
    monkeypatch.setattr(torch.Tensor, "is_pinned", lambda self, *a, **k: True)


def run(ins, outs, units, align=1):
    return _pipelined_on_host(fake_launch(), ins, outs, units, align, never)


def test_arrays_that_are_not_page_locked_take_the_generic_path():
    x, y = np.zeros(N, np.float32), np.zeros(N, np.float32)
    assert run([("x", x, 1)], [("y", y, 1)], N) is False


@pytest.mark.usefixtures("pinned")
def test_generic_path_rules():
    x, y = np.zeros(N, np.float32), np.zeros(N, np.float32)
    assert run([("x", x, 1)], [("y", y, 1)], 0) is False                             # nothing to do
    small = np.zeros(1024, np.float32)
    assert run([("x", small, 1)], [("y", small.copy(), 1)], 1024) is False           # under the threshold
    assert run([("x", x.astype(np.float64), 1)], [("y", y, 1)], N) is False          # not float32
    wide = np.zeros((N, 2), np.float32)
    assert run([("x", wide[:, 0], 1)], [("y", y, 1)], N) is False                    # not contiguous
    assert run([("x", x, 1)], [("y", y[: N // 2], 1)], N) is False                    # output too short
    ro = y.copy()
    ro.flags.writeable = False
    assert run([("x", x, 1)], [("y", ro, 1)], N) is False                            # read-only output
    both = np.zeros(2 * N, np.float32)
    assert run([("x", both[:N + 8], 1)], [("y", both[N:], 1)], N) is False           # output overlaps input
    assert run([("x", [0.0] * 8, 1)], [("y", y, 1)], N) is False                     # not a numpy array
    lt = fake_launch()
    lt.capturing = True
    assert _pipelined_on_host(lt, [("x", x, 1)], [("y", y, 1)], N, 1, never) is False  # under graph capture


@pytest.mark.usefixtures("pinned")
def test_a_qualifying_launch_goes_on_to_the_copy_streams():
    if torch.cuda.is_available():
        pytest.skip("checked on a machine without a GPU (the GPU tests run the path itself)")
    x, y = np.zeros(N, np.float32), np.zeros(N, np.float32)
    with pytest.raises(Exception):
        run([("x", x, 1)], [("y", y, 1)], N)
