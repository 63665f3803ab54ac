"""The reference's own launcher with the B200 branch applied (CPU, no GPU).

``piton_b200/integration/reference_launcher_b200.patch`` is the one change a
PIton maintainer makes: a ``device="b200"`` branch in ``Launcher.__call__``
(piton/runtime/launcher.py:238-244) that skips ``compile()`` and hands the
bound launch to ``run_on_b200``.  This test applies the patch to a temporary
copy of a reference checkout and launches the reference's own
``examples/kernels.py`` JITFunctions through it with ``run_on_b200`` replaced
by a recorder, so it checks, without a GPU, that dispatch reaches the B200
backend with exactly the arguments the reference's ``bind()`` produced and
that every such launch finds a B200 implementation in the registry.

The checkout is taken from the ``PITON_REFERENCE`` environment variable; the
test is skipped when it is unset.
"""

import os
import shutil
import subprocess
import sys
import textwrap

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PATCH = os.path.join(REPO, "piton_b200", "integration", "reference_launcher_b200.patch")
REF = os.environ.get("PITON_REFERENCE", "")

pytestmark = pytest.mark.skipif(not (REF and os.path.isfile(os.path.join(REF, "piton", "runtime", "launcher.py"))),
                                reason="PITON_REFERENCE (a reference checkout) is not set")

DRIVER = textwrap.dedent('''
    import json, sys
    import numpy as np
    sys.path.insert(0, sys.argv[1])                       # the patched reference copy
    sys.path.insert(1, sys.argv[1] + "/examples")
    sys.path.insert(2, sys.argv[2])                       # this repository (piton_b200)
    import piton.runtime.launcher as ref_launcher
    import piton_b200.runtime.cuda as b200
    from piton_b200.runtime.cuda import _REGISTRY

    def no_compile(*a, **k):
        raise AssertionError("compile() ran on the b200 branch")
    ref_launcher.compile = no_compile

    calls = []
    def recorder(jitfn, grid, constants, values, device=None, qpu=False):
        params = tuple(jitfn.arg_names)
        calls.append({"name": jitfn.__name__, "grid": list(grid), "constants": constants,
                      "values": sorted(values), "device": device, "qpu": qpu,
                      "registered": (jitfn.__name__, params) in _REGISTRY,
                      "same_arrays": all(values[k] is v for k, v in LAST.items())})
        return {"time_us": 0.0}
    b200.run_on_b200 = recorder

    import kernels as K
    n = 65537
    x, y, out = (np.zeros(n, np.float32) for _ in range(3))
    LAST = {"x_ptr": x, "y_ptr": y, "output_ptr": out}
    h = K.add_kernel[(257,)](x, y, out, n, BLOCK_SIZE=256, device="b200")
    assert h.last_stats == {"time_us": 0.0}, h.last_stats
    M = N = Kd = 128
    a, b, c = np.zeros((M, Kd), np.float32), np.zeros((Kd, N), np.float32), np.zeros((M, N), np.float32)
    LAST = {"a_ptr": a, "b_ptr": b, "c_ptr": c}
    K.matmul_kernel[lambda meta: (16 * 2,)](a, b, c, M, N, Kd, Kd, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64,
                                            BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200:1")
    sm_in, sm_out = np.zeros((4, 781), np.float32), np.zeros((4, 781), np.float32)
    LAST = {"output_ptr": sm_out, "input_ptr": sm_in}
    K.softmax_kernel[(4,)](sm_out, sm_in, 781, 781, 781, BLOCK_SIZE=1024, device="b200")
    # other devices still take the reference's own path: compile(), then its device check
    ref_launcher.compile = lambda *a, **k: type("StubCompiled", (), {})()
    try:
        K.add_kernel[(1,)](x, y, out, n, BLOCK_SIZE=256, device="b100")
        raise AssertionError("unknown device accepted")
    except ValueError:
        pass
    print(json.dumps(calls))
''')


def _patched_copy(tmp_path):
    dst = tmp_path / "ref"
    shutil.copytree(os.path.join(REF, "piton"), dst / "piton",
                    ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    shutil.copytree(os.path.join(REF, "examples"), dst / "examples",
                    ignore=shutil.ignore_patterns("__pycache__", "*.pyc", "data"))
    r = subprocess.run(["patch", "-p1", "--forward", "-i", PATCH], cwd=dst, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return dst


def test_patch_applies_and_dispatches_with_the_reference_binding(tmp_path):
    import json
    dst = _patched_copy(tmp_path)
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, "-c", DRIVER, str(dst), REPO], capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    calls = json.loads(r.stdout.strip().splitlines()[-1])
    assert [c["name"] for c in calls] == ["add_kernel", "matmul_kernel", "softmax_kernel"]
    add, mm, sm = calls
    assert add["grid"] == [257] and add["constants"] == {"BLOCK_SIZE": 256} and add["device"] is None
    assert add["values"] == ["n_elements", "output_ptr", "x_ptr", "y_ptr"]
    # the reference's bind(): ints equal to 1 become constants, the grid callable is evaluated
    assert mm["grid"] == [32] and mm["device"] == 1
    assert mm["constants"] == {"stride_ak": 1, "stride_bn": 1, "stride_cn": 1, "BLOCK_SIZE_M": 8,
                               "BLOCK_SIZE_N": 64, "BLOCK_SIZE_K": 8, "GROUP_SIZE_M": 8}
    assert sm["constants"] == {"BLOCK_SIZE": 1024}
    for c in calls:
        assert c["registered"], c["name"]          # the registry finds a B200 implementation
        assert c["same_arrays"], c["name"]         # the caller's arrays themselves, for copy-back
        assert c["qpu"] is False
