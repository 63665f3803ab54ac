"""AOT launcher emission (piton_b200.tools.compile), on the CPU: every operator's
emitted C compiles warning-free against include/piton_b200.h and links against
libpiton_b200.so; bad signatures are rejected as the reference's tool rejects
them (piton/tools/compile.py:55-169)."""

import os
import shutil
import subprocess
import sys

import pytest

from aot_cases import CASES
from piton_b200.tools import compile as aot

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KERNELS = os.path.join(ROOT, "piton_b200", "kernels.py")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(ROOT, "piton_b200")
CC = shutil.which("gcc") or shutil.which("cc")


@pytest.fixture(scope="module")
def emitted(tmp_path_factory):
    out = tmp_path_factory.mktemp("aot")
    for name, kern, sig, cons, opts in CASES:
        aot.compile_kernel(KERNELS, kern, sig, cons, name, str(out), **opts)
    return out


@pytest.mark.skipif(CC is None, reason="no C compiler")
def test_every_launcher_compiles_without_warnings(emitted):
    for name, *_ in CASES:
        r = subprocess.run([CC, "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", INCLUDE, "-c",
                            str(emitted / f"{name}.c"), "-o", str(emitted / f"{name}.o")],
                           capture_output=True, text=True)
        assert r.returncode == 0, f"{name}:\n{r.stderr}"


@pytest.mark.skipif(CC is None or not os.path.exists(os.path.join(LIBDIR, "libpiton_b200.so")),
                    reason="no C compiler or library not built")
def test_launchers_link_against_the_library(emitted):
    main = emitted / "main.c"
    lines = [f'#include "{n}.h"' for n, *_ in CASES] + ["typedef void (*fn_t)(void);", "int main(int argc, char **argv) {",
                                                        "    (void)argv;", "    fn_t fns[] = {"]
    lines += [f"        (fn_t){n}_launch, (fn_t){n}_launch_async," for n, *_ in CASES]
    lines += ["    };", "    return fns[argc % (sizeof fns / sizeof fns[0])] == 0;", "}"]
    main.write_text("\n".join(lines) + "\n")
    srcs = [str(main)] + [str(emitted / f"{n}.c") for n, *_ in CASES]
    exe = emitted / "main"
    r = subprocess.run([CC, "-std=c99", "-Wall", "-Werror", "-I", INCLUDE, "-I", str(emitted), *srcs, "-o", str(exe),
                        "-L", LIBDIR, "-lpiton_b200", f"-Wl,-rpath,{LIBDIR}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_header_keeps_the_reference_launch_interface(emitted):
    h = (emitted / "aot_matmul.h").read_text()
    assert "uint32_t aot_matmul_launch(const aot_matmul_args_t *args, unsigned gx, unsigned gy, unsigned gz);" in h
    # runtime arguments in parameter order; constants only in the comment
    body = h[h.index("typedef struct {"):h.index("} aot_matmul_args_t;")]
    names = [ln.split()[1].rstrip(";") for ln in body.splitlines()[1:]]
    assert names == ["a_ptr", "b_ptr", "c_ptr", "M", "N", "stride_am", "stride_bk", "stride_cm"]
    assert "K=512" in h
    c = (emitted / "aot_matmul.c").read_text()
    assert "a.K = 512;" in c and "a.grid_x = gx;" in c and "piton_b200_matmul_workspace_size" in c
    assert "PITON_B200_QPU_ROUNDING" in (emitted / "aot_add_qpu.c").read_text()
    assert "a.is_signed = 0;" in (emitted / "aot_udiv.c").read_text()
    assert "a.op = 4 + ((4) < 0 ? 0 : (4) > 5 ? 5 : (4));" in (emitted / "aot_exp.c").read_text()


def test_ctypes_mirror_matches_the_emitted_struct():
    import ctypes as C
    params = aot.kernel_params(aot.load_kernel(KERNELS, "attn_fwd_kernel"))
    T = aot.ctypes_args(params, CASES[7][2])
    assert [f[0] for f in T._fields_] == ["Q", "K", "V", "Out", "sm_scale", "stride_qh", "stride_kh", "stride_vh",
                                          "stride_oh"]
    assert C.sizeof(T) == 4 * 8 + 4 + 4 * 4 + 4   # trailing padding to 8


@pytest.mark.parametrize("kern,sig,cons,opts,msg", [
    ("add_kernel", "x_ptr=*fp32,y_ptr=*fp32,output_ptr=*fp32", "BLOCK_SIZE=256", {}, "neither"),
    ("add_kernel", "x_ptr=*fp32,y_ptr=*fp32,output_ptr=*fp32,n_elements=i32", "BLOCK_SIZE=256,n_elements=4", {},
     "both"),
    ("add_kernel", "x_ptr=*fp32,y_ptr=*fp32,output_ptr=*fp32,n_elements=i32,bogus=i32", "BLOCK_SIZE=256", {},
     "not parameters"),
    ("add_kernel", "x_ptr=*fp32,y_ptr=*fp32,n_elements=i32", "BLOCK_SIZE=256,output_ptr=0", {}, "pointer"),
    ("add_kernel", "x_ptr=*fp32,y_ptr=*fp32,output_ptr=*fp32,n_elements=f16", "BLOCK_SIZE=256", {}, "type"),
    ("layernorm_kernel", "x_ptr=*fp32,out_ptr=*fp32,n=i32,eps=fp32", "BLOCK=128", {"qpu_rounding": True},
     "qpu-rounding"),
    ("add_kernel", "x_ptr=*fp32,y_ptr=*fp32,output_ptr=*fp32,n_elements=i32", "BLOCK_SIZE=256",
     {"force_simt": True}, "force-simt"),
    ("idiv_kernel", "x_ptr=*i32,y_ptr=*u32,q_ptr=*i32,r_ptr=*i32,n=i32", "BLOCK=256", {}, "must all be"),
    ("no_such_kernel", "", "", {}, "no kernel"),
])
def test_bad_signatures_are_rejected(tmp_path, kern, sig, cons, opts, msg):
    with pytest.raises(aot.CompileError, match=msg):
        aot.compile_kernel(KERNELS, kern, sig, cons, "x", str(tmp_path), **opts)


def test_command_line(tmp_path):
    name, kern, sig, cons, _ = CASES[3]
    r = subprocess.run([sys.executable, "-m", "piton_b200.tools.compile", KERNELS, "--kernel-name", kern,
                        "--signature", sig, "--constants", cons, "--out-name", "mm", "-o", str(tmp_path)],
                       capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    assert (tmp_path / "mm.h").exists() and (tmp_path / "mm.c").exists()
    r = subprocess.run([sys.executable, "-m", "piton_b200.tools.compile", KERNELS, "--kernel-name", kern,
                        "--signature", sig, "-o", str(tmp_path)], capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 2 and "neither" in r.stderr
