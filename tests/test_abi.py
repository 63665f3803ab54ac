"""The C-ABI boundary without a GPU: the library loads, exports every function
include/piton_b200.h declares, and the ctypes mirrors of the argument structs
have the C layout (size and every field offset, checked by compiling a small
C program against the header)."""

import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from conftest import REPO
from piton_b200.runtime.cuda import _lib

HEADER = os.path.join(REPO, "include", "piton_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"PITON_B200_API\s+[\w\s\*]+?\b(piton_b200_\w+)\s*\(", text)))


def declared_structs():
    text = open(HEADER).read()
    out = {}
    for body, name in re.findall(r"typedef struct \{(.*?)\}\s*(\w+);", text, flags=re.S):
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            m = re.match(r"([\w\s]+?)\s+([\w\s,\[\]]+)$", decl)
            assert m, decl
            fields += [re.sub(r"\[\d+\]", "", f).strip() for f in m.group(2).split(",")]
        out[name] = fields
    return out


def test_library_loads_and_reports_its_abi():
    lib = _lib.lib()
    assert lib.piton_b200_abi_version() == 1
    assert isinstance(lib.piton_b200_launch_count(), int)


def test_every_declared_function_is_exported_and_bound():
    names = declared_functions()
    assert len(names) >= 20
    lib = C.CDLL(_lib.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    assert set(names) == set(_lib.PROTOTYPES), "ctypes prototypes and the header disagree"


def test_struct_layouts_match_the_header():
    structs = declared_structs()
    assert set(structs) == set(_lib.STRUCTS)
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "piton_b200.h"', "int main(void) {"]
    for name, fields in structs.items():
        lines.append(f'printf("{name} size %zu\\n", sizeof({name}));')
        for f in fields:
            lines.append(f'printf("{name} {f} %zu\\n", offsetof({name}, {f}));')
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "layout.c"), os.path.join(d, "layout")
        with open(src, "w") as fh:
            fh.write("\n".join(lines))
        subprocess.run(["gcc", "-std=c11", "-I", os.path.dirname(HEADER), src, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    c_layout = {}
    for line in filter(None, out):
        name, field, val = line.split()
        c_layout[(name, field)] = int(val)
    for name, cls in _lib.STRUCTS.items():
        assert C.sizeof(cls) == c_layout[(name, "size")], name
        py_fields = [f for f, _ in cls._fields_]
        c_fields = structs[name]
        assert len(py_fields) == len(c_fields), name
        for pf, cf in zip(py_fields, c_fields):
            assert getattr(cls, pf).offset == c_layout[(name, cf)], (name, pf, cf)


def test_argument_errors_need_no_gpu():
    lib = _lib.lib()
    # a NULL args pointer and bad shapes are rejected before any CUDA call
    assert lib.piton_b200_add_f32(None, None) == _lib.EINVAL
    a = _lib.AddArgs(0, 0, 0, -5, 256, 1, 0, 0)
    assert lib.piton_b200_add_f32(C.byref(a), None) == _lib.EINVAL
    assert b"n_elements" in lib.piton_b200_last_error()
    s = _lib.SoftmaxArgs(0, 0, 4, 4, 4, 4, 2, 7, 0)
    assert lib.piton_b200_softmax_f32(C.byref(s), None) == _lib.EINVAL
    m = _lib.MatmulArgs(0, 0, 0, 4, 4, 4, 4, 1, 4, 1, 4, 1, 0, 64, 8, 8, 1, 0, 0, 0, 0)
    assert lib.piton_b200_matmul_f32(C.byref(m), None) == _lib.EINVAL
    # zero-size launches are no-ops
    z = _lib.AddArgs(0, 0, 0, 0, 256, 0, 0, 0)
    assert lib.piton_b200_add_f32(C.byref(z), None) == _lib.OK


def _attention_args(heads=2, n=128, stride_om=64):
    sd = n * 64
    return _lib.AttentionArgs(0, 0, 0, 0, 0.125, sd, 64, sd, 64, 1, sd, 64, sd, stride_om, n, 64, 64, 64, -(-n // 64),
                              heads, 1, 1, 0, 0, 0, 0)


def test_attention_allgather_argument_errors_need_no_gpu():
    lib = _lib.lib()
    f = lib.piton_b200_attention_allgather_f32
    g = _lib.AllgatherArgs()
    g.peer_c[0], g.peer_c[1] = 4096, 8192
    g.world, g.rank = 2, 0
    a = _attention_args()
    assert f(C.byref(a), None, None) == _lib.EINVAL
    g.world = 0
    assert f(C.byref(a), C.byref(g), None) == _lib.EINVAL
    g.world, g.rank = 2, 2
    assert f(C.byref(a), C.byref(g), None) == _lib.EINVAL
    g.rank, g.row_offset = 1, -1
    assert f(C.byref(a), C.byref(g), None) == _lib.EINVAL
    g.row_offset = 0
    g.multicast_c = 4096                       # the attention all-gather has no multicast form
    assert f(C.byref(a), C.byref(g), None) == _lib.ENOTSUP
    g.multicast_c = 0
    g.peer_c[1] = 8200                         # not 16-byte aligned
    assert f(C.byref(a), C.byref(g), None) == _lib.EINVAL
    g.peer_c[1] = 8192
    odd = _attention_args(stride_om=66)         # rows must stay 16-byte aligned on every rank
    assert f(C.byref(odd), C.byref(g), None) == _lib.EINVAL
    none = _attention_args(heads=0)            # no heads: nothing to do
    assert f(C.byref(none), C.byref(g), None) == _lib.OK


def test_check_maps_status_codes():
    with pytest.raises(ValueError):
        _lib.check(_lib.lib().piton_b200_add_f32(None, None))
    _lib.check(_lib.OK)
