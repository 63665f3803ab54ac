"""Ahead-of-time launchers for the B200 backend, the counterpart of the
reference's ``python -m piton.tools.compile`` (piton/tools/compile.py:1-13, 55-169).

    python -m piton_b200.tools.compile piton_b200/kernels.py --kernel-name matmul_kernel \\
        --signature "a_ptr=*fp32,b_ptr=*fp32,c_ptr=*fp32,M=i32,N=i32,stride_am=i32,stride_bk=i32,stride_cm=i32" \\
        --constants "K=512,stride_ak=1,stride_bn=1,stride_cn=1,BLOCK_SIZE_M=8,BLOCK_SIZE_N=64,BLOCK_SIZE_K=4,GROUP_SIZE_M=4" \\
        --out-name matmul -o build/

writes build/matmul.h and build/matmul.c.  On the reference those files carry
the kernel's QPU machine code and a bare-metal launcher; on the B200 the
machine code already lives in libpiton_b200.so (hand-written sm_100a kernels,
one per operator), so the emitted C is the launcher alone: it keeps the
reference's interface

    matmul_args_t args = { .a_ptr = A, ..., .M = 512, ... };
    uint32_t usec = matmul_launch(&args, grid_x, 1, 1);

(pointer arguments are device addresses instead of bus addresses) and maps the
kernel's runtime arguments plus the constants baked in at compile time onto
the operator's ``piton_b200_*`` entry point.  ``<sym>_launch`` runs on the
legacy default stream and returns the elapsed microseconds, or UINT32_MAX
when the call failed (``piton_b200_last_error()`` says why) or did not finish
within 20 s (the reference's launch timeout, pi/runtime/piton_rt.c:150-189).
``<sym>_launch_async`` enqueues on a caller's stream and returns the status.

Build a program with ``cc main.c matmul.c -Iinclude -Lpiton_b200 -lpiton_b200``.
The emitted C uses only libpiton_b200.so and libc.
"""

from __future__ import annotations

import argparse
import importlib
import importlib.util
import inspect
import os
import sys

C_TYPES = {"*fp32": "uint64_t", "*i32": "uint64_t", "*u32": "uint64_t", "*u8": "uint64_t",
           "i32": "int32_t", "u32": "uint32_t", "i64": "int64_t", "fp32": "float", "fp64": "double",
           "i1": "int32_t"}

# operators that accept PITON_B200_QPU_ROUNDING / PITON_B200_FORCE_SIMT
QPU_OK = {"add_kernel", "softmax_kernel", "matmul_kernel", "dense_layer_kernel", "attn_fwd_kernel", "copy_kernel",
          "mul_kernel", "fma_kernel", "scaled_relu_kernel"}
SIMT_OK = {"matmul_kernel", "dense_layer_kernel", "attn_fwd_kernel"}


class CompileError(ValueError):
    pass


def _parse_kv(text: str) -> dict:
    """``name=value,...``; values are ints (any base), floats, True/False, or type names."""
    out = {}
    for item in filter(None, (t.strip() for t in (text or "").split(","))):
        if "=" not in item:
            raise CompileError(f"expected name=value, got {item!r}")
        k, v = (s.strip() for s in item.split("=", 1))
        if v in ("True", "False"):
            out[k] = v == "True"
            continue
        try:
            out[k] = int(v, 0)
        except ValueError:
            try:
                out[k] = float(v)
            except ValueError:
                out[k] = v
    return out


def load_kernel(path: str, name: str):
    """The ``@jit`` function `name` from a Python file or an importable module."""
    if path.endswith(".py") and os.path.exists(os.path.join(os.path.dirname(os.path.abspath(path)), "__init__.py")):
        # a module inside a package (relative imports): import it by its dotted name
        parts = [os.path.splitext(os.path.basename(path))[0]]
        d = os.path.dirname(os.path.abspath(path))
        while os.path.exists(os.path.join(d, "__init__.py")):
            parts.insert(0, os.path.basename(d))
            d = os.path.dirname(d)
        if d not in sys.path:
            sys.path.insert(0, d)
        mod = importlib.import_module(".".join(parts))
    elif path.endswith(".py") or os.path.sep in path:
        modname = os.path.splitext(os.path.basename(path))[0]
        spec = importlib.util.spec_from_file_location(modname, path)
        if spec is None:
            raise CompileError(f"cannot load {path}")
        mod = importlib.util.module_from_spec(spec)
        sys.path.insert(0, os.path.dirname(os.path.abspath(path)))
        try:
            spec.loader.exec_module(mod)
        finally:
            sys.path.pop(0)
    else:
        mod = importlib.import_module(path)
    if not hasattr(mod, name):
        raise CompileError(f"{path} has no kernel {name!r}")
    return getattr(mod, name)


def kernel_params(kernel) -> list:
    names = getattr(kernel, "arg_names", None)
    if names:
        return list(names)
    fn = getattr(kernel, "fn", kernel)
    return list(inspect.signature(fn).parameters)


class Emitter:
    """Resolves kernel parameters to C expressions: runtime arguments read
    ``args->name``; constants become literals."""

    def __init__(self, name, params, signature, constants):
        self.name = name
        self.params = params
        self.signature = signature
        self.constants = constants
        missing = [p for p in params if p not in signature and p not in constants]
        both = [p for p in params if p in signature and p in constants]
        unknown = [k for k in list(signature) + list(constants) if k not in params]
        if missing:
            raise CompileError(f"{name}: parameters {missing} are in neither --signature nor --constants")
        if both:
            raise CompileError(f"{name}: parameters {both} are in both --signature and --constants")
        if unknown:
            raise CompileError(f"{name}: {unknown} are not parameters of the kernel {params}")
        for k, t in signature.items():
            if t not in C_TYPES:
                raise CompileError(f"{name}: argument {k} has type {t!r}; known: {sorted(C_TYPES)}")

    def v(self, p: str) -> str:
        if p in self.signature:
            return f"args->{p}"
        c = self.constants[p]
        if isinstance(c, bool):
            return "1" if c else "0"
        if isinstance(c, int):
            return f"{c}LL" if abs(c) >= 1 << 31 else str(c)
        if isinstance(c, float):
            return repr(c)
        raise CompileError(f"{self.name}: constant {p}={c!r} is not a number")

    def ptr(self, p: str) -> str:
        t = self.signature.get(p)
        if t is None or not t.startswith("*"):
            raise CompileError(f"{self.name}: {p} is a pointer and must be a runtime argument of a pointer type")
        return f"args->{p}"

    def ptr_type(self, p: str) -> str:
        self.ptr(p)
        return self.signature[p]


def _min(a, b):
    return f"(({a}) < ({b}) ? ({a}) : ({b}))"


def _op_add(e):
    return "piton_add_args", "piton_b200_add_f32", None, [
        ("x", e.ptr("x_ptr")), ("y", e.ptr("y_ptr")), ("out", e.ptr("output_ptr")),
        ("n_elements", e.v("n_elements")), ("block_size", e.v("BLOCK_SIZE")), ("grid_x", "gx")]


def _op_softmax(e):
    return "piton_softmax_args", "piton_b200_softmax_f32", None, [
        ("out", e.ptr("output_ptr")), ("in", e.ptr("input_ptr")), ("in_row_stride", e.v("input_row_stride")),
        ("out_row_stride", e.v("output_row_stride")), ("n_cols", e.v("n_cols")),
        ("block_size", e.v("BLOCK_SIZE")), ("grid_x", "gx")]


def _op_matmul(e):
    f = [("a", e.ptr("a_ptr")), ("b", e.ptr("b_ptr")), ("c", e.ptr("c_ptr"))]
    f += [(k, e.v(k)) for k in ("M", "N", "K", "stride_am", "stride_ak", "stride_bk", "stride_bn", "stride_cm",
                                 "stride_cn")]
    f += [("block_m", e.v("BLOCK_SIZE_M")), ("block_n", e.v("BLOCK_SIZE_N")), ("block_k", e.v("BLOCK_SIZE_K")),
          ("group_m", e.v("GROUP_SIZE_M")), ("grid_x", "gx")]
    return "piton_matmul_args", "piton_b200_matmul_f32", "piton_b200_matmul_workspace_size", f


def _op_dense(e):
    f = [("x", e.ptr("x_ptr")), ("w", e.ptr("w_ptr")), ("bias", f"({e.v('ADD_BIAS')}) ? {e.ptr('bias_ptr')} : 0"),
         ("y", e.ptr("y_ptr")), ("M", e.v("M")), ("N", e.v("N")), ("K", e.v("K")),
         ("block_m", e.v("BLOCK_SIZE_M")), ("block_n", e.v("BLOCK_SIZE_N")), ("block_k", e.v("BLOCK_SIZE_K")),
         ("group_m", e.v("GROUP_SIZE_M")), ("grid_x", "gx"),
         ("add_bias", f"({e.v('ADD_BIAS')}) != 0"), ("relu", f"({e.v('RELU')}) != 0")]
    return "piton_dense_args", "piton_b200_dense_f32", None, f


def _op_attention(e):
    f = [("q", e.ptr("Q")), ("k", e.ptr("K")), ("v", e.ptr("V")), ("out", e.ptr("Out")),
         ("sm_scale", f"(double)({e.v('sm_scale')})")]
    f += [(k, e.v(k)) for k in ("stride_qh", "stride_qm", "stride_kh", "stride_kn", "stride_kk", "stride_vh",
                                 "stride_vn", "stride_oh", "stride_om")]
    f += [("n_ctx", e.v("N_CTX")), ("head_dim", e.v("HEAD_DIM")), ("block_m", e.v("BLOCK_M")),
          ("block_n", e.v("BLOCK_N")), ("grid_x", "gx"), ("grid_y", "gy"),
          ("causal", f"({e.v('CAUSAL')}) != 0"), ("even_n", f"({e.v('EVEN_N')}) != 0")]
    return "piton_attention_args", "piton_b200_attention_f32", "piton_b200_attention_workspace_size", f


def _op_layernorm(e):
    n, blk = e.v("n"), e.v("BLOCK")
    return "piton_layernorm_args", "piton_b200_layernorm_f32", None, [
        ("x", e.ptr("x_ptr")), ("y", e.ptr("out_ptr")), ("rows", "gx"),
        ("n_cols", f"({n}) < 0 ? 0 : {_min(n, blk)}"), ("x_row_stride", blk), ("y_row_stride", blk),
        ("eps", f"(double)({e.v('eps')})")]


def _elementwise(op, x="x_ptr", y=None, out="out_ptr", alpha=None):
    def f(e):
        fields = [("x", e.ptr(x)), ("y", e.ptr(y) if y else "0"), ("out", e.ptr(out)),
                  ("n_elements", e.v("n")), ("block_size", e.v("BLOCK")), ("grid_x", "gx"),
                  ("alpha", f"(double)({e.v(alpha)})" if alpha else "0.0"),
                  ("op", op if isinstance(op, str) else str(op))]
        return "piton_elementwise_args", "piton_b200_elementwise_f32", None, fields
    return f


def _op_sfu(e):
    op = e.v("OP")
    return _elementwise(f"4 + (({op}) < 0 ? 0 : ({op}) > 5 ? 5 : ({op}))")(e)


def _op_idiv(e):
    types = {e.ptr_type(p) for p in ("x_ptr", "y_ptr", "q_ptr", "r_ptr")}
    if not types <= {"*i32", "*u32"} or len(types) != 1:
        raise CompileError("idiv_kernel: x_ptr, y_ptr, q_ptr, r_ptr must all be *i32 or all *u32")
    return "piton_idiv_args", "piton_b200_idiv_i32", None, [
        ("x", e.ptr("x_ptr")), ("y", e.ptr("y_ptr")), ("q", e.ptr("q_ptr")), ("r", e.ptr("r_ptr")),
        ("n_elements", e.v("n")), ("block_size", e.v("BLOCK")), ("grid_x", "gx"),
        ("is_signed", "1" if types == {"*i32"} else "0")]


def _row_reduce(reduce):
    def f(e):
        return "piton_row_reduce_args", "piton_b200_row_reduce_f32", None, [
            ("x", e.ptr("x_ptr")), ("out", e.ptr("out_ptr")), ("n_cols", e.v("n_cols")), ("stride", e.v("stride")),
            ("block_m", e.v("BLOCK_M")), ("block_n", e.v("BLOCK_N")), ("grid_x", "gx"), ("reduce", str(reduce))]
    return f


def _op_transpose(e):
    return "piton_transpose_args", "piton_b200_transpose_f32", None, [
        ("x", e.ptr("x_ptr")), ("out", e.ptr("out_ptr")), ("n_rows", e.v("n_rows")), ("n_cols", e.v("n_cols")),
        ("stride_x", e.v("stride_x")), ("stride_out", e.v("stride_out")), ("block_m", e.v("BLOCK_M")),
        ("block_n", e.v("BLOCK_N")), ("grid_x", "gx")]


def _life(mode, cols, br, bc):
    def f(e):
        return "piton_life_args", "piton_b200_life_step", None, [
            ("src", e.ptr("src_ptr")), ("dst", e.ptr("dst_ptr")), ("n_rows", e.v("n_rows")), ("n_cols", e.v(cols)),
            ("stride", e.v("stride")), ("block_r", e.v(br)), ("block_c", e.v(bc)), ("grid_x", "gx"),
            ("grid_y", "gy"), ("mode", str(mode))]
    return f


# kernel name -> field mapping; the parameter lists are those of piton_b200/kernels.py
OPERATORS = {
    "add_kernel": _op_add,
    "softmax_kernel": _op_softmax,
    "matmul_kernel": _op_matmul,
    "dense_layer_kernel": _op_dense,
    "attn_fwd_kernel": _op_attention,
    "layernorm_kernel": _op_layernorm,
    "copy_kernel": _elementwise(0),
    "mul_kernel": _elementwise(1, y="y_ptr"),
    "fma_kernel": _elementwise(2, y="y_ptr", alpha="alpha"),
    "scaled_relu_kernel": _elementwise(3, alpha="alpha"),
    "sfu_kernel": _op_sfu,
    "log_kernel": _elementwise(10),
    "sigmoid_kernel": _elementwise(11),
    "idiv_kernel": _op_idiv,
    "row_sum_kernel": _row_reduce(0),
    "row_max_kernel": _row_reduce(1),
    "transpose_kernel": _op_transpose,
    "life_kernel": _life(0, "n_cols", "BLOCK_R", "BLOCK_C"),
    "life_rows_kernel": _life(1, "n_cols", "ROWS", "BLOCK"),
    "life_bits_kernel": _life(2, "n_words", "ROWS", "BLOCK"),
}


def emit_c(name: str, params: list, signature: dict, constants: dict, out_name: str,
           qpu_rounding: bool = False, force_simt: bool = False) -> tuple:
    """(header, source) of the AOT launcher for kernel `name`."""
    if name not in OPERATORS:
        raise CompileError(f"{name} has no B200 implementation (known: {sorted(OPERATORS)})")
    if qpu_rounding and name not in QPU_OK:
        raise CompileError(f"{name}: --qpu-rounding applies to {sorted(QPU_OK)}")
    if force_simt and name not in SIMT_OK:
        raise CompileError(f"{name}: --force-simt applies to {sorted(SIMT_OK)}")
    if not out_name.isidentifier():
        raise CompileError(f"--out-name {out_name!r} is not a C identifier")
    e = Emitter(name, params, signature, constants)
    struct, entry, ws_fn, fields = OPERATORS[name](e)
    flags = " | ".join(f for f, on in (("PITON_B200_QPU_ROUNDING", qpu_rounding),
                                        ("PITON_B200_FORCE_SIMT", force_simt)) if on) or "0"
    sym, SYM = out_name, out_name.upper()
    args = [(n, signature[n]) for n in params if n in signature]

    h = [f"// Generated by piton_b200.tools.compile from kernel `{name}` (B200, sm_100a; libpiton_b200.so).",
         f"// constants: {', '.join(f'{k}={v}' for k, v in constants.items()) or '(none)'}",
         f"// entry point: {entry}" + (f", flags {flags}" if flags != "0" else ""),
         f"#ifndef {SYM}_H", f"#define {SYM}_H", "",
         "#include <stdint.h>", '#include "piton_b200.h"', "",
         "#ifdef __cplusplus", 'extern "C" {', "#endif", "",
         "// Pointer arguments are device addresses (piton_b200_malloc, cudaMalloc, a tensor's data_ptr()).",
         "typedef struct {"]
    h += [f"    {C_TYPES[t]} {n};   // {t}" for n, t in args] or ["    int32_t _unused;"]
    h += [f"}} {sym}_args_t;", "",
          "// Launch gx*gy*gz programs on the legacy default stream and wait for them (20 s at most).",
          "// Returns the elapsed microseconds, or UINT32_MAX on failure (piton_b200_last_error()).",
          f"uint32_t {sym}_launch(const {sym}_args_t *args, unsigned gx, unsigned gy, unsigned gz);", "",
          "// Enqueue the launch on `stream` (a cudaStream_t; NULL = legacy default) without waiting.",
          "// Returns PITON_B200_OK or a negative PITON_B200_E* status.",
          f"int {sym}_launch_async(const {sym}_args_t *args, unsigned gx, unsigned gy, unsigned gz, void *stream);",
          "", "#ifdef __cplusplus", "}", "#endif", "#endif", ""]

    c = [f"// Generated by piton_b200.tools.compile from kernel `{name}`.",
         "#define _POSIX_C_SOURCE 199309L", "#include <time.h>", f'#include "{sym}.h"', ""]
    if ws_fn:
        c += ["// Tensor-core scratch, grown on demand and kept, one per device (as the reference's launcher",
              "// keeps its code and uniform buffers).  Launchers of this kernel on one device must not overlap.",
              "#define WS_DEVICES 64",
              "static uint64_t ws_ptr[WS_DEVICES];", "static size_t ws_bytes[WS_DEVICES];", ""]
    c += [f"int {sym}_launch_async(const {sym}_args_t *args, unsigned gx, unsigned gy, unsigned gz, void *stream) {{",
          "    (void)args; (void)gx; (void)gy; (void)gz;",
          f"    {struct} a = {{0}};"]
    c += [f"    a.{fld} = {expr};" for fld, expr in fields]
    c += [f"    a.flags = {flags};"]
    if ws_fn:
        c += ["    int dev = 0;",
              "    int rc = piton_b200_get_device(&dev);",
              "    if (rc != PITON_B200_OK) return rc;",
              "    if (dev < 0 || dev >= WS_DEVICES) return PITON_B200_EINVAL;",
              f"    size_t need = {ws_fn}(&a);",
              "    if (need > ws_bytes[dev]) {",
              "        if (ws_ptr[dev]) piton_b200_free(ws_ptr[dev]);",
              "        ws_ptr[dev] = 0;",
              "        ws_bytes[dev] = 0;",
              "        rc = piton_b200_malloc(&ws_ptr[dev], need);",
              "        if (rc != PITON_B200_OK) return rc;",
              "        ws_bytes[dev] = need;",
              "    }",
              "    a.workspace = ws_ptr[dev];",
              "    a.workspace_bytes = ws_bytes[dev];"]
    c += [f"    return {entry}(&a, stream);", "}", "",
          f"uint32_t {sym}_launch(const {sym}_args_t *args, unsigned gx, unsigned gy, unsigned gz) {{",
          "    struct timespec t0, t1;",
          "    clock_gettime(CLOCK_MONOTONIC, &t0);",
          f"    if ({sym}_launch_async(args, gx, gy, gz, 0) != PITON_B200_OK) return UINT32_MAX;",
          "    if (piton_b200_stream_wait(0, 20.0) != PITON_B200_OK) return UINT32_MAX;",
          "    clock_gettime(CLOCK_MONOTONIC, &t1);",
          "    int64_t us = (int64_t)(t1.tv_sec - t0.tv_sec) * 1000000 + (t1.tv_nsec - t0.tv_nsec) / 1000;",
          "    return us >= (int64_t)UINT32_MAX ? UINT32_MAX - 1u : (uint32_t)us;", "}", ""]
    return "\n".join(h), "\n".join(c)


def ctypes_args(params: list, signature) -> type:
    """A ctypes Structure laid out like the emitted ``<sym>_args_t``."""
    import ctypes as C
    sig = _parse_kv(signature) if isinstance(signature, str) else dict(signature)
    ct = {"uint64_t": C.c_uint64, "int32_t": C.c_int32, "uint32_t": C.c_uint32, "int64_t": C.c_int64,
          "float": C.c_float, "double": C.c_double}
    fields = [(n, ct[C_TYPES[sig[n]]]) for n in params if n in sig] or [("_unused", C.c_int32)]
    return type("args_t", (C.Structure,), {"_fields_": fields})


def compile_kernel(path, kernel_name, signature="", constants="", out_name=None, out_dir=".",
                   qpu_rounding=False, force_simt=False):
    """Write <out_dir>/<out_name>.h and .c; returns their paths."""
    kernel = load_kernel(path, kernel_name)
    sig = _parse_kv(signature) if isinstance(signature, str) else dict(signature)
    cons = _parse_kv(constants) if isinstance(constants, str) else dict(constants)
    name = out_name or kernel_name
    h, c = emit_c(kernel_name, kernel_params(kernel), sig, cons, name, qpu_rounding, force_simt)
    os.makedirs(out_dir, exist_ok=True)
    ph, pc = os.path.join(out_dir, name + ".h"), os.path.join(out_dir, name + ".c")
    with open(ph, "w") as f:
        f.write(h)
    with open(pc, "w") as f:
        f.write(c)
    return ph, pc


def main(argv=None):
    ap = argparse.ArgumentParser(description="Emit a C launcher for a PIton kernel on the B200 backend")
    ap.add_argument("path", help="python file (or module) containing the @jit kernel")
    ap.add_argument("--kernel-name", "-n", required=True)
    ap.add_argument("--signature", "-s", default="", help="name=type,... for runtime arguments")
    ap.add_argument("--constants", "-c", default="", help="name=value,... constexpr / specialised args")
    ap.add_argument("--out-name", default=None)
    ap.add_argument("--qpu-rounding", action="store_true", help="reproduce the QPU's float rounding bit for bit")
    ap.add_argument("--force-simt", action="store_true", help="take the CUDA-core path where tensor cores apply")
    ap.add_argument("-o", "--out-dir", default=".")
    args = ap.parse_args(argv)
    try:
        ph, pc = compile_kernel(args.path, args.kernel_name, args.signature, args.constants, args.out_name,
                                args.out_dir, args.qpu_rounding, args.force_simt)
    except CompileError as e:
        ap.exit(2, f"error: {e}\n")
    print(f"{args.kernel_name}: wrote {ph} and {pc}")


if __name__ == "__main__":
    main()
