"""The ``device="b200"`` backend: operator registry and argument marshalling.

``run_on_b200`` is what ``Launcher.__call__`` calls for a B200 launch (the
counterpart of the reference's ``run_emulator``, piton/runtime/launcher.py:168-214):

1. the launched kernel is looked up in the registry by its name and parameter
   list (the reference's ``JITFunction`` objects match too);
2. pointer arguments become device pointers: CUDA torch tensors are used in
   place; numpy arrays are copied to device buffers and, after the launch,
   **every array is copied back**, as the emulator path does
   (launcher.py:209-211), so in-place outputs behave the same;
3. the accessed extent of every buffer is checked against its size before
   anything launches (the kernels trust their pointers);
4. one ``extern "C"`` entry point of libpiton_b200.so runs on the current
   torch stream; its status code becomes a Python exception.

A kernel (or constexpr combination) without a B200 implementation raises
``NotImplementedError``; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import math
import os

import numpy as np

from ..launcher import offset_ptr, _is_torch_tensor
from . import _lib
from ._lib import check, lib

_REGISTRY = {}
_WORKSPACE = {}


def register(name: str, params: tuple):
    def deco(fn):
        _REGISTRY[(name, tuple(params))] = fn
        return fn
    return deco


def registered():
    return sorted(_REGISTRY)


def _torch():
    import torch
    return torch


class Buffer:
    """A pointer argument resolved to a device address.

    ``addr`` is the address the kernel indexes from; ``lo``/``hi`` bound the
    element indices (relative to ``addr``) that lie inside the allocation.
    numpy arrays are copied to a device buffer on the launch's stream
    (asynchronously from page-locked memory); ``copy_back`` copies the device
    buffer into the array again."""

    def __init__(self, name, value, device, stream, overwrite=False):
        torch = _torch()
        self.name = name
        off = 0
        base = value
        if isinstance(value, offset_ptr):
            base, off = value.base, value.elements
        self.host = None
        self.h2d_bytes = 0
        if isinstance(base, np.ndarray):
            self.host = base
            host_t = torch.from_numpy(np.ascontiguousarray(base).reshape(-1))
            self.pinned = bool(host_t.is_pinned())
            self.tensor = torch.empty(host_t.shape, dtype=host_t.dtype, device=device)
            if not overwrite:   # an output the launch writes in full needs no copy in
                with torch.cuda.stream(stream):
                    self.tensor.copy_(host_t, non_blocking=self.pinned)
                self.h2d_bytes = host_t.numel() * host_t.element_size()
        elif _is_torch_tensor(base):
            if base.device.type != "cuda":
                raise TypeError(f"argument {name}: tensor on {base.device}, expected a CUDA tensor or numpy array")
            self.tensor = base
        else:
            raise TypeError(f"argument {name}: expected an array, got {type(base).__name__}")
        t = self.tensor
        self.itemsize = t.element_size()
        storage_elems = t.untyped_storage().nbytes() // self.itemsize
        start = t.storage_offset() if self.host is None else 0
        self.addr = t.data_ptr() + off * self.itemsize
        self.lo = -(start + off)
        self.hi = storage_elems - start - off - 1

    def require(self, lo: int, hi: int):
        """Every index in [lo, hi] (relative to addr) must be inside the buffer."""
        if hi < lo:
            return
        if lo < self.lo or hi > self.hi:
            raise ValueError(f"argument {self.name}: the launch reads/writes elements [{lo}, {hi}] "
                             f"but the buffer holds [{self.lo}, {self.hi}]")

    def copy_back(self, stream):
        """Enqueue the device-to-host copy; returns its byte count."""
        if self.host is None:
            return 0
        torch = _torch()
        if self.host.flags.c_contiguous:
            dst = torch.from_numpy(self.host.reshape(-1))
            with torch.cuda.stream(stream):
                dst.copy_(self.tensor, non_blocking=self.pinned)
        else:
            self.host[...] = self.tensor.cpu().numpy().reshape(self.host.shape)
        return self.tensor.numel() * self.itemsize


def extent(*dims):
    """(min, max) of sum(i_k * stride_k) over 0 <= i_k < n_k; dims = (n, stride) pairs."""
    lo = hi = 0
    for n, s in dims:
        if n <= 0:
            return 0, -1
        lo += min(0, (n - 1) * s)
        hi += max(0, (n - 1) * s)
    return lo, hi


class Launch:
    """State of one B200 launch: marshalled buffers, the stream, the flags."""

    def __init__(self, values, constants, device, qpu):
        self.args = dict(constants)
        self.args.update(values)
        self.device = device
        self.qpu = qpu
        self.buffers = {}
        self.written = set()
        torch = _torch()
        self.stream = torch.cuda.current_stream(device)
        self.stream_ptr = C.c_void_p(self.stream.cuda_stream)
        # under CUDA-graph capture the launch is recorded, not run: no host copies, no
        # timing events, no synchronisation (torch.cuda.graph / CUDAGraph.capture_begin)
        self.capturing = torch.cuda.is_current_stream_capturing()
        self.ev0 = None if self.capturing else torch.cuda.Event(enable_timing=True)
        self.ev1 = None if self.capturing else torch.cuda.Event(enable_timing=True)
        self.called = False
        self.launches = 0                    # entry-point calls (several on the pipelined host-buffer paths)
        self.host_h2d = self.host_d2h = 0   # bytes an entry point copied itself (host-buffer paths)

    def call(self, fname: str, args, what: str):
        """Run one C-ABI entry point on the launch's stream, timed with CUDA events."""
        f = getattr(lib(), fname)
        if self.ev0 is not None:
            self.ev0.record(self.stream)
        rc = f(C.byref(args), self.stream_ptr)
        if self.ev1 is not None:
            self.ev1.record(self.stream)
        self.called = True
        self.launches += 1
        check(rc, what)

    def call_untimed(self, fname: str, args, what: str):
        """One C-ABI entry point on the launch's stream, inside a region the caller times."""
        rc = getattr(lib(), fname)(C.byref(args), self.stream_ptr)
        self.called = True
        self.launches += 1
        check(rc, what)

    def ptr(self, name, written: bool = False, covers: int = -1) -> Buffer:
        """The device buffer of pointer argument `name`; `written` marks the
        arguments the operator stores to (the ones copied back).  `covers` is the
        number of leading elements the launch writes, every one of them: when that
        is the whole of a plain numpy array, its old contents are never observable
        and the copy to the device is skipped."""
        if name not in self.buffers:
            v = self.args[name]
            if self.capturing and not _is_torch_tensor(getattr(v, "base", v)):
                raise TypeError(f"argument {name}: under CUDA-graph capture pass CUDA tensors (numpy arrays "
                                f"need host copies, which a graph cannot hold)")
            overwrite = (written and isinstance(v, np.ndarray) and covers == v.size and
                         not any(b.host is v for b in self.buffers.values()))
            self.buffers[name] = Buffer(name, v, self.device, self.stream, overwrite)
        if written:
            self.written.add(name)
        return self.buffers[name]

    def int(self, name) -> int:
        v = self.args[name]
        if isinstance(v, (bool, np.bool_)):
            return int(v)
        if not isinstance(v, (int, np.integer)):
            raise TypeError(f"argument {name}: expected an integer, got {type(v).__name__}")
        return int(v)

    def float(self, name) -> float:
        return float(self.args[name])

    def workspace(self, nbytes: int) -> int:
        torch = _torch()
        if nbytes == 0:
            return 0
        if self.capturing:
            # allocated from the graph's private pool, which stays reserved for the graph's
            # replays after this tensor is released
            buf = torch.empty(nbytes, dtype=torch.uint8, device=self.device or "cuda")
            return buf.data_ptr()
        key = torch.cuda.current_device() if self.device is None else self.device
        buf = _WORKSPACE.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(nbytes, dtype=torch.uint8, device=self.device or "cuda")
            _WORKSPACE[key] = buf
        return buf.data_ptr()

    def finish(self):
        """Copy the written arrays back to the host (the reference copies every
        array back, launcher.py:209-211; arrays a kernel only reads come back
        unchanged, so only the written ones need the copy)."""
        d2h = sum(self.buffers[n].copy_back(self.stream) for n in self.written) + self.host_d2h
        if not self.capturing:
            self.stream.synchronize()
        return sum(b.h2d_bytes for b in self.buffers.values()) + self.host_h2d, d2h


def run_on_b200(jitfn, grid, constants, values, device=None, qpu=False):
    """Run one launch; returns its stats dict."""
    fn = getattr(jitfn, "fn", jitfn)
    name = getattr(fn, "__name__", str(fn))
    params = tuple(getattr(jitfn, "arg_names", None) or fn.__code__.co_varnames[:fn.__code__.co_argcount])
    handler = _REGISTRY.get((name, params))
    if handler is None:
        raise NotImplementedError(f"{name}{params} has no B200 implementation "
                                  f"(registered: {[k[0] for k in registered()]})")
    torch = _torch()
    if not torch.cuda.is_available():
        raise RuntimeError("device='b200' needs a CUDA device; none is visible")
    lib()      # fail loudly before touching any buffer if the library is missing
    dev = torch.device("cuda", device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        launch = Launch(values, constants, dev, qpu)
        stats = dict(handler(launch, tuple(grid) + (1,) * (3 - len(grid))) or {})
        h2d, d2h = launch.finish()
        if launch.called and launch.ev0 is not None:
            stats["time_us"] = launch.ev0.elapsed_time(launch.ev1) * 1e3
        stats["h2d_bytes"], stats["d2h_bytes"] = h2d, d2h
        stats["launches"] = launch.launches
    return stats


def _flags(launch, allowed_qpu=True, simt_ok=False):
    """Flags word of an entry point: QPU rounding (launch option), and the CUDA-core
    path forced where an operator has both (PITON_B200_FORCE_SIMT=1, for comparisons)."""
    if launch.qpu and not allowed_qpu:
        raise NotImplementedError("qpu_rounding is implemented for add, softmax, matmul, dense and attention only")
    f = _lib.QPU_ROUNDING if launch.qpu else 0
    if simt_ok and os.environ.get("PITON_B200_FORCE_SIMT", "0") not in ("", "0"):
        f |= _lib.FORCE_SIMT
    return f


# ---------------------------------------------------------------------------------------
# host buffers: copies in, launches and copies back overlapped chunk by chunk
# ---------------------------------------------------------------------------------------

PIPE_MIN_BYTES = 64 << 20   # below this a transfer is short next to the per-chunk launch costs
PIPE_CHUNKS = 8
_COPY_STREAMS = {}


def _copy_streams(device):
    torch = _torch()
    key = device.index if device.index is not None else torch.cuda.current_device()
    st = _COPY_STREAMS.get(key)
    if st is None:
        st = (torch.cuda.Stream(device), torch.cuda.Stream(device))
        _COPY_STREAMS[key] = st
    return st


def _pipelined_on_host(L: Launch, ins, outs, units: int, align: int, launch_chunk) -> bool:
    """An operator whose inputs and outputs split along one leading dimension (rows of a
    softmax, elements of an add, heads of an attention), given as page-locked numpy arrays:
    chunk i's launch runs on the launch's stream while chunk i + 1 is copied in on one copy
    stream and chunk i - 1 is copied back on another, instead of all copies in, the launch,
    all copies back one after the other (the generic path, ``Buffer``).  ``ins`` / ``outs``
    are (argument name, array, elements per unit); ``launch_chunk(u0, u1, in_addrs,
    out_addrs)`` enqueues the operator for units [u0, u1) on the device copies (chunk
    boundaries are multiples of ``align`` units).  Elements of an output past ``units`` are
    neither copied in nor back, so they keep their host values, as the generic path leaves
    them.  Returns False, having done nothing, when the arguments do not qualify: under
    graph capture, fewer than PIPE_MIN_BYTES, arrays that are not C-contiguous page-locked
    float32 numpy arrays holding the units, or an output sharing memory with an input."""
    torch = _torch()
    if L.capturing or units <= 0:
        return False
    every = ins + outs
    arrs = [a for _, a, _ in every]
    if not all(type(a) is np.ndarray and a.dtype == np.float32 and a.flags.c_contiguous and a.size > 0
               for a in arrs):
        return False
    if any(a.size < units * e for _, a, e in every) or sum(4 * units * e for _, _, e in every) < PIPE_MIN_BYTES:
        return False
    if not all(a.flags.writeable for _, a, _ in outs):
        return False
    if any(np.may_share_memory(o, i) for _, o, _ in outs for _, i, _ in ins):
        return False
    host_in = [torch.from_numpy(a.reshape(-1)) for _, a, _ in ins]
    host_out = [torch.from_numpy(a.reshape(-1)) for _, a, _ in outs]
    if not all(t.is_pinned() for t in host_in + host_out):
        return False
    h2d, d2h = _copy_streams(L.device)
    dev_in = [torch.empty(units * e, dtype=torch.float32, device=L.device) for _, _, e in ins]
    dev_out = [torch.empty(units * e, dtype=torch.float32, device=L.device) for _, _, e in outs]
    # the device copies are used on the copy streams too: the allocator must not hand their
    # memory out again before the work queued there is done (also when a launch below fails)
    for t in dev_in:
        t.record_stream(h2d)
    for t in dev_out:
        t.record_stream(d2h)
    step = -(-units // PIPE_CHUNKS)
    step = -(-step // align) * align
    bounds = [(u, min(units, u + step)) for u in range(0, units, step)]
    start = torch.cuda.Event()
    start.record(L.stream)          # the copies follow whatever the stream already holds
    h2d.wait_event(start)
    d2h.wait_event(start)
    arrived = []
    with torch.cuda.stream(h2d):
        for u0, u1 in bounds:
            for t, h, (_, _, e) in zip(dev_in, host_in, ins):
                t[u0 * e:u1 * e].copy_(h[u0 * e:u1 * e], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
            arrived.append(ev)
    if L.ev0 is not None:
        L.ev0.record(L.stream)
    for (u0, u1), ev in zip(bounds, arrived):
        L.stream.wait_event(ev)
        launch_chunk(u0, u1, [t.data_ptr() + 4 * u0 * e for t, (_, _, e) in zip(dev_in, ins)],
                     [t.data_ptr() + 4 * u0 * e for t, (_, _, e) in zip(dev_out, outs)])
        done = torch.cuda.Event()
        done.record(L.stream)
        d2h.wait_event(done)
        with torch.cuda.stream(d2h):
            for t, h, (_, _, e) in zip(dev_out, host_out, outs):
                h[u0 * e:u1 * e].copy_(t[u0 * e:u1 * e], non_blocking=True)
    if L.ev1 is not None:
        L.ev1.record(L.stream)
    L.stream.wait_stream(d2h)       # finish() synchronises the stream: every copy back is done
    L.host_h2d += sum(4 * units * e for _, _, e in ins)
    L.host_d2h += sum(4 * units * e for _, _, e in outs)
    return True


# ---------------------------------------------------------------------------------------
# operators
# ---------------------------------------------------------------------------------------

@register("add_kernel", ("x_ptr", "y_ptr", "output_ptr", "n_elements", "BLOCK_SIZE"))
def _add(L: Launch, grid):
    n, blk = L.int("n_elements"), L.int("BLOCK_SIZE")
    n_eff = max(0, min(n, grid[0] * blk))
    flags = _flags(L)

    def chunk(u0, u1, ins, outs):
        L.call_untimed("piton_b200_add_f32",
                       _lib.AddArgs(ins[0], ins[1], outs[0], u1 - u0, blk, -(-(u1 - u0) // blk), flags, 0), "add_kernel")

    # whole programs per chunk (BLOCK_SIZE elements each), 16-byte aligned chunk starts
    if blk > 0 and _pipelined_on_host(L, [("x_ptr", L.args["x_ptr"], 1), ("y_ptr", L.args["y_ptr"], 1)],
                                      [("output_ptr", L.args["output_ptr"], 1)], n_eff, blk * (4 // math.gcd(blk, 4)),
                                      chunk):
        return {"bytes": 12 * n_eff, "flops": n_eff, "path": "add_vec4_host_pipelined"}
    x, y, out = L.ptr("x_ptr"), L.ptr("y_ptr"), L.ptr("output_ptr", written=True, covers=n_eff)
    for b in (x, y, out):
        b.require(0, n_eff - 1)
    a = _lib.AddArgs(x.addr, y.addr, out.addr, n, blk, grid[0], _flags(L), 0)
    L.call("piton_b200_add_f32", a, "add_kernel")
    return {"bytes": 12 * n_eff, "flops": n_eff, "path": "add_vec4"}


@register("softmax_kernel", ("output_ptr", "input_ptr", "input_row_stride", "output_row_stride", "n_cols",
                             "BLOCK_SIZE"))
def _softmax(L: Launch, grid):
    rows, ncols, blk = grid[0], L.int("n_cols"), L.int("BLOCK_SIZE")
    sin, sout = L.int("input_row_stride"), L.int("output_row_stride")
    n = max(0, min(ncols, blk))
    flags = _flags(L)

    def chunk(u0, u1, ins, outs):
        L.call_untimed("piton_b200_softmax_f32",
                       _lib.SoftmaxArgs(outs[0], ins[0], sin, sout, ncols, blk, u1 - u0, flags, 0), "softmax_kernel")

    # dense rows (row strides = n_cols, every column inside BLOCK_SIZE): chunks of whole rows
    if sin == sout == n == ncols and _pipelined_on_host(L, [("input_ptr", L.args["input_ptr"], n)],
                                                        [("output_ptr", L.args["output_ptr"], n)], rows, 1, chunk):
        return {"bytes": 8 * rows * n, "flops": 4 * rows * n, "path": "softmax_host_pipelined"}
    out, inp = L.ptr("output_ptr", written=True, covers=rows * n if sout == n else -1), L.ptr("input_ptr")
    inp.require(*extent((rows, sin), (n, 1)))
    out.require(*extent((rows, sout), (n, 1)))
    a = _lib.SoftmaxArgs(out.addr, inp.addr, sin, sout, ncols, blk, rows, _flags(L), 0)
    L.call("piton_b200_softmax_f32", a, "softmax_kernel")
    return {"bytes": 8 * rows * n, "flops": 4 * rows * n, "path": "softmax"}


@register("matmul_kernel", ("a_ptr", "b_ptr", "c_ptr", "M", "N", "K", "stride_am", "stride_ak", "stride_bk",
                            "stride_bn", "stride_cm", "stride_cn", "BLOCK_SIZE_M", "BLOCK_SIZE_N", "BLOCK_SIZE_K",
                            "GROUP_SIZE_M"))
def _matmul(L: Launch, grid):
    M, N, K = L.int("M"), L.int("N"), L.int("K")
    s = {k: L.int(k) for k in ("stride_am", "stride_ak", "stride_bk", "stride_bn", "stride_cm", "stride_cn")}
    bm, bn, bk, g = (L.int(k) for k in ("BLOCK_SIZE_M", "BLOCK_SIZE_N", "BLOCK_SIZE_K", "GROUP_SIZE_M"))
    full_grid = grid[0] >= -(-M // bm) * -(-N // bn)
    dense_c = s["stride_cm"] == N and s["stride_cn"] == 1 and full_grid
    if full_grid and M > 0 and N > 0 and not L.capturing and _matmul_on_host_buffers(L, M, N, K, s, bm, bn, bk, g,
                                                                                     grid):
        return {"bytes": 4 * (M * K + K * N + M * N), "flops": 2 * M * N * K, "path": "tcgen05_f16x3_host_pipelined"}
    A, B, Cb = L.ptr("a_ptr"), L.ptr("b_ptr"), L.ptr("c_ptr", written=True, covers=M * N if dense_c else -1)
    if M > 0 and N > 0 and grid[0] > 0:
        A.require(*extent((M, s["stride_am"]), (K, s["stride_ak"])))
        B.require(*extent((K, s["stride_bk"]), (N, s["stride_bn"])))
        Cb.require(*extent((M, s["stride_cm"]), (N, s["stride_cn"])))
    a = _lib.MatmulArgs(A.addr, B.addr, Cb.addr, M, N, K, s["stride_am"], s["stride_ak"], s["stride_bk"],
                        s["stride_bn"], s["stride_cm"], s["stride_cn"], bm, bn, bk, g, grid[0], 0, 0,
                        _flags(L, simt_ok=True), 0)
    ws = lib().piton_b200_matmul_workspace_size(C.byref(a))
    a.workspace, a.workspace_bytes = L.workspace(ws), ws
    L.call("piton_b200_matmul_f32", a, "matmul_kernel")
    return {"bytes": 4 * (M * K + K * N + M * N), "flops": 2 * M * N * K,
            "path": "qpu_rounding" if L.qpu else ("tcgen05_f16x3" if ws else "cuda_core")}


def _matmul_on_host_buffers(L: Launch, M, N, K, s, bm, bn, bk, g, grid) -> bool:
    """numpy A, B, C in dense row-major layout: one call of the host-buffer entry point,
    which pipelines the copies of A's row blocks and C's with the GEMM (the generic path
    copies everything in, launches, and copies back, one after the other).  False when the
    launch does not qualify; the generic path then runs."""
    arrs = [L.args[k] for k in ("a_ptr", "b_ptr", "c_ptr")]
    if not all(type(x) is np.ndarray and x.dtype == np.float32 and x.flags.c_contiguous for x in arrs):
        return False
    A, B, Cm = arrs
    if not Cm.flags.writeable or np.shares_memory(Cm, A) or np.shares_memory(Cm, B):
        return False
    if (s["stride_am"], s["stride_ak"], s["stride_bk"], s["stride_bn"], s["stride_cm"], s["stride_cn"]) != (K, 1, N, 1,
                                                                                                           N, 1):
        return False
    if A.size < M * K or B.size < K * N or Cm.size < M * N:
        return False
    flags = _flags(L, simt_ok=True)
    if flags:
        return False
    a = _lib.MatmulArgs(A.ctypes.data, B.ctypes.data, Cm.ctypes.data, M, N, K, K, 1, N, 1, N, 1, bm, bn, bk, g,
                        grid[0], 0, 0, 0, 0)
    ws = lib().piton_b200_matmul_host_workspace_size(C.byref(a))
    if ws == 0:
        return False
    a.workspace, a.workspace_bytes = L.workspace(ws), ws
    L.call("piton_b200_matmul_f32_host", a, "matmul_kernel")
    L.host_h2d, L.host_d2h = 4 * (M * K + K * N), 4 * M * N
    return True


@register("dense_layer_kernel", ("x_ptr", "w_ptr", "bias_ptr", "y_ptr", "M", "N", "K", "BLOCK_SIZE_M",
                                 "BLOCK_SIZE_N", "BLOCK_SIZE_K", "GROUP_SIZE_M", "ADD_BIAS", "RELU"))
def _dense(L: Launch, grid):
    M, N, K = L.int("M"), L.int("N"), L.int("K")
    bm, bn, bk, g = (L.int(k) for k in ("BLOCK_SIZE_M", "BLOCK_SIZE_N", "BLOCK_SIZE_K", "GROUP_SIZE_M"))
    add_bias, relu = bool(L.args["ADD_BIAS"]), bool(L.args["RELU"])
    X, Wt, Y = L.ptr("x_ptr"), L.ptr("w_ptr"), L.ptr("y_ptr", written=True)
    bias = L.ptr("bias_ptr") if add_bias else None
    if M > 0 and grid[0] > 0:
        X.require(0, M * K - 1)
        Wt.require(0, K * N - 1)
        Y.require(0, M * N - 1)
        if bias is not None:
            bias.require(0, N - 1)
    a = _lib.DenseArgs(X.addr, Wt.addr, bias.addr if bias else 0, Y.addr, M, N, K, bm, bn, bk, g, grid[0],
                       int(add_bias), int(relu), _flags(L), 0)
    L.call("piton_b200_dense_f32", a, "dense_layer_kernel")
    return {"bytes": 4 * (M * K + K * N + M * N + N), "flops": 2 * M * N * K, "path": "cuda_core"}


@register("attn_fwd_kernel", ("Q", "K", "V", "Out", "sm_scale", "stride_qh", "stride_qm", "stride_kh", "stride_kn",
                              "stride_kk", "stride_vh", "stride_vn", "stride_oh", "stride_om", "N_CTX", "HEAD_DIM",
                              "BLOCK_M", "BLOCK_N", "CAUSAL", "EVEN_N"))
def _attention(L: Launch, grid):
    n_ctx, d = L.int("N_CTX"), L.int("HEAD_DIM")
    bm, bn = L.int("BLOCK_M"), L.int("BLOCK_N")
    causal, even = bool(L.args["CAUSAL"]), bool(L.args["EVEN_N"])
    st = {k: L.int(k) for k in ("stride_qh", "stride_qm", "stride_kh", "stride_kn", "stride_kk", "stride_vh",
                                "stride_vn", "stride_oh", "stride_om")}
    heads = grid[1]
    rows = max(0, min(n_ctx, grid[0] * bm))
    keys = n_ctx if (causal or not even) else (n_ctx // bn) * bn
    hd = n_ctx * d
    flops = 4.0 * n_ctx * n_ctx * d * heads * (0.5 if causal else 1.0)
    flags = _flags(L, True, simt_ok=True)

    def chunk(h0, h1, ins, outs):
        a = _lib.AttentionArgs(ins[0], ins[1], ins[2], outs[0], L.float("sm_scale"), hd, d, hd, d, 1, hd, d, hd, d,
                               n_ctx, d, bm, bn, grid[0], h1 - h0, int(causal), int(even), 0, 0, flags, 0)
        ws = lib().piton_b200_attention_workspace_size(C.byref(a))
        a.workspace, a.workspace_bytes = L.workspace(ws), ws
        L.call_untimed("piton_b200_attention_f32", a, "attn_fwd_kernel")

    # dense [heads, N_CTX, HEAD_DIM] operands and every query row written: chunks of whole heads
    dense = all(st[k] == hd for k in ("stride_qh", "stride_kh", "stride_vh", "stride_oh")) and \
        all(st[k] == d for k in ("stride_qm", "stride_kn", "stride_vn", "stride_om")) and st["stride_kk"] == 1
    if dense and rows == n_ctx and _pipelined_on_host(L, [("Q", L.args["Q"], hd), ("K", L.args["K"], hd),
                                                          ("V", L.args["V"], hd)], [("Out", L.args["Out"], hd)],
                                                      heads, 1, chunk):
        return {"bytes": 4 * 4 * heads * n_ctx * d, "flops": flops, "path": "attention_host_pipelined"}
    Q, K, V, O = L.ptr("Q"), L.ptr("K"), L.ptr("V"), L.ptr("Out", written=True)
    if rows > 0 and heads > 0:
        Q.require(*extent((heads, st["stride_qh"]), (rows, st["stride_qm"]), (d, 1)))
        O.require(*extent((heads, st["stride_oh"]), (rows, st["stride_om"]), (d, 1)))
        kmax = min(keys, rows) if causal else keys
        K.require(*extent((heads, st["stride_kh"]), (kmax, st["stride_kn"]), (d, st["stride_kk"])))
        V.require(*extent((heads, st["stride_vh"]), (kmax, st["stride_vn"]), (d, 1)))
    a = _lib.AttentionArgs(Q.addr, K.addr, V.addr, O.addr, L.float("sm_scale"), st["stride_qh"], st["stride_qm"],
                           st["stride_kh"], st["stride_kn"], st["stride_kk"], st["stride_vh"], st["stride_vn"],
                           st["stride_oh"], st["stride_om"], n_ctx, d, bm, bn, grid[0], heads, int(causal),
                           int(even), 0, 0, _flags(L, True, simt_ok=True), 0)
    ws = lib().piton_b200_attention_workspace_size(C.byref(a))
    a.workspace, a.workspace_bytes = L.workspace(ws), ws
    L.call("piton_b200_attention_f32", a, "attn_fwd_kernel")
    return {"bytes": 4 * 4 * heads * n_ctx * d, "flops": flops,
            "path": "qpu_rounding" if L.qpu else ("tcgen05_f16x3" if ws else "cuda_core")}


@register("layernorm_kernel", ("x_ptr", "out_ptr", "n", "eps", "BLOCK"))
def _layernorm(L: Launch, grid):
    rows, n, blk = grid[0], L.int("n"), L.int("BLOCK")
    n_eff = max(0, min(n, blk))
    X, Y = L.ptr("x_ptr"), L.ptr("out_ptr", written=True)
    X.require(*extent((rows, blk), (n_eff, 1)))
    Y.require(*extent((rows, blk), (n_eff, 1)))
    a = _lib.LayernormArgs(X.addr, Y.addr, rows, n_eff, blk, blk, L.float("eps"), _flags(L, False), 0)
    L.call("piton_b200_layernorm_f32", a, "layernorm_kernel")
    return {"bytes": 8 * rows * n_eff, "flops": 5 * rows * n_eff, "path": "layernorm"}


def pinned_empty(shape, dtype=np.float32) -> np.ndarray:
    """A numpy array in page-locked host memory (fast, asynchronous H2D/D2H)."""
    torch = _torch()
    t = torch.empty(int(np.prod(shape)), dtype=getattr(torch, np.dtype(dtype).name), pin_memory=True)
    return t.numpy().reshape(shape)


__all__ = ["run_on_b200", "register", "registered", "Buffer", "Launch", "extent", "pinned_empty", "lib", "check"]


# ---- element-wise, integer, reduction, transpose and Life operators --------------------------

_ELEM_OPS = {"copy": 0, "mul": 1, "fma": 2, "scaled_relu": 3, "exp2": 4, "log2": 5, "recip": 6, "rsqrt": 7,
             "exp": 8, "sqrt": 9, "log": 10, "sigmoid": 11}


def _elementwise(L: Launch, grid, op: str, x: str, y, out: str, alpha: float = 0.0):
    n, blk = L.int("n"), L.int("BLOCK")
    n_eff = max(0, min(n, grid[0] * blk))
    bx, bo = L.ptr(x), L.ptr(out, written=True, covers=n_eff)
    by = L.ptr(y) if y else None
    for b in (bx, bo, by):
        if b is not None:
            b.require(0, n_eff - 1)
    qpu = L.qpu and _ELEM_OPS[op] <= 3
    if L.qpu and not qpu:
        raise NotImplementedError("qpu_rounding applies to copy, mul, fma and scaled_relu")
    a = _lib.ElementwiseArgs(bx.addr, by.addr if by else 0, bo.addr, n, blk, grid[0], float(alpha), _ELEM_OPS[op],
                             _lib.QPU_ROUNDING if qpu else 0)
    L.call("piton_b200_elementwise_f32", a, op)
    return {"bytes": 4 * n_eff * (3 if by else 2), "flops": n_eff, "path": f"elementwise_{op}"}


@register("copy_kernel", ("x_ptr", "out_ptr", "n", "BLOCK"))
def _copy(L, grid):
    return _elementwise(L, grid, "copy", "x_ptr", None, "out_ptr")


@register("mul_kernel", ("x_ptr", "y_ptr", "out_ptr", "n", "BLOCK"))
def _mul(L, grid):
    return _elementwise(L, grid, "mul", "x_ptr", "y_ptr", "out_ptr")


@register("fma_kernel", ("x_ptr", "y_ptr", "out_ptr", "n", "alpha", "BLOCK"))
def _fma(L, grid):
    return _elementwise(L, grid, "fma", "x_ptr", "y_ptr", "out_ptr", L.float("alpha"))


@register("scaled_relu_kernel", ("x_ptr", "out_ptr", "n", "alpha", "BLOCK"))
def _scaled_relu(L, grid):
    return _elementwise(L, grid, "scaled_relu", "x_ptr", None, "out_ptr", L.float("alpha"))


@register("sfu_kernel", ("x_ptr", "out_ptr", "n", "OP", "BLOCK"))
def _sfu(L, grid):
    op = ["exp2", "log2", "recip", "rsqrt", "exp", "sqrt"][min(max(L.int("OP"), 0), 5)]
    return _elementwise(L, grid, op, "x_ptr", None, "out_ptr")


@register("log_kernel", ("x_ptr", "out_ptr", "n", "BLOCK"))
def _log(L, grid):
    return _elementwise(L, grid, "log", "x_ptr", None, "out_ptr")


@register("sigmoid_kernel", ("x_ptr", "out_ptr", "n", "BLOCK"))
def _sigmoid(L, grid):
    return _elementwise(L, grid, "sigmoid", "x_ptr", None, "out_ptr")


@register("idiv_kernel", ("x_ptr", "y_ptr", "q_ptr", "r_ptr", "n", "BLOCK"))
def _idiv(L, grid):
    n, blk = L.int("n"), L.int("BLOCK")
    n_eff = max(0, min(n, grid[0] * blk))
    X, Y = L.ptr("x_ptr"), L.ptr("y_ptr")
    Q, R = L.ptr("q_ptr", written=True), L.ptr("r_ptr", written=True)
    for b in (X, Y, Q, R):
        if b.itemsize != 4:
            raise TypeError("idiv_kernel takes int32 or uint32 arrays")
        b.require(0, n_eff - 1)
    signed = str(X.tensor.dtype) in ("torch.int32",)
    a = _lib.IdivArgs(X.addr, Y.addr, Q.addr, R.addr, n, blk, grid[0], int(signed), 0)
    L.call("piton_b200_idiv_i32", a, "idiv_kernel")
    return {"bytes": 16 * n_eff, "flops": n_eff, "path": "idiv"}


def _row_reduce(L, grid, reduce):
    bm, bn = L.int("BLOCK_M"), L.int("BLOCK_N")
    n_cols, stride = L.int("n_cols"), L.int("stride")
    rows = grid[0] * bm
    cols = -(-n_cols // bn) * bn
    X, O = L.ptr("x_ptr"), L.ptr("out_ptr", written=True)
    X.require(*extent((rows, stride), (cols, 1)))
    O.require(0, rows - 1)
    a = _lib.RowReduceArgs(X.addr, O.addr, n_cols, stride, bm, bn, grid[0], reduce, 0)
    L.call("piton_b200_row_reduce_f32", a, "row_reduce")
    return {"bytes": 4 * rows * (cols + 1), "flops": rows * cols, "path": "row_max" if reduce else "row_sum"}


@register("row_sum_kernel", ("x_ptr", "out_ptr", "n_cols", "stride", "BLOCK_M", "BLOCK_N"))
def _row_sum(L, grid):
    return _row_reduce(L, grid, 0)


@register("row_max_kernel", ("x_ptr", "out_ptr", "n_cols", "stride", "BLOCK_M", "BLOCK_N"))
def _row_max(L, grid):
    return _row_reduce(L, grid, 1)


@register("transpose_kernel", ("x_ptr", "out_ptr", "n_rows", "n_cols", "stride_x", "stride_out", "BLOCK_M",
                               "BLOCK_N"))
def _transpose(L, grid):
    nr, nc = L.int("n_rows"), L.int("n_cols")
    sx, so = L.int("stride_x"), L.int("stride_out")
    X, O = L.ptr("x_ptr"), L.ptr("out_ptr", written=True)
    X.require(*extent((nr, sx), (nc, 1)))
    O.require(*extent((nc, so), (nr, 1)))
    a = _lib.TransposeArgs(X.addr, O.addr, nr, nc, sx, so, L.int("BLOCK_M"), L.int("BLOCK_N"), grid[0], 0, 0)
    L.call("piton_b200_transpose_f32", a, "transpose_kernel")
    return {"bytes": 8 * nr * nc, "flops": 0, "path": "transpose"}


def _life(L, grid, mode, cols_name, br_name, bc_name):
    nr, nc, st = L.int("n_rows"), L.int(cols_name), L.int("stride")
    S, D = L.ptr("src_ptr"), L.ptr("dst_ptr", written=True)
    for b in (S, D):
        if b.itemsize != 4:
            raise TypeError("Life grids are int32 cells or uint32 words")
        b.require(*extent((nr, st), (nc, 1)))
    a = _lib.LifeArgs(S.addr, D.addr, nr, nc, st, L.int(br_name), L.int(bc_name), grid[0], grid[1], mode, 0)
    L.call("piton_b200_life_step", a, "life")
    return {"bytes": 8 * nr * nc, "flops": 0, "path": ["life_tiles", "life_rows", "life_bits"][mode]}


@register("life_kernel", ("src_ptr", "dst_ptr", "n_rows", "n_cols", "stride", "BLOCK_R", "BLOCK_C"))
def _life_tiles(L, grid):
    return _life(L, grid, 0, "n_cols", "BLOCK_R", "BLOCK_C")


@register("life_rows_kernel", ("src_ptr", "dst_ptr", "n_rows", "n_cols", "stride", "ROWS", "BLOCK"))
def _life_rows(L, grid):
    return _life(L, grid, 1, "n_cols", "ROWS", "BLOCK")


@register("life_bits_kernel", ("src_ptr", "dst_ptr", "n_rows", "n_words", "stride", "ROWS", "BLOCK"))
def _life_bits(L, grid):
    return _life(L, grid, 2, "n_words", "ROWS", "BLOCK")
