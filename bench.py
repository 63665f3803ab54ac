"""Benchmark of the B200 backend on the hot-path configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--ops matmul,softmax,...]

Headline (``value``): fp32 matmul C = A @ B at 8192^3 (A, B ~ U[-1, 1]), the
operator the metric names first, sharded by M-tiles across ranks with an
NCCL all-gather of C at the end of every step (strong scaling: the total
problem is fixed).  The same line carries the other operators of the metric
in ``secondary``: row softmax (M = 32768 x N = 16384, GB/s), causal
attention (B=32, H=32, S=4096, D=64, TFLOP/s and GB/s), vector add
(n = 2^28, GB/s), the digits MLP on 1797 images (images/s) and TinyGPT
greedy decoding at batch 1 and 256 (tokens/s), each sharded the same way
(rows / batch x head / elements / images / sequences).

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
``torch.cuda.synchronize()``, measured with CUDA events on the launching
stream; the max over ranks is reported.  Inputs are larger than L2 (126 MB)
for every timed operator.  ``e2e`` runs the same matmul through the public
``kernel[grid](..., device="b200")`` call with pinned host numpy arrays:
host-to-device copies of A and B, the launch and the device-to-host copy of
C are inside its timed region.

``--impl reference`` times the reference's CPU algorithm for the headline
operator (the oracle restatement of the QPU emulator's sequential-k
round-toward-zero dot, all host threads) on a bounded row sample of the same
workload; under torchrun only rank 0 works.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "fp32 matmul TFLOPS + softmax/attn GB/s vs roofline at 1/2/4/8 B200"
MM = 8192
SM_M, SM_N = 32768, 16384
AT_B, AT_H, AT_S, AT_D = 32, 32, 4096, 64
ADD_N = 1 << 28
ATTN_BH = AT_B * AT_H


def profiled_traffic(name: str):
    """DRAM bytes of one launch (dram__bytes_read.sum + dram__bytes_write.sum) from the single-pass
    ncu capture summarised in profiles/<name>.md, whose line 'traffic per launch: <bytes> bytes
    (<units> ...)' gives the bytes and the units the captured launch processed: (bytes, units), or
    None when the summary is absent.  The capture is of an earlier run of the same kernel, not of
    this run; the bench line says so."""
    import re
    try:
        with open(os.path.join(REPO, "profiles", name + ".md")) as f:
            for line in f:
                m = re.match(r"traffic per launch: ([0-9.eE+]+) bytes \(([0-9.eE+]+) ", line.strip())
                if m:
                    return float(m.group(1)), float(m.group(2))
    except OSError:
        pass
    return None


def traffic_for(name: str, units: float):
    """The profiled DRAM bytes per launch of `name`, scaled to a launch of `units` (traffic of these
    streaming kernels grows in proportion to the units processed)."""
    t = profiled_traffic(name)
    if t is None:
        return None, None
    b, u = t
    return b * units / u, f"ncu capture in profiles/{name}.md ({u:g} units; scaled to {units:g})" if u != units \
        else f"ncu capture in profiles/{name}.md"


def roofline(bound: str, achieved: float, peak: float, unit: str, traffic=None, traffic_source=None, **extra):
    r = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak if peak else None,
         "traffic": traffic}
    if traffic_source:
        r["traffic_source"] = traffic_source
    r.update(extra)
    return r


def timed_e2e(torch, D, step, steps, warmup=1):
    """Seconds per step (max over ranks) of `step`, a call through the public API with host
    buffers; it returns the launch stats ({'h2d_bytes', 'd2h_bytes'})."""
    for _ in range(warmup):
        st = step()
    D.barrier(torch)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        st = step()
    e1.record(s)
    e1.synchronize()
    return D.max(torch, e0.elapsed_time(e1) / 1e3 / steps), st


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p["bf16_tflops_sustained"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, torch):
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self, torch):
        if self.pg is not None:
            self.pg.barrier()
        torch.cuda.synchronize()

    def max(self, torch, v: float) -> float:
        if self.pg is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def allgather(self, torch, out, piece):
        if self.pg is not None:
            from piton_b200 import sharding
            sharding.gather(self.pg, out, piece)

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def timed(torch, D, step, steps, warmup):
    """Run warmup + steps of `step()`, return (max-over-ranks seconds per step, seconds of the last kernel-only event pair)."""
    for _ in range(warmup):
        step()
    D.barrier(torch)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        step()
    e1.record(s)
    e1.synchronize()
    D.barrier(torch)
    sec = e0.elapsed_time(e1) / 1e3 / steps
    return D.max(torch, sec)


def shard(n, world, rank):
    from piton_b200 import sharding
    return sharding.shard(n, world, rank)


def bench_matmul(torch, D, args, lib_calls):
    """Rank r computes rows [r*M/N, (r+1)*M/N) of C.  At N > 1 the all-gather is fused into the
    GEMM epilogue (every finished tile is stored into each rank's full C over NVLink) and a
    1-element NCCL all-reduce after it is the completion barrier."""
    import ctypes as C
    from piton_b200 import sharding
    from piton_b200.runtime.cuda import _lib
    from piton_b200.runtime.cuda._lib import lib
    M = N = K = MM
    r0, mloc = shard(M, D.world, D.rank)
    g = torch.Generator(device="cuda").manual_seed(1234 + D.rank)
    A = torch.rand(mloc, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=torch.Generator(device="cuda").manual_seed(99)) * 2 - 1
    Cl = torch.empty(mloc, N, device="cuda")
    a = _lib.MatmulArgs(A.data_ptr(), B.data_ptr(), Cl.data_ptr(), mloc, N, K, K, 1, N, 1, N, 1, 8, 64, 8, 8,
                        (mloc // 8) * (N // 64), 0, 0, 0, 0)
    ws = lib().piton_b200_matmul_workspace_size(C.byref(a))
    wbuf = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = wbuf.data_ptr(), ws
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    f = lib().piton_b200_matmul_f32

    def kernel_only():
        _lib.check(f(C.byref(a), stream), "matmul")

    peer = None
    multicast = False
    if D.world > 1:
        # Peer stores (CUDA IPC buffers), spread over the next tile's chunks.  The NVSwitch
        # multicast variant (--allgather multicast) stores each element once, but every GPU then
        # also receives its own shard back through the switch: the all-gather is bound by each
        # GPU's NVLink ingress, which multicast raises from (N-1) to N shards.
        multicast = args.allgather == "multicast"
        if multicast:
            flag = torch.tensor([1 if sharding.SymmetricOutput.multicast_supported(torch.cuda.current_device())
                                 else 0], device="cuda")
            D.pg.all_reduce(flag, op=D.pg.ReduceOp.MIN)
            multicast = bool(flag.item())
        peer = sharding.SymmetricOutput(D.pg, M * N * 4) if multicast else sharding.PeerOutput(D.pg, M * N * 4)
        multicast = multicast and peer.multicast_ptr != 0
        gargs = _lib.AllgatherArgs()
        for r, p in enumerate(peer.peer_ptrs):
            gargs.peer_c[r] = p
        gargs.world, gargs.rank, gargs.row_offset, gargs.ldc = D.world, D.rank, r0, N
        if multicast:
            gargs.multicast_c = peer.multicast_ptr
        done = torch.zeros(1, device="cuda")
        fg = lib().piton_b200_matmul_allgather_f32

        def step():
            _lib.check(fg(C.byref(a), C.byref(gargs), stream), "matmul_allgather")
            D.pg.all_reduce(done)
    else:
        step = kernel_only

    n0 = lib().piton_b200_launch_count()
    kernel_only()
    torch.cuda.synchronize()
    per_call = lib().piton_b200_launch_count() - n0
    t_kernel = timed(torch, D, kernel_only, args.steps, args.warmup)
    # at N = 1 the step is the kernel-only call itself: one measurement serves both
    t_step = timed(torch, D, step, args.steps, args.warmup) if D.world > 1 else t_kernel
    lib_calls["launches"] += per_call * args.steps * (2 if D.world > 1 else 1)
    flops = 2.0 * M * N * K
    # correctness spot check of this rank's first rows against float64 (and, with the fused
    # all-gather, of the rows every rank wrote into this rank's full C)
    ref = A[:4].double() @ B.double()
    err = float((Cl[:4].double() - ref).abs().max() / ref.abs().max())
    if peer is not None:
        torch.cuda.synchronize()
        D.pg.barrier()
        got = peer.read(r0 * N * 4, 4 * N * 4).view(np.float32).reshape(4, N)
        err = max(err, float(np.abs(got - ref.cpu().numpy()).max() / float(ref.abs().max())))
        D.pg.barrier()
        peer.close()
    return {"flops": flops, "t_step": t_step, "t_kernel": t_kernel, "tc": ws > 0, "per_call": per_call,
            "err": err, "local_flops": 2.0 * mloc * N * K, "multicast": multicast}


def bench_softmax(torch, D, args, lib_calls):
    from piton_b200.kernels import softmax_kernel
    r0, mloc = shard(SM_M, D.world, D.rank)
    x = softmax_rows(torch, mloc, SM_N, 7 + D.rank)
    y = torch.empty_like(x)
    yfull = torch.empty(SM_M, SM_N, device="cuda") if D.world > 1 else y
    from piton_b200.runtime.cuda import _lib
    import ctypes as C
    from piton_b200.runtime.cuda._lib import lib
    a = _lib.SoftmaxArgs(y.data_ptr(), x.data_ptr(), SM_N, SM_N, SM_N, SM_N, mloc, 0, 0)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def kernel_only():
        _lib.check(lib().piton_b200_softmax_f32(C.byref(a), stream), "softmax")

    peer = None
    if D.world > 1 and args.allgather == "peer":
        # the all-gather fused into the kernel: every finished row is stored into each rank's full
        # output over NVLink; a 1-element NCCL all-reduce after it is the completion barrier
        from piton_b200 import sharding
        del yfull
        peer = sharding.PeerOutput(D.pg, SM_M * SM_N * 4)
        gargs = _lib.AllgatherArgs()
        for r, p in enumerate(peer.peer_ptrs):
            gargs.peer_c[r] = p
        gargs.world, gargs.rank, gargs.row_offset, gargs.ldc = D.world, D.rank, r0, SM_N
        done = torch.zeros(1, device="cuda")
        fs = lib().piton_b200_softmax_allgather_f32

        def step():
            _lib.check(fs(C.byref(a), C.byref(gargs), stream), "softmax_allgather")
            D.pg.all_reduce(done)
    else:
        def step():
            kernel_only()
            D.allgather(torch, yfull, y)

    t_kernel = timed(torch, D, kernel_only, args.steps, args.warmup)
    # at N = 1 the step is the kernel-only call itself: one measurement serves both
    t_step = timed(torch, D, step, args.steps, args.warmup) if D.world > 1 else t_kernel
    lib_calls["launches"] += args.steps * (2 if D.world > 1 else 1)
    ref = torch.softmax(x[:8].double(), 1)
    err = float(((y[:8].double() - ref).abs() / ref.abs().clamp_min(1e-37)).max())
    if peer is not None:
        # this rank's first rows as every rank stored them into this rank's full output
        torch.cuda.synchronize()
        D.pg.barrier()
        firsts = [None] * D.world
        D.pg.all_gather_object(firsts, ref[0].cpu().numpy())
        for r in range(D.world):
            got = peer.read(r * mloc * SM_N * 4, SM_N * 4).view(np.float32).astype(np.float64)
            err = max(err, float((np.abs(got - firsts[r]) / np.maximum(np.abs(firsts[r]), 1e-37)).max()))
        D.pg.barrier()
        peer.close()
        yfull = None
    del x, y, yfull
    e2e = None
    if not args.no_e2e:
        # the public launch with pinned host arrays: the rank's rows in, its rows out
        from piton_b200.runtime.cuda import pinned_empty
        xh, yh = pinned_empty((mloc, SM_N)), pinned_empty((mloc, SM_N))
        torch.from_numpy(xh).copy_(softmax_rows(torch, mloc, SM_N, 7 + D.rank))
        launch = softmax_kernel[(mloc,)]
        sec, st = timed_e2e(torch, D, lambda: launch(yh, xh, SM_N, SM_N, SM_N, BLOCK_SIZE=SM_N,
                                                     device="b200").last_stats, max(2, args.steps // 10))
        lib_calls["launches"] += (max(2, args.steps // 10) + 1) * st.get("launches", 1)
        e2e = {"sec": sec, "h2d": st["h2d_bytes"], "d2h": st["d2h_bytes"], "op_path": st.get("path")}
        del xh, yh
    return {"bytes": 8.0 * SM_M * SM_N, "t_step": t_step, "t_kernel": t_kernel, "err": err,
            "local_bytes": 8.0 * mloc * SM_N, "e2e": e2e}


def softmax_rows(torch, rows, cols, seed):
    """normal(0, 1) * 4 with 1 % of each row's entries set to -inf (never a whole row), the
    configuration's value distribution, generated on the device."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, cols, device="cuda", generator=g) * 4
    mask = torch.rand(rows, cols, device="cuda", generator=g) < 0.01
    mask[:, 0] = False
    return x.masked_fill_(mask, float("-inf"))


def bench_attention(torch, D, args, lib_calls):
    import ctypes as C
    from piton_b200.runtime.cuda import _lib
    from piton_b200.runtime.cuda._lib import lib
    BH = ATTN_BH
    h0, hloc = shard(BH, D.world, D.rank)
    q, k, v = (torch.randn(hloc, AT_S, AT_D, device="cuda") for _ in range(3))
    o = torch.empty_like(q)
    # at N > 1 (peer all-gather) the kernel stores each finished block of rows into every rank's full
    # output itself: a gather warp trails the softmax warps with NVLink peer stores
    fused = D.world > 1 and args.allgather == "peer"
    ofull = torch.empty(BH, AT_S, AT_D, device="cuda") if (D.world > 1 and not fused) else o
    sd = AT_S * AT_D
    a = _lib.AttentionArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 1.0 / np.sqrt(AT_D), sd, AT_D, sd,
                           AT_D, 1, sd, AT_D, sd, AT_D, AT_S, AT_D, 64, 64, AT_S // 64, hloc, 1, 1, 0, 0, 0, 0)
    ws = lib().piton_b200_attention_workspace_size(C.byref(a))
    wbuf = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = wbuf.data_ptr(), ws
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def kernel_only():
        _lib.check(lib().piton_b200_attention_f32(C.byref(a), stream), "attention")

    peer = None
    if fused:
        from piton_b200 import sharding
        peer = sharding.PeerOutput(D.pg, BH * sd * 4)
        gargs = _lib.AllgatherArgs()
        for r, p in enumerate(peer.peer_ptrs):
            gargs.peer_c[r] = p
        gargs.world, gargs.rank, gargs.row_offset = D.world, D.rank, h0
        done = torch.zeros(1, device="cuda")
        fa = lib().piton_b200_attention_allgather_f32

        def step():
            _lib.check(fa(C.byref(a), C.byref(gargs), stream), "attention_allgather")
            D.pg.all_reduce(done)   # completion barrier: every rank's stores have landed
    else:
        def step():
            kernel_only()
            D.allgather(torch, ofull, o)

    steps = max(1, args.steps // 4)
    n0 = lib().piton_b200_launch_count()
    kernel_only()
    per_call = lib().piton_b200_launch_count() - n0
    t_kernel = timed(torch, D, kernel_only, steps, args.warmup)
    # at N = 1 the step is the kernel-only call itself: one measurement serves both
    t_step = timed(torch, D, step, steps, args.warmup) if D.world > 1 else t_kernel
    lib_calls["launches"] += per_call * steps * (2 if D.world > 1 else 1)
    # spot check: head 0, first 64 query rows against float64
    qs, ks, vs = q[0].double(), k[0].double(), v[0].double()
    s = (qs[:64] @ ks.t()) / np.sqrt(AT_D)
    s = s.masked_fill(torch.ones(64, AT_S, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    ref = torch.softmax(s, 1) @ vs
    err = float((o[0, :64].double() - ref).abs().max())
    if peer is not None:
        # the fused all-gather's output: this rank's first rows in its own full output, and the next
        # rank's first rows as that rank's gather warp stored them here, against that rank's own copy
        torch.cuda.synchronize()
        D.pg.barrier()
        mine = peer.read(h0 * sd * 4, 64 * AT_D * 4).view(np.float32).reshape(64, AT_D)
        err = max(err, float(np.abs(mine - ref.cpu().numpy()).max()))
        sums = [None] * D.world
        D.pg.all_gather_object(sums, float(np.abs(mine.ravel().astype(np.float64)).sum()))
        nxt = (D.rank + 1) % D.world
        theirs = peer.read(nxt * hloc * sd * 4, 64 * AT_D * 4).view(np.float32)
        if float(np.abs(theirs.astype(np.float64)).sum()) != sums[nxt]:
            err = float("inf")
        D.pg.barrier()
        peer.close()
    flops = 4.0 * BH * AT_S * AT_S * AT_D * 0.5
    e2e = None
    if not args.no_e2e:
        # the public launch with pinned host arrays: the rank's heads of Q, K, V in, of O out
        from piton_b200.kernels import attn_fwd_kernel
        from piton_b200.runtime.cuda import pinned_empty
        hq, hk, hv, ho = (pinned_empty((hloc, AT_S, AT_D)) for _ in range(4))
        for h_, d_ in ((hq, q), (hk, k), (hv, v)):
            torch.from_numpy(h_).copy_(d_)
        del q, k, v, o, ofull, wbuf
        launch = attn_fwd_kernel[(AT_S // 2, hloc)]
        sm = float(1.0 / np.sqrt(AT_D))
        sec, st = timed_e2e(torch, D, lambda: launch(hq, hk, hv, ho, sm, sd, AT_D, sd, AT_D, 1, sd, AT_D, sd, AT_D, AT_S,
                                                     HEAD_DIM=AT_D, BLOCK_M=2, BLOCK_N=16, CAUSAL=True, EVEN_N=True,
                                                     device="b200").last_stats, 2)
        lib_calls["launches"] += 3 * st.get("launches", 1) * per_call
        e2e = {"sec": sec, "h2d": st["h2d_bytes"], "d2h": st["d2h_bytes"], "op_path": st.get("path")}
        del hq, hk, hv, ho
    return {"flops": flops, "bytes": 16.0 * BH * AT_S * AT_D, "t_step": t_step, "t_kernel": t_kernel, "err": err,
            "local_flops": flops * hloc / BH, "tc": ws > 0, "fused": fused, "e2e": e2e, "heads_local": hloc}


def bench_add(torch, D, args, lib_calls):
    import ctypes as C
    from piton_b200.runtime.cuda import _lib
    from piton_b200.runtime.cuda._lib import lib
    n0, nloc = shard(ADD_N, D.world, D.rank)
    g = torch.Generator(device="cuda").manual_seed(11 + D.rank)
    x = torch.rand(nloc, device="cuda", generator=g) * 2 - 1          # U[-1, 1], the configuration's inputs
    y = torch.rand(nloc, device="cuda", generator=g) * 2 - 1
    out = torch.empty_like(x)
    ofull = torch.empty(ADD_N, device="cuda") if D.world > 1 else out
    a = _lib.AddArgs(x.data_ptr(), y.data_ptr(), out.data_ptr(), nloc, 1024, (nloc + 1023) // 1024, 0, 0)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def kernel_only():
        _lib.check(lib().piton_b200_add_f32(C.byref(a), stream), "add")

    peer = None
    if D.world > 1 and args.allgather == "peer":
        # the all-gather fused into the kernel (NVLink peer stores of every result element), a
        # 1-element NCCL all-reduce after it as the completion barrier
        from piton_b200 import sharding
        del ofull
        ofull = None
        peer = sharding.PeerOutput(D.pg, nloc * D.world * 4)
        gargs = _lib.AllgatherArgs()
        for r, p in enumerate(peer.peer_ptrs):
            gargs.peer_c[r] = p
        gargs.world, gargs.rank, gargs.row_offset = D.world, D.rank, n0
        done = torch.zeros(1, device="cuda")
        fa = lib().piton_b200_add_allgather_f32

        def step():
            _lib.check(fa(C.byref(a), C.byref(gargs), stream), "add_allgather")
            D.pg.all_reduce(done)
    else:
        def step():
            kernel_only()
            D.allgather(torch, ofull, out)

    t_kernel = timed(torch, D, kernel_only, args.steps, args.warmup)
    # at N = 1 the step is the kernel-only call itself: one measurement serves both
    t_step = timed(torch, D, step, args.steps, args.warmup) if D.world > 1 else t_kernel
    lib_calls["launches"] += args.steps * (2 if D.world > 1 else 1)
    err = float((out[:1 << 20] - (x[:1 << 20] + y[:1 << 20])).abs().max())
    if peer is not None:
        # this rank's range in its own full output, and a checksum of every rank's range there
        torch.cuda.synchronize()
        D.pg.barrier()
        got = torch.from_numpy(peer.read(n0 * 4, (1 << 20) * 4).view(np.float32)).cuda()
        err = max(err, float((got - (x[:1 << 20] + y[:1 << 20])).abs().max()))
        sums = [None] * D.world
        D.pg.all_gather_object(sums, float((x + y).double().sum()))
        for r in range(D.world):
            theirs = peer.read(r * nloc * 4, nloc * 4).view(np.float32).astype(np.float64).sum()
            if abs(theirs - sums[r]) > 1e-6 * max(1.0, abs(sums[r])):
                err = float("inf")
        D.pg.barrier()
        peer.close()
    e2e = None
    if not args.no_e2e:
        from piton_b200.kernels import add_kernel
        from piton_b200.runtime.cuda import pinned_empty
        xh, yh, oh = pinned_empty((nloc,)), pinned_empty((nloc,)), pinned_empty((nloc,))
        torch.from_numpy(xh).copy_(x)
        torch.from_numpy(yh).copy_(y)
        del x, y, out, ofull
        launch = add_kernel[((nloc + 1023) // 1024,)]
        k = max(2, args.steps // 10)
        sec, st = timed_e2e(torch, D, lambda: launch(xh, yh, oh, nloc, BLOCK_SIZE=1024, device="b200").last_stats, k)
        lib_calls["launches"] += (k + 1) * st.get("launches", 1)
        e2e = {"sec": sec, "h2d": st["h2d_bytes"], "d2h": st["d2h_bytes"], "op_path": st.get("path")}
        del xh, yh, oh
    return {"bytes": 12.0 * ADD_N, "t_step": t_step, "t_kernel": t_kernel, "err": err, "local_bytes": 12.0 * nloc,
            "e2e": e2e}


def bench_tinygpt(torch, D, args, lib_calls, batch):
    """Greedy decode of `batch` sequences sharded by batch (sharding.batch_piece: each rank decodes
    its ceil(batch / N) prompts of one fixed seeded batch).  A batch smaller than N (batch 1)
    cannot shard: there every rank decodes its own single sequence (weak scaling, labelled so)."""
    from piton_b200 import sharding, tinygpt
    model = tinygpt.TinyGPT(tinygpt.init_weights(0))
    if batch >= D.world:
        prompts, _ = sharding.batch_piece(tinygpt.random_prompts(batch, seed=100), D.world, D.rank)
    else:
        prompts = tinygpt.random_prompts(1, seed=100 + D.rank)
    per = len(prompts)
    buf = np.zeros((per, tinygpt.CTX), np.int32)
    buf[:, :tinygpt.PROMPT_LEN] = prompts
    base = torch.from_numpy(buf).cuda()
    toks = base.clone()
    full = torch.empty(per * D.world, tinygpt.CTX, dtype=torch.int32, device="cuda") if D.world > 1 else toks

    def run(graph):
        def step():
            toks.copy_(base)
            model.generate_device(toks, tinygpt.PROMPT_LEN, tinygpt.NEW_TOKENS, graph=graph)
            D.allgather(torch, full, toks)
        return step

    steps = max(2, args.steps // 4)
    t_eager = timed(torch, D, run(False), steps, args.warmup)
    # the decode's launches replayed from a CUDA graph the library captured on first use
    t = timed(torch, D, run(True), steps, args.warmup)
    from piton_b200.runtime.cuda._lib import lib
    n0 = lib().piton_b200_launch_count()
    model.generate_device(toks, tinygpt.PROMPT_LEN, tinygpt.NEW_TOKENS)
    torch.cuda.synchronize()
    per_decode = lib().piton_b200_launch_count() - n0
    lib_calls["launches"] += 2 * steps * per_decode
    e2e = None
    if not args.no_e2e:
        # the public call with host prompts in and host tokens out (TinyGPT.generate)
        k = max(2, args.steps // 10)
        sec, _ = timed_e2e(torch, D, lambda: (model.generate(prompts), {})[1], k)
        lib_calls["launches"] += (k + 1) * per_decode
        e2e = {"sec": sec, "h2d": int(buf.nbytes), "d2h": int(buf.nbytes)}
    return {"tokens": per * D.world * tinygpt.NEW_TOKENS, "t_step": t, "t_eager": t_eager, "e2e": e2e,
            "batch": per * D.world, "per_rank": per, "weak": batch < D.world}


def bench_mlp(torch, D, args, lib_calls):
    from piton_b200 import digits, sharding, workloads as W
    rows = 1797
    imgs, _ = sharding.batch_piece(W.digits_images(rows, 0), D.world, D.rank)
    per = len(imgs)
    model = digits.DigitsMLP(W.digits_model(0))
    x = torch.from_numpy(imgs).cuda()
    logits = torch.empty(per, 16, device="cuda")
    pred = torch.empty(per, dtype=torch.int32, device="cuda")
    full = torch.empty(per * D.world, dtype=torch.int32, device="cuda") if D.world > 1 else pred

    def step():
        model.forward_device(x, logits, pred)
        D.allgather(torch, full, pred)

    t = timed(torch, D, step, args.steps, args.warmup)
    lib_calls["launches"] += args.steps
    out = {"images": rows, "t_step": t, "t_eager": t}
    if D.world == 1:
        # the same forward captured once into a CUDA graph and replayed: one graph launch per step
        # instead of a Python call into the library, as a serving loop would run it
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            model.forward_device(x, logits, pred)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            model.forward_device(x, logits, pred)
        out["t_step"] = timed(torch, D, g.replay, args.steps, args.warmup)
        lib_calls["launches"] += args.steps
        del g
    if not args.no_e2e:
        # the public call: host uint8 images in, host logits and predictions out
        sec, _ = timed_e2e(torch, D, lambda: (model(imgs, return_pred=True), {})[1], args.steps)
        lib_calls["launches"] += args.steps + 1
        out["e2e"] = {"sec": sec, "h2d": int(imgs.nbytes), "d2h": per * (16 * 4 + 4)}
    return out


def run_sweep(args):
    """The HBM-bound operators over the sizes of the B200 sweep (one GPU): add n = 2^20 ... 2^28 and
    softmax 32768 x N, N = 256 ... 16384.  Each launch is timed alone with CUDA events after a
    256 MB write has evicted the 126 MB L2 (the smaller inputs would otherwise be served from
    it); the median of 10 launches.  One JSON line."""
    import ctypes as C
    import statistics

    import torch
    from piton_b200.runtime.cuda import _lib
    from piton_b200.runtime.cuda._lib import lib
    peaks = load_peaks()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def median_seconds(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(10):
            flush.zero_()
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) / 1e3)
        return statistics.median(ts)

    out = {"add": [], "softmax": []}
    for lg in (20, 22, 24, 26, 28):
        n = 1 << lg
        x, y = torch.rand(n, device="cuda"), torch.rand(n, device="cuda")
        z = torch.empty_like(x)
        a = _lib.AddArgs(x.data_ptr(), y.data_ptr(), z.data_ptr(), n, 1024, (n + 1023) // 1024, 0, 0)
        t = median_seconds(lambda: _lib.check(lib().piton_b200_add_f32(C.byref(a), stream), "add"))
        out["add"].append({"n": n, "us": 1e6 * t, "gbs": 12.0 * n / t / 1e9,
                           "frac_of_copy": 12.0 * n / t / 1e9 / peaks["hbm_gbs"]})
        del x, y, z
    M = 32768
    for N in (256, 1024, 4096, 16384):
        x = torch.randn(M, N, device="cuda") * 4
        y = torch.empty_like(x)
        a = _lib.SoftmaxArgs(y.data_ptr(), x.data_ptr(), N, N, N, N, M, 0, 0)
        t = median_seconds(lambda: _lib.check(lib().piton_b200_softmax_f32(C.byref(a), stream), "softmax"))
        out["softmax"].append({"M": M, "N": N, "us": 1e6 * t, "gbs": 8.0 * M * N / t / 1e9,
                               "frac_of_copy": 8.0 * M * N / t / 1e9 / peaks["hbm_gbs"]})
        del x, y
    print(json.dumps({"sweep": out, "timing": "median of 10 launches, L2 evicted before each",
                      "peaks": {"hbm_gbs": peaks["hbm_gbs"], "source": peaks["source"]}}))
    return 0


def tf32_peak(torch):
    """cuBLAS TF32 GEMM throughput at 8192^3 (the denominator of the tensor-core GEMM roofline)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(8192, 8192, device="cuda")
    b = torch.randn(8192, 8192, device="cuda")
    for _ in range(3):
        torch.matmul(a, b)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 1e9
    for _ in range(5):
        e0.record()
        torch.matmul(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1) / 1e3)
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    return 2.0 * 8192 ** 3 / best / 1e12


def e2e_matmul(torch, D, steps):
    """The public launch with pinned host arrays: H2D of A and B, kernel, D2H of C."""
    import piton_b200 as triton
    from piton_b200.kernels import matmul_kernel
    from piton_b200.runtime.cuda import pinned_empty
    M = N = K = MM
    r0, mloc = shard(M, D.world, D.rank)
    rng = np.random.default_rng(5 + D.rank)
    A = pinned_empty((mloc, K))
    A[...] = rng.uniform(-1, 1, (mloc, K)).astype(np.float32)
    B = pinned_empty((K, N))
    B[...] = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    Cm = pinned_empty((mloc, N))
    grid = (triton.cdiv(mloc, 8) * triton.cdiv(N, 64),)

    if D.world > 1:
        # every rank uploads its A rows and 1/N of B; B is completed over NVLink (peer stores)
        from piton_b200 import sharding
        hs = sharding.HostShardedMatmul(D.pg, mloc, N, K)

        def step():
            hs(A, B, Cm)
            return {"h2d_bytes": hs.h2d_bytes(), "d2h_bytes": hs.d2h_bytes()}
    else:
        hs = None

        def step():
            return matmul_kernel[grid](A, B, Cm, mloc, N, K, K, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64,
                                       BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200").last_stats

    st = step()
    D.barrier(torch)
    t0 = time.perf_counter()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        step()
    e1.record(s)
    e1.synchronize()
    sec = D.max(torch, max(e0.elapsed_time(e1) / 1e3, 0.0) / steps)
    _ = t0
    if hs is not None:
        D.barrier(torch)
        hs.close()
    return {"sec": sec, "h2d": st["h2d_bytes"], "d2h": st["d2h_bytes"], "flops": 2.0 * M * N * K}


def cpu_baseline_matmul(rows: int, threads: int):
    """The oracle's restatement of the emulator's matmul on `rows` rows of the 8192^3 workload."""
    from oracle import oracle as O
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (rows, MM)).astype(np.float32)
    b = rng.uniform(-1, 1, (MM, MM)).astype(np.float32)
    t0 = time.perf_counter()
    O.qpu_matmul(a, b, threads=threads)
    sec = time.perf_counter() - t0
    return 2.0 * rows * MM * MM / sec / 1e12, sec


def cpu_baseline_blas(threads: int) -> dict:
    """numpy float32 A @ B at the full 8192^3 size on the host's BLAS (OpenBLAS sgemm, all host
    threads): a plain fp32 CPU product beside the reference-semantics port, not the reference."""
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, (MM, MM)).astype(np.float32)
    b = rng.uniform(-1, 1, (MM, MM)).astype(np.float32)
    a[:64] @ b                                        # warm the BLAS threads
    t0 = time.perf_counter()
    a @ b
    sec = time.perf_counter() - t0
    try:
        import threadpoolctl
        info = [p for p in threadpoolctl.threadpool_info() if p.get("user_api") == "blas"]
        blas = f"{info[0]['internal_api']} {info[0]['version']}, {info[0]['num_threads']} threads" if info else "BLAS"
        cores = info[0]["num_threads"] if info else threads
    except Exception:   # threadpoolctl is optional: report the host's thread count
        blas, cores = "BLAS", threads
    return {"value": 2.0 * MM ** 3 / sec / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "numpy",
            "sample": f"one full {MM}^3 numpy float32 A @ B ({sec:.2f} s, {blas}); not the reference's arithmetic"}


def sample_rows(seconds: float, rate_tflops: float, threads: int) -> int:
    """Rows of the 8192^3 product that take about `seconds` at `rate_tflops`, a whole number per
    thread (at least one, at most all 8192)."""
    rows = int(seconds * rate_tflops * 1e12 / (2.0 * MM * MM)) // threads * threads
    return max(threads, min(MM, rows))


def cpu_baselines_secondary(threads: int) -> dict:
    """The oracle's restatements of the reference's CPU path for the other operators, each on a
    bounded sample of its benchmark workload (a few seconds in all), reported beside the B200
    figures (the oracle's C kernels are single-threaded unless noted)."""
    from oracle import oracle as O
    from oracle import tinygpt_ref
    from piton_b200 import tinygpt, workloads as W
    out = {}
    rng = np.random.default_rng(0)
    n = 1 << 24
    x, y = rng.uniform(-1, 1, n).astype(np.float32), rng.uniform(-1, 1, n).astype(np.float32)
    t0 = time.perf_counter()
    O.qpu_add(x, y)
    sec = time.perf_counter() - t0
    out["add"] = {"value": 12.0 * n / sec / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
                  "sample": f"n = 2^24 of the 2^28-element workload, round-toward-zero adds"}
    rows = 128
    xs = W.softmax_input(rows, SM_N, 0)
    t0 = time.perf_counter()
    O.qpu_softmax(xs, SM_N)
    sec = time.perf_counter() - t0
    out["softmax"] = {"value": 8.0 * rows * SM_N / sec / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
                      "sample": f"{rows} of the 32768 rows x {SM_N} columns, the QPU exp polynomial and butterflies"}
    s_len = 1024
    q, k, v = W.attention_inputs(1, s_len, AT_D, 0)
    t0 = time.perf_counter()
    O.qpu_attention(q, k, v, True, 2, 16)
    sec = time.perf_counter() - t0
    out["attention"] = {"value": 4.0 * s_len * s_len * AT_D * 0.5 / sec / 1e12, "unit": "TFLOP/s", "cores": 1,
                        "kind": "port", "sample": f"one head, S = {s_len}, D = 64, causal (the benchmark has 1024 "
                                                  f"heads of S = 4096)"}
    imgs = W.digits_images(1797, 0)
    t0 = time.perf_counter()
    O.qpu_mlp(imgs, W.digits_model(0), threads=threads)
    sec = time.perf_counter() - t0
    out["mlp_digits_1797"] = {"value": 1797 / sec, "unit": "images/s", "cores": threads, "kind": "port",
                              "sample": "all 1797 images, the three dense layers with round-toward-zero dots"}
    w = tinygpt.init_weights(0)
    prompts = tinygpt.random_prompts(1, seed=100)
    new = 8
    t0 = time.perf_counter()
    tinygpt_ref.generate(w, prompts, new)
    sec = time.perf_counter() - t0
    out["tinygpt_b1"] = {"value": new / sec, "unit": "tokens/s", "cores": 1, "kind": "port",
                         "sample": f"batch 1, {new} of the 64 greedy tokens, float64 numpy host model"}
    prompts = tinygpt.random_prompts(256, seed=100)
    t0 = time.perf_counter()
    tinygpt_ref.generate(w, prompts, new)
    sec = time.perf_counter() - t0
    out["tinygpt_b256"] = {"value": 256 * new / sec, "unit": "tokens/s", "cores": threads, "kind": "port",
                           "sample": f"batch 256, {new} of the 64 greedy tokens (the first steps, the cheapest "
                                     f"per token), float64 numpy host model with a KV cache, BLAS threads"}
    return out


def run_reference(args):
    D = Dist()
    if D.rank != 0:
        return 0
    threads = os.cpu_count() or 1
    # calibrate on one row per thread (the oracle splits rows over threads), then size each step to
    # ~min(10 s, 120 s / steps) in whole rows per thread
    rate, _ = cpu_baseline_matmul(threads, threads)
    per_step = min(10.0, 120.0 / max(1, args.steps))
    rows = sample_rows(per_step, rate, threads)
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_baseline_matmul(max(1, rows // 4), threads)
    vals, t_all = [], 0.0
    for _ in range(args.steps):
        v, sec = cpu_baseline_matmul(rows, threads)
        vals.append(v)
        t_all += sec
    value = statistics.median(vals)
    sample = (f"{rows} of 8192 rows of C per step ({rows}x8192x8192 multiply-adds), the oracle's restatement of the "
              f"emulator's sequential-k round-toward-zero dot on {threads} threads")
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * t_all / max(1, args.steps), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"matmul C=A@B fp32 {MM}x{MM}x{MM}, A,B ~ U[-1,1] (bounded row sample)"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    global MM, ATTN_BH, ADD_N, SM_M
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ops", default="matmul,softmax,attention,add,mlp,tinygpt")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mm-size", type=int, default=MM, help="matmul M=N=K (profiling runs use a smaller case)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--allgather", default="peer", choices=["peer", "multicast"],
                    help="matmul all-gather at N > 1: peer stores, or multimem stores to an NVSwitch multicast address")
    ap.add_argument("--attn-bh", type=int, default=AT_B * AT_H, help="attention batch x heads (profiling runs use fewer)")
    ap.add_argument("--add-n", type=int, default=1 << 28, help="vector add elements (profiling runs use fewer)")
    ap.add_argument("--softmax-m", type=int, default=32768, help="softmax rows (profiling runs use fewer)")
    ap.add_argument("--sweep", action="store_true",
                    help="instead of the benchmark line: add and softmax over the sweep sizes (1 GPU)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    MM = args.mm_size
    ATTN_BH, ADD_N, SM_M = args.attn_bh, args.add_n, args.softmax_m
    if args.impl == "reference":
        return run_reference(args)
    if args.sweep:
        return run_sweep(args)

    import torch
    D = Dist()
    D.init(torch)
    ops = args.ops.split(",")
    peaks = load_peaks()
    sampler = ClockSampler(D.local)
    lib_calls = {"launches": 0}
    res = {}
    sampler.start()
    try:
        if "matmul" in ops:
            res["matmul"] = bench_matmul(torch, D, args, lib_calls)
        if "softmax" in ops:
            res["softmax"] = bench_softmax(torch, D, args, lib_calls)
        if "attention" in ops:
            res["attention"] = bench_attention(torch, D, args, lib_calls)
        if "add" in ops:
            res["add"] = bench_add(torch, D, args, lib_calls)
        if "mlp" in ops:
            res["mlp"] = bench_mlp(torch, D, args, lib_calls)
        if "tinygpt" in ops:
            res["tinygpt_b1"] = bench_tinygpt(torch, D, args, lib_calls, D.world)
            res["tinygpt_b256"] = bench_tinygpt(torch, D, args, lib_calls, 256)
    finally:
        sampler.stop()
    e2e = e2e_matmul(torch, D, max(2, args.steps // 5)) if "matmul" in ops and not args.no_e2e else None
    tf32 = tf32_peak(torch) if ("matmul" in ops or "attention" in ops) else None
    D.close()
    if D.rank != 0:
        return 0

    from piton_b200 import tinygpt
    hbm = peaks["hbm_gbs"]
    tf32_src = f"cuBLAS TF32 8192^3 measured in this run ({tf32:.1f} TFLOP/s)" if tf32 else None

    def e2e_entry(r, units, unit, scale):
        e = r.get("e2e")
        if not e:
            return None
        return {"value": units / e["sec"] / scale, "unit": unit, "h2d_bytes_per_step": e["h2d"],
                "d2h_bytes_per_step": e["d2h"], "ms_per_step": 1e3 * e["sec"],
                "path": "the public call with pinned host buffers (copy in, launch, copy back every step"
                        + ("; the copies overlapped with the launches chunk by chunk)"
                           if "host_pipelined" in (e.get("op_path") or "") else ")")
                        + ("; per rank: its own shard in and out, max over ranks" if D.world > 1 else "")}

    sec = {}
    for name, kernel, cfg in (("softmax", "softmax_reg_kernel", f"{SM_M} x {SM_N}"),
                              ("add", "add_vec4_kernel", f"n = {ADD_N}")):
        if name in res:
            r = res[name]
            ach = r["local_bytes"] / r["t_kernel"] / 1e9
            units = SM_M * SM_N if name == "softmax" else ADD_N
            trf, trf_src = traffic_for(name + "_dram", units / D.world) if D.world == 1 else (None, None)
            sec[name] = {"value": r["bytes"] / r["t_step"] / 1e9, "unit": "GB/s", "workload": cfg,
                         "kernel_gbs_per_gpu": ach,
                         "roofline": roofline("hbm", ach, hbm, "GB/s", trf, trf_src, kernel=kernel,
                                              algorithmic_bytes_per_launch=r["local_bytes"],
                                              peak_source=f"MEASURED_PEAKS.json hbm_gbs ({peaks['source']})"),
                         "ms_per_step": 1e3 * r["t_step"],
                         "max_rel_err" if name == "softmax" else "max_abs_err": r["err"]}
            e = e2e_entry(r, r["local_bytes"] * D.world, "GB/s", 1e9)
            if e:
                sec[name]["e2e"] = e
            if D.world > 1:
                sec[name]["value_without_allgather"] = r["bytes"] / r["t_kernel"] / 1e9
    if "attention" in res:
        r = res["attention"]
        ach = r["local_flops"] / r["t_kernel"] / 1e12
        peak = peaks["bf16_tflops"] / 3.0
        trf, trf_src = traffic_for("attn_f16x3_bh64", r["heads_local"]) if D.world == 1 else (None, None)
        sec["attention"] = {"value": r["flops"] / r["t_step"] / 1e12, "unit": "TFLOP/s",
                            "workload": f"B={AT_B} H={AT_H} S={AT_S} D={AT_D} causal (B x H = {ATTN_BH})",
                            "gbs": r["bytes"] / r["t_step"] / 1e9,
                            "kernel_tflops_per_gpu": ach,
                            "roofline": roofline("tensor", ach, peak, "TFLOP/s", trf, trf_src,
                                                 kernel="attn_f16x3_kernel",
                                                 peak_source=f"MEASURED_PEAKS.json bf16_tflops "
                                                             f"({peaks['bf16_tflops']:.1f}, {peaks['source']}) / 3: per "
                                                             "useful 16-deep product the kernel issues one N=128 fp16 "
                                                             "MMA (hi.[hi;lo], two units) and one N=64 (lo.hi, one "
                                                             "unit)",
                                                 frac_of_tf32_over_3=(ach / (tf32 / 3.0)) if tf32 else None,
                                                 gbs_over_4BHSD4=r["bytes"] / r["t_kernel"] / 1e9 / D.world
                                                 if D.world > 1 else r["bytes"] / r["t_kernel"] / 1e9),
                            "path": "tcgen05 fp16 split (Q per row, K and V per 64-key block, P x 2^14: "
                                    "hi.hi + hi.lo + lo.hi)" if r.get("tc")
                                    else "CUDA-core fp32",
                            "allgather": ("fused: the kernel's gather warp stores finished rows to every rank "
                                          "(NVLink peer stores)" if r.get("fused") else
                                          "NCCL all_gather_into_tensor after the kernel") if D.world > 1 else None,
                            "ms_per_step": 1e3 * r["t_step"], "max_abs_err_vs_f64": r["err"]}
        e = e2e_entry(r, r["local_flops"] * D.world, "TFLOP/s", 1e12)
        if e:
            sec["attention"]["e2e"] = e
        if D.world > 1:
            sec["attention"]["value_without_allgather"] = r["flops"] / r["t_kernel"] / 1e12
    if "mlp" in res:
        r = res["mlp"]
        flops = 2.0 * r["images"] * (64 * 128 + 128 * 64 + 64 * 16)
        ffma = 148 * 128 * 2 * 1.965e9 / 1e12
        sec["mlp_digits_1797"] = {"value": r["images"] / r["t_step"], "unit": "images/s",
                                  "ms_per_step": 1e3 * r["t_step"], "eager_value": r["images"] / r["t_eager"],
                                  "roofline": roofline("latency", flops / D.world / r["t_step"] / 1e12, ffma,
                                                       "TFLOP/s", kernel="mlp_kernel",
                                                       us_per_forward=1e6 * r["t_step"],
                                                       peak_source="fp32 FFMA nominal: 148 SMs x 128 lanes x 2 x "
                                                                   "1.965 GHz; 62.6 MFLOP per forward is far below "
                                                                   "any throughput roof, the time is launch and L2 "
                                                                   "latency"),
                                  "workload": "1797 images through 64-128-64-16 in one launch; value: the launch "
                                              "replayed from a CUDA graph (N = 1), eager_value: one library call "
                                              "per step from Python"}
        e = e2e_entry(r, r["images"], "images/s", 1.0)
        if e:
            sec["mlp_digits_1797"]["e2e"] = e
    for key in ("tinygpt_b1", "tinygpt_b256"):
        if key in res:
            r = res[key]
            pos = tinygpt.PROMPT_LEN + tinygpt.NEW_TOKENS - 1
            ent = {"value": r["tokens"] / r["t_step"], "unit": "tokens/s", "ms_per_step": 1e3 * r["t_step"],
                   "eager_value": r["tokens"] / r["t_eager"], "batch": r["batch"],
                   "workload": "greedy decode of 64 tokens after 16-token prompts; batches up to the "
                               "number of 16-CTA clusters that fit (9 on 148 SMs) run as one cluster launch "
                               "per decode with the weights in shared memory, larger batches with 2 sequences "
                               "per CTA as one launch per decode (each CTA feeds its sequences' positions in "
                               "turn); value: replayed from a CUDA graph, eager_value: launched directly"}
            if r["weak"]:
                ent["scaling"] = "weak"
                ent["workload"] += f"; at N = {D.world} every GPU decodes its own single sequence (batch 1 " \
                                   f"cannot shard): {r['batch']} sequences in all"
            if key == "tinygpt_b256":
                # algorithmic bytes of one decode: the weights once per fed position plus, per sequence
                # and position p, the K and V rows 0..p of every layer read and row p written
                wbytes = 4.0 * tinygpt.pack(tinygpt.init_weights(0)).size
                kv = 2 * tinygpt.N_LAYER * tinygpt.D_MODEL * 4.0
                per_seq = sum(kv * (p + 1) + kv for p in range(pos))
                byts = pos * wbytes + r["per_rank"] * per_seq
                ent["roofline"] = roofline("hbm", byts / r["t_step"] / 1e9, hbm, "GB/s",
                                           kernel="tinygpt_step_kernel",
                                           algorithmic_bytes_per_decode=byts,
                                           note="KV cache (134 MB at batch 256) and weights mostly L2-resident")
            else:
                ent["roofline"] = roofline("latency", 1e6 * r["t_step"] / pos, None, "us per fed position",
                                           kernel="tinygpt_cluster_kernel")
            e = e2e_entry(r, r["tokens"], "tokens/s", 1.0)
            if e:
                ent["e2e"] = e
            sec[key] = ent
    line = {"metric": METRIC, "n_gpus": D.world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded torch.rand / randn on device)"}
    if "matmul" in res:
        r = res["matmul"]
        value = r["flops"] / r["t_step"] / 1e12
        ach = r["local_flops"] / r["t_kernel"] / 1e12
        # per 16-deep k-step of useful work the GEMM issues three fp16 MMAs of depth 16 (A_hi B_hi,
        # A_hi B_lo, A_lo B_hi), fp16 running at the bf16 rate: the instruction mix's peak is the
        # measured dense bf16 throughput / 3; classic 3xTF32 (the north star's bound) is TF32 / 3
        peak = peaks["bf16_tflops"] / 3.0
        gemm_traffic = (profiled_traffic("gemm_dram_8192") or (None, None))[0] if (D.world == 1 and MM == 8192) \
            else None
        gemm_traffic = (gemm_traffic, "ncu capture of an earlier run of this kernel, profiles/gemm_dram_8192.md"
                        if gemm_traffic else None)
        line.update({"value": value, "unit": "TFLOP/s", "ms_per_step": 1e3 * r["t_step"],
                     "config": {"workload": f"matmul C=A@B fp32 {MM}x{MM}x{MM}, A,B ~ U[-1,1], sharded by M-tiles, "
                                            f"all-gather of C each step" + (
                                                (" fused into the GEMM epilogue (multimem stores to an NVSwitch "
                                                 "multicast address)" if r["multicast"] else
                                                 " fused into the GEMM epilogue (NVLink peer stores)")
                                                if D.world > 1 else ""),
                                "M": MM, "N": MM, "K": MM, "parallelism": f"m-tiles x{D.world}",
                                "l2": "inputs larger than L2 (A+B = 512 MB)",
                                "path": "tcgen05 fp16 split, per 256-deep chunk power-of-two scaling: "
                                        "A_hi B_hi + A_hi B_lo + A_lo B_hi (three kind::f16 MMAs per 16 k-values)"
                                        if r["tc"] else "CUDA-core fp32 FFMA"},
                     "roofline": {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                                  "frac": ach / peak,
                                  # DRAM bytes of one launch of the CTA-pair GEMM at 8192^3 from the committed
                                  # single-pass ncu capture (dram__bytes_read.sum + dram__bytes_write.sum)
                                  "traffic": gemm_traffic[0], "traffic_source": gemm_traffic[1],
                                  "traffic_unit": "bytes per launch",
                                  "peak_source": f"MEASURED_PEAKS.json bf16_tflops ({peaks['bf16_tflops']:.1f}, "
                                                 f"{peaks['source']}, burst) / 3: three 16-deep fp16 MMAs per 16-deep "
                                                 "k-step of useful work",
                                  "frac_of_bf16_sustained_over_3": ach / (peaks["bf16_tflops_sustained"] / 3.0),
                                  "frac_of_tf32_over_3": ach / (tf32 / 3.0),
                                  "tf32_measured_tflops": tf32},
                     "max_norm_err_vs_f64": r["err"]})
        if D.world > 1:
            # the same sharded product with each rank's C rows left local (no all-gather), timed as the max
            # over ranks: the scaling of the computation alone
            line["value_without_allgather"] = r["flops"] / r["t_kernel"] / 1e12
        lib_calls_total = lib_calls["launches"]
        line["gpu_launches"] = lib_calls_total
    else:
        line["gpu_launches"] = lib_calls["launches"]
    if e2e:
        line["e2e"] = {"value": e2e["flops"] / e2e["sec"] / 1e12, "unit": "TFLOP/s",
                       "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                       "ms_per_step": 1e3 * e2e["sec"],
                       "path": ("kernel[grid](numpy pinned host arrays): H2D of A and B, GEMM, D2H of C, pipelined "
                                "by row blocks" if D.world == 1 else
                                "sharding.HostShardedMatmul (pinned host arrays): each rank uploads its A rows and "
                                "1/N of B's rows, B completed over NVLink, GEMM, D2H of its C rows; bytes per rank")}
    line["secondary"] = sec
    line["peaks"] = {"hbm_gbs": hbm, "source": peaks["source"]}
    line["clocks"] = sampler.summary()
    if "matmul" in ops and D.world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, _ = cpu_baseline_matmul(threads, threads)   # one row per thread: the calibration
        rows = sample_rows(15.0, rate, threads)
        v, s = cpu_baseline_matmul(rows, threads)
        line["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                                "sample": f"{rows} of {MM} rows of the {MM}^3 product ({s:.1f} s): the oracle's "
                                          f"restatement of the emulator's sequential-k round-toward-zero dot"}
        line["cpu_baseline_blas"] = cpu_baseline_blas(threads)
    if D.world == 1 and not args.no_cpu_baseline and line.get("secondary"):
        # the reference's CPU path for the other operators, beside their B200 figures
        for key, cb in cpu_baselines_secondary(os.cpu_count() or 1).items():
            if key in line["secondary"]:
                line["secondary"][key]["cpu_baseline"] = cb
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
