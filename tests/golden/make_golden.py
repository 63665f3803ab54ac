"""Generate golden output fixtures by running the PIton reference itself.

This script imports the reference (PIton, a pure-Python package) from a local
checkout and runs its strict QPU emulator on the hot-path operators:

* ``add_kernel`` / ``softmax_kernel`` / ``matmul_kernel``  examples/kernels.py
* ``dense_layer_kernel``                                  examples/nn_kernels.py
* ``attn_fwd_kernel``                                     examples/attention.py

It writes one ``.npz`` per case next to this file.  Small cases keep their
inputs and outputs; large cases keep the seed (inputs are rebuilt with
``piton_b200.workloads``), a SHA-256 of the input and output bytes and a
sample of the outputs.  The fixtures are what the CPU oracle (``oracle/``) is
pinned against and what the GPU parity tests compare with.

Usage (in a container that has the reference checkout):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --ref /path/to/PIton [--big] [--procs 8]

Large launches are split across processes by program id: every program of
these kernels writes a disjoint set of output elements, so each worker runs a
slice of the grid on its own emulator instance and the parent merges the
elements each slice wrote.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import multiprocessing as mp
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from piton_b200 import workloads as W  # noqa: E402

REF_FILES = ["piton/qpu/emulator.py", "piton/backend/lower.py", "piton/runtime/launcher.py",
             "examples/kernels.py", "examples/nn_kernels.py", "examples/attention.py"]

_STATE = {}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_fingerprint(ref: str) -> str:
    h = hashlib.sha256()
    for f in REF_FILES:
        with open(os.path.join(ref, f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def save(name: str, meta: dict, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, meta=json.dumps(meta, sort_keys=True), **arrays)
    print(f"wrote {os.path.relpath(path, REPO)} ({os.path.getsize(path) // 1024} KB)", flush=True)


def exists(name: str) -> bool:
    return os.path.exists(os.path.join(HERE, name + ".npz"))


# -- split runner --------------------------------------------------------------------

def _worker(args):
    """Run the programs `pids` of the kernel compiled in the parent; return the
    output array element indices that changed and their new bits."""
    progs, out_name, offsets = args
    from piton.qpu.emulator import V3D
    from piton.runtime.launcher import uniforms_for, slot_semaphores, semaphore_programs
    ck, values, k = _STATE["ck"], _STATE["values"], _STATE["coarsen"]
    v = V3D(num_qpus=12, strict=True)
    addrs = {}
    sentinel = None
    for name, val in values.items():
        if isinstance(val, np.ndarray):
            base = v.mem.alloc(max(val.nbytes, 4), 64)
            arr = val
            if name == out_name:
                sentinel = np.full(val.shape, np.float32(-7.25e33), np.float32)
                arr = sentinel
            v.mem.write_array(base, arr)
            addrs[name] = base + 4 * offsets.get(name, 0)
    zero = v.mem.alloc(64, 64)
    scratch = v.mem.alloc(64, 64)
    unifs = []
    for pid, g in progs:
        a = v.mem.alloc(4 * max(len(ck.uniforms), 1), 16)
        u = uniforms_for(ck, values, addrs, pid, g, zero, scratch, a, k)
        if u:
            v.mem.write_words(a, np.array(u, dtype=np.uint32))
        unifs.append(a)
    sems = slot_semaphores(ck.words)
    if sems:
        init, fini = semaphore_programs(sems)
        v.run(v.load(init), [zero])
    v.run(v.load(ck.words), unifs)
    if sems:
        v.run(v.load(fini), [zero])
    base = addrs[out_name] - 4 * offsets.get(out_name, 0)
    got = v.mem.read_array(base, values[out_name].shape, np.float32).ravel()
    changed = np.flatnonzero(got.view(np.uint32) != sentinel.ravel().view(np.uint32))
    return changed, got[changed]


def run_split(jitfn, grid, signature, constants, values, out_name, procs, offsets=None):
    """Emulate `jitfn` on `grid`, its programs split over `procs` processes."""
    from piton.compiler import compile as pcompile
    from piton.runtime.launcher import launch_coarsen, program_ids
    bound = tuple(1 << max(0, int(g) - 1).bit_length() for g in grid)
    ck = pcompile(jitfn, signature, constants, num_stages=2, grid=bound)
    k = launch_coarsen(ck, grid)
    _STATE.update(ck=ck, values=values, coarsen=k)
    progs = list(program_ids(grid, k))
    chunks = [progs[i::procs] for i in range(procs)]
    out = values[out_name].ravel().copy()
    with mp.get_context("fork").Pool(procs) as pool:
        for changed, bits in pool.imap_unordered(_worker, [(c, out_name, offsets or {}) for c in chunks if c]):
            out[changed] = bits
    return out.reshape(values[out_name].shape)


# -- cases ----------------------------------------------------------------------------

def case_add(fp, procs, big):
    import piton
    from kernels import add_kernel
    cases = [(64, 64, 1), (1000, 64, 2), (4096, 256, 3), (37, 16, 4), (16, 16, 5), (65537, 256, 0)]
    for n, block, seed in cases:
        name = f"add_n{n}_b{block}"
        if exists(name):
            continue
        x, y = W.vector_add(n, seed)
        t = time.time()
        if n <= 4096:
            out = np.full(n + 16, np.float32(7.0), np.float32)
            add_kernel[(piton.cdiv(n, block),)](x, y, out, n, BLOCK_SIZE=block)
            assert np.all(out[n:] == 7.0)
            out = out[:n]
        else:
            sig = {"x_ptr": "*fp32", "y_ptr": "*fp32", "output_ptr": "*fp32", "n_elements": "i32"}
            out = run_split(add_kernel, (piton.cdiv(n, block),), sig, {"BLOCK_SIZE": block},
                            dict(x_ptr=x, y_ptr=y, output_ptr=np.zeros(n, np.float32), n_elements=n),
                            "output_ptr", procs)
        meta = dict(op="add", n=n, block=block, seed=seed, ref=fp, emu_seconds=time.time() - t,
                    sha_x=sha(x), sha_y=sha(y), sha_out=sha(out))
        if n <= 4096:
            save(name, meta, x=x, y=y, out=out)
        else:
            idx = np.arange(0, n, 61)
            save(name, meta, sample_idx=idx, sample=out[idx])


def case_softmax(fp, procs, big):
    import piton
    from kernels import softmax_kernel
    # the reference's own test shapes, then rows of the 1823 x 781 configuration
    cases = [(4, 64, 64, 11), (3, 100, 128, 12), (5, 16, 16, 13), (24, 781, 1024, 0)]
    if big:
        cases.append((1823, 781, 1024, 0))
    for m, n, block, seed in cases:
        name = f"softmax_m{m}_n{n}_b{block}"
        if exists(name):
            continue
        # rows of the config case come from the full 1823-row input
        x = W.softmax_input(1823 if n == 781 else m, n, seed)[:m]
        t = time.time()
        sig = {"output_ptr": "*fp32", "input_ptr": "*fp32", "input_row_stride": "i32",
               "output_row_stride": "i32", "n_cols": "i32"}
        y = run_split(softmax_kernel, (m,), sig, {"BLOCK_SIZE": block},
                      dict(output_ptr=np.zeros((m, n), np.float32), input_ptr=x, input_row_stride=n,
                           output_row_stride=n, n_cols=n), "output_ptr", procs)
        meta = dict(op="softmax", m=m, n=n, block=block, seed=seed, ref=fp, emu_seconds=time.time() - t,
                    sha_x=sha(x), sha_out=sha(y))
        if m * n <= 24 * 781:
            save(name, meta, x=x, out=y)
        else:
            save(name, meta, rows=np.arange(0, m, 37), sample=y[::37])


def case_matmul(fp, procs, big):
    import piton
    from kernels import matmul_kernel
    # (M, N, K, BM, BN, BK, G, K_const, negative C row stride, seed).  The reference's
    # compiler runs out of QPU registers for an 8x64x8 tile whose K has a masked tail
    # (K % 8 != 0, regalloc.py:660), so those shapes use BLOCK_SIZE_K = 4.
    cases = [(64, 64, 64, 8, 64, 4, 4, True, False, 21), (72, 100, 64, 8, 64, 4, 4, True, False, 22),
             (40, 70, 36, 8, 64, 4, 4, False, False, 23), (16, 128, 32, 8, 64, 4, 4, True, False, 24),
             (40, 70, 36, 8, 64, 4, 8, True, True, 25), (128, 128, 128, 8, 64, 8, 8, True, False, 0)]
    if big:
        cases += [(512, 512, 512, 8, 64, 8, 8, True, False, 0), (1000, 777, 513, 8, 64, 4, 8, True, True, 0),
                  (1024, 1024, 1024, 8, 64, 8, 8, True, False, 0)]
    for M, N, K, bm, bn, bk, g, kconst, neg, seed in cases:
        name = f"matmul_{M}x{N}x{K}_t{bm}x{bn}x{bk}_g{g}" + ("_negc" if neg else "") + ("" if kconst else "_rtk")
        if exists(name):
            continue
        a, b = W.matmul_inputs(M, N, K, seed)
        t = time.time()
        consts = dict(BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk, GROUP_SIZE_M=g,
                      stride_ak=1, stride_bn=1, stride_cn=1)
        sig = {n_: "*fp32" for n_ in ("a_ptr", "b_ptr", "c_ptr")}
        sig.update({n_: "i32" for n_ in ("M", "N", "stride_am", "stride_bk", "stride_cm")})
        if kconst:
            consts["K"] = K
        else:
            sig["K"] = "i32"
        # C is stored bottom-up when the row stride is negative: row m at (M-1-m)*N
        stride_cm = -N if neg else N
        offsets = {"c_ptr": (M - 1) * N} if neg else {}
        vals = dict(a_ptr=a, b_ptr=b, c_ptr=np.zeros((M, N), np.float32), M=M, N=N,
                    stride_am=K, stride_bk=N, stride_cm=stride_cm)
        if not kconst:
            vals["K"] = K
        grid = (piton.cdiv(M, bm) * piton.cdiv(N, bn),)
        store = run_split(matmul_kernel, grid, sig, consts, vals, "c_ptr", procs, offsets)
        c = store[::-1] if neg else store            # c[m] = row m of the product
        meta = dict(op="matmul", M=M, N=N, K=K, block=[bm, bn, bk], group=g, k_const=kconst,
                    negative_stride_cm=neg, seed=seed, ref=fp, emu_seconds=time.time() - t,
                    sha_a=sha(a), sha_b=sha(b), sha_c=sha(np.ascontiguousarray(c)))
        if M * N * K <= 128 ** 3:
            save(name, meta, a=a, b=b, c=np.ascontiguousarray(c))
        else:
            rows = np.arange(0, M, 29)
            save(name, meta, rows=rows, sample=np.ascontiguousarray(c[rows]))


def case_dense(fp, procs, big):
    from nn_kernels import dense_layer_kernel, dense_tiles
    import piton.compiler as pc
    from piton.runtime.launcher import run_emulator
    # dyadic cases (products and sums exact): the reference test's shapes
    for m, n, k, add_bias, relu in [(8, 64, 64, True, True), (9, 17, 11, True, False),
                                    (3, 10, 7, False, True), (1, 16, 8, False, False)]:
        name = f"dense_dyadic_m{m}_n{n}_k{k}_b{int(add_bias)}_r{int(relu)}"
        if exists(name):
            continue
        rng = np.random.default_rng(340 + m)
        x = W.dyadic((m, k), -4, 4, rng)
        w = W.dyadic((k, n), -4, 4, rng)
        bias = W.dyadic((n,), -8, 8, rng)
        y = _run_dense(pc, run_emulator, dense_layer_kernel, dense_tiles, x, w, bias, add_bias, relu)
        save(name, dict(op="dense", m=m, n=n, k=k, add_bias=add_bias, relu=relu, ref=fp,
                        tiles=list(dense_tiles(n))), x=x, w=w, bias=bias, out=y)
    # three-layer digits MLP on synthetic images and synthetic weights
    for rows, seed in ([(64, 0)] + ([(1797, 0)] if big else [])):
        name = f"mlp_digits_m{rows}"
        if exists(name):
            continue
        imgs = W.digits_images(rows, seed)
        model = W.digits_model(seed)
        h = (imgs.astype(np.float32) / np.float32(16)).astype(np.float32)
        t = time.time()
        for layer in (1, 2, 3):
            h = _run_dense(pc, run_emulator, dense_layer_kernel, dense_tiles, h, model[f"w{layer}"],
                           model[f"b{layer}"], True, layer < 3)
        meta = dict(op="mlp", m=rows, seed=seed, ref=fp, emu_seconds=time.time() - t, sha_out=sha(h))
        save(name, meta, images=imgs, logits=h, **model)


def _run_dense(pc, run_emulator, kern, tiles_fn, x, w, bias, add_bias, relu):
    m, k = x.shape
    n = w.shape[1]
    bm, bn, bk = tiles_fn(n)
    grid = ((m + bm - 1) // bm * ((n + bn - 1) // bn),)
    constants = dict(N=n, K=k, BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk, GROUP_SIZE_M=1,
                     ADD_BIAS=add_bias, RELU=relu)
    sig = dict.fromkeys(("x_ptr", "w_ptr", "bias_ptr", "y_ptr"), "*fp32")
    sig["M"] = "i32"
    ck = pc.compile(kern, sig, constants, grid=grid, num_stages=2)
    y = np.zeros(m * n, np.float32)
    run_emulator(ck, grid, dict(x_ptr=np.ascontiguousarray(x), w_ptr=w, bias_ptr=bias, y_ptr=y, M=m))
    return y.reshape(m, n)


def case_attention(fp, procs, big):
    import attention as A
    # (heads, n_ctx, head_dim, block_m, block_n, causal, seed)
    cases = [(1, 64, 16, 2, 16, False, 82), (1, 64, 16, 2, 16, True, 83), (1, 64, 32, 2, 32, True, 99),
             (1, 37, 16, 2, 16, False, 37), (1, 37, 16, 2, 16, True, 38), (2, 48, 16, 2, 16, True, 5),
             (1, 256, 64, 2, 16, True, 0)]
    if big:
        cases.append((16, 256, 64, 2, 16, True, 0))
    for heads, n, d, bm, bn, causal, seed in cases:
        name = f"attn_h{heads}_n{n}_d{d}_t{bm}x{bn}_c{int(causal)}"
        if exists(name):
            continue
        q, k, v = W.attention_inputs(heads, n, d, seed)
        t = time.time()
        even = n % bn == 0
        consts = dict(HEAD_DIM=d, BLOCK_M=bm, BLOCK_N=bn, CAUSAL=bool(causal), EVEN_N=bool(even),
                      **A.contiguous_strides(d, "nd", n))
        sig = A.signature_for(consts)
        vals = dict(Q=q, K=k, V=v, Out=np.zeros_like(q), sm_scale=float(1 / np.sqrt(d)), N_CTX=n,
                    stride_qh=n * d, stride_kh=n * d, stride_vh=n * d, stride_oh=n * d)
        vals = {key: val for key, val in vals.items() if key in sig}
        out = run_split(A.attn_fwd_kernel, (-(-n // bm), heads), sig, consts, vals, "Out", procs)
        meta = dict(op="attention", heads=heads, n=n, d=d, block=[bm, bn], causal=causal, seed=seed,
                    ref=fp, emu_seconds=time.time() - t, sha_out=sha(out))
        if heads * n * d <= 256 * 64:
            save(name, meta, q=q, k=k, v=v, out=out)
        else:
            save(name, meta, heads_kept=np.arange(2), out_first_heads=out[:2])


def case_tinygpt(fp, procs, big):
    """TinyGPT -- a model the reference does not have -- composed from the reference's own
    kernels on its emulator: dense_layer_kernel (RELU off) for every linear layer,
    attn_fwd_kernel for the causal heads (head dim 32), layernorm_kernel
    (tests/test_reroll_reduce.py) for the LayerNorms; the embeddings, the LayerNorm gain and
    bias, GELU and the residual adds on the host in float32.  A prefill of a short prompt,
    the logits of every position: pins the float64 host model (oracle/tinygpt_ref.py) and the
    B200 decode to the reference's kernels at small size."""
    from nn_kernels import dense_layer_kernel, dense_tiles
    import attention as A
    import piton.compiler as pc
    from piton.runtime.launcher import run_emulator
    sys.path.insert(0, os.path.join(_STATE["ref"], "tests"))
    import test_reroll_reduce as RR
    from piton_b200 import tinygpt
    plen, seed = 5, 0
    name = f"tinygpt_emu_p{plen}_seed{seed}"
    if exists(name):
        return
    t = time.time()
    w = tinygpt.init_weights(seed)
    prompt = tinygpt.random_prompts(1, seed=7, length=plen)[0]
    f32 = np.float32
    x = (w["wte"][prompt] + w["wpe"][:plen]).astype(f32)

    def ln(v, g, b):
        rows = v.shape[0]
        sig = {"x_ptr": "*fp32", "out_ptr": "*fp32", "n": "i32", "eps": "fp32"}
        ck = pc.compile(RR.layernorm_kernel, sig, {"BLOCK": tinygpt.D_MODEL}, grid=(rows,), num_stages=2)
        y = np.zeros_like(v)
        run_emulator(ck, (rows,), dict(x_ptr=np.ascontiguousarray(v), out_ptr=y, n=tinygpt.D_MODEL, eps=1e-5))
        return (y * g + b).astype(f32)

    def dense(v, wm, b):
        return _run_dense(pc, run_emulator, dense_layer_kernel, dense_tiles, np.ascontiguousarray(v, f32),
                          np.ascontiguousarray(wm, f32), np.ascontiguousarray(b, f32), True, False)

    def heads(m):   # [plen, 128] -> [4, plen, 32]
        return np.ascontiguousarray(m.reshape(plen, tinygpt.N_HEAD, -1).transpose(1, 0, 2))

    hd = tinygpt.D_MODEL // tinygpt.N_HEAD
    consts = dict(HEAD_DIM=hd, BLOCK_M=2, BLOCK_N=16, CAUSAL=True, EVEN_N=plen % 16 == 0,
                  **A.contiguous_strides(hd, "nd", plen))
    asig = A.signature_for(consts)
    for layer in range(tinygpt.N_LAYER):
        p = {k: w[f"h{layer}.{k}"] for k, _ in tinygpt.LAYER_TENSORS}
        h = ln(x, p["ln1_g"], p["ln1_b"])
        qkv = dense(h, p["w_qkv"], p["b_qkv"])
        d = tinygpt.D_MODEL
        q, k, v = heads(qkv[:, :d]), heads(qkv[:, d:2 * d]), heads(qkv[:, 2 * d:])
        vals = dict(Q=q, K=k, V=v, Out=np.zeros_like(q), sm_scale=float(1 / np.sqrt(hd)), N_CTX=plen,
                    stride_qh=plen * hd, stride_kh=plen * hd, stride_vh=plen * hd, stride_oh=plen * hd)
        vals = {key: val for key, val in vals.items() if key in asig}
        att = run_split(A.attn_fwd_kernel, (-(-plen // 2), tinygpt.N_HEAD), asig, consts, vals, "Out", procs)
        att = np.ascontiguousarray(att.reshape(tinygpt.N_HEAD, plen, hd).transpose(1, 0, 2).reshape(plen, d))
        x = (x + dense(att, p["w_o"], p["b_o"])).astype(f32)
        h2 = ln(x, p["ln2_g"], p["ln2_b"])
        fpre = dense(h2, p["w_fc"], p["b_fc"]).astype(np.float64)
        import math
        gelu = (0.5 * fpre * (1.0 + np.vectorize(math.erf)(fpre / math.sqrt(2.0)))).astype(f32)
        x = (x + dense(gelu, p["w_pr"], p["b_pr"])).astype(f32)
    hf = ln(x, w["lnf_g"], w["lnf_b"])
    logits = dense(hf, np.ascontiguousarray(w["wte"].T), np.zeros(tinygpt.VOCAB, f32))
    meta = dict(op="tinygpt_prefill", prompt_len=plen, weight_seed=seed, prompt_seed=7, ref=fp,
                emu_seconds=time.time() - t)
    save(name, meta, prompt=prompt.astype(np.int32), logits=logits)


def case_tinygpt_decode(fp, procs, big):
    """TinyGPT greedy decoding composed from the reference's own kernels on its emulator, the
    way the B200 decode runs it: a prefill of a 16-token prompt, then 4 greedy steps that each
    feed one new token through every layer (dense_layer_kernel on that row only; the K and V
    rows of earlier positions are the emulator's own outputs from earlier steps, a KV cache)
    with attn_fwd_kernel over all positions so far, of which the new row is kept.  The
    embeddings, LayerNorm gain and bias, GELU, residual adds and the argmax run on the host in
    float32.  Records the prompt, the 4 greedy tokens and the logits that chose each of them;
    pins the float64 host model and the B200 decode beyond the prefill."""
    from nn_kernels import dense_layer_kernel, dense_tiles
    import attention as A
    import math
    import piton.compiler as pc
    from piton.runtime.launcher import run_emulator
    sys.path.insert(0, os.path.join(_STATE["ref"], "tests"))
    import test_reroll_reduce as RR
    from piton_b200 import tinygpt
    plen, steps, seed = 16, 4, 0
    name = f"tinygpt_emu_decode_p{plen}_n{steps}_seed{seed}"
    if exists(name):
        return
    t = time.time()
    w = tinygpt.init_weights(seed)
    prompt = tinygpt.random_prompts(1, seed=7, length=plen)[0]
    f32 = np.float32
    d, nh = tinygpt.D_MODEL, tinygpt.N_HEAD
    hd = d // nh

    def ln(v, g, b):
        rows = v.shape[0]
        sig = {"x_ptr": "*fp32", "out_ptr": "*fp32", "n": "i32", "eps": "fp32"}
        ck = pc.compile(RR.layernorm_kernel, sig, {"BLOCK": d}, grid=(rows,), num_stages=2)
        y = np.zeros_like(v)
        run_emulator(ck, (rows,), dict(x_ptr=np.ascontiguousarray(v), out_ptr=y, n=d, eps=1e-5))
        return (y * g + b).astype(f32)

    def dense(v, wm, b):
        return _run_dense(pc, run_emulator, dense_layer_kernel, dense_tiles, np.ascontiguousarray(v, f32),
                          np.ascontiguousarray(wm, f32), np.ascontiguousarray(b, f32), True, False)

    def heads(m):   # [S, 128] -> [4, S, 32]
        return np.ascontiguousarray(m.reshape(m.shape[0], nh, -1).transpose(1, 0, 2))

    def attend(q, k, v):   # all positions so far, [S, 128] each -> [S, 128]
        n = q.shape[0]
        consts = dict(HEAD_DIM=hd, BLOCK_M=2, BLOCK_N=16, CAUSAL=True, EVEN_N=n % 16 == 0,
                      **A.contiguous_strides(hd, "nd", n))
        asig = A.signature_for(consts)
        qh, kh, vh = heads(q), heads(k), heads(v)
        vals = dict(Q=qh, K=kh, V=vh, Out=np.zeros_like(qh), sm_scale=float(1 / np.sqrt(hd)), N_CTX=n,
                    stride_qh=n * hd, stride_kh=n * hd, stride_vh=n * hd, stride_oh=n * hd)
        vals = {key: val for key, val in vals.items() if key in asig}
        att = run_split(A.attn_fwd_kernel, (-(-n // 2), nh), asig, consts, vals, "Out", procs)
        return np.ascontiguousarray(att.reshape(nh, n, hd).transpose(1, 0, 2).reshape(n, d))

    cache = [{"q": np.zeros((0, d), f32), "k": np.zeros((0, d), f32), "v": np.zeros((0, d), f32)}
             for _ in range(tinygpt.N_LAYER)]

    def feed(tokens, start):
        """Feed `tokens` at positions start.. through every layer; the logits of the last one."""
        x = (w["wte"][tokens] + w["wpe"][start:start + len(tokens)]).astype(f32)
        for layer in range(tinygpt.N_LAYER):
            p = {k: w[f"h{layer}.{k}"] for k, _ in tinygpt.LAYER_TENSORS}
            c = cache[layer]
            qkv = dense(ln(x, p["ln1_g"], p["ln1_b"]), p["w_qkv"], p["b_qkv"])
            c["q"] = np.concatenate([c["q"], qkv[:, :d]])
            c["k"] = np.concatenate([c["k"], qkv[:, d:2 * d]])
            c["v"] = np.concatenate([c["v"], qkv[:, 2 * d:]])
            att = attend(c["q"], c["k"], c["v"])[start:]
            x = (x + dense(att, p["w_o"], p["b_o"])).astype(f32)
            fpre = dense(ln(x, p["ln2_g"], p["ln2_b"]), p["w_fc"], p["b_fc"]).astype(np.float64)
            gelu = (0.5 * fpre * (1.0 + np.vectorize(math.erf)(fpre / math.sqrt(2.0)))).astype(f32)
            x = (x + dense(gelu, p["w_pr"], p["b_pr"])).astype(f32)
        hf = ln(x[-1:], w["lnf_g"], w["lnf_b"])
        return dense(hf, np.ascontiguousarray(w["wte"].T), np.zeros(tinygpt.VOCAB, f32))[0]

    logits = [feed(prompt, 0)]
    tokens = []
    for step in range(steps):
        tokens.append(int(np.argmax(logits[-1])))          # first maximum, like the decode
        if step + 1 < steps:
            logits.append(feed(np.array([tokens[-1]]), plen + step))
    logits = np.stack(logits).astype(f32)
    top2 = np.sort(logits, 1)[:, -2:]
    meta = dict(op="tinygpt_decode", prompt_len=plen, new_tokens=steps, weight_seed=seed, prompt_seed=7, ref=fp,
                min_top2_margin=float((top2[:, 1] - top2[:, 0]).min()), emu_seconds=time.time() - t)
    save(name, meta, prompt=prompt.astype(np.int32), tokens=np.array(tokens, np.int32), logits=logits)


def case_idiv(fp, procs, big):
    import piton
    from primitive_kernels import idiv_kernel
    M32 = 0xFFFFFFFF
    for signed in (True, False):
        name = f"idiv_{'i32' if signed else 'u32'}"
        if exists(name):
            continue
        rng = np.random.default_rng(10 + signed)
        edges = [0, 1, 2, 3, 7, 255, 256, 0x7FFFFFFF, 0x80000000, 0xFFFFFFFF, 0x80000001, 0xFFFFFFFE]
        edges += [((1 << e) + d) & M32 for e in range(33) for d in (-1, 0, 1)]
        xe = np.array(edges, np.uint64)
        x = np.concatenate([xe, rng.integers(0, 1 << 32, 300, dtype=np.uint64)]).astype(np.uint32)
        y = np.concatenate([xe[::-1], rng.integers(0, 1 << 32, 300, dtype=np.uint64)
                            >> rng.integers(0, 32, 300).astype(np.uint64)]).astype(np.uint32)
        y[y == 0] = 1
        if signed:
            x, y = x.view(np.int32), y.view(np.int32)
        n = x.size
        q = np.zeros_like(x)
        r = np.zeros_like(x)
        t = time.time()
        idiv_kernel[(piton.cdiv(n, 64),)](x, y, q, r, n, BLOCK=64)
        save(name, dict(op="idiv", signed=signed, n=n, ref=fp, emu_seconds=time.time() - t), x=x, y=y, q=q, r=r)


def case_life(fp, procs, big):
    import piton
    import life as Lf
    for kname, shape, seed in (("tile", (13, 37), 1), ("rows", (21, 50), 2), ("bits", (9, 128), 3)):
        name = f"life_{kname}_{shape[0]}x{shape[1]}"
        if exists(name):
            continue
        rng = np.random.default_rng(seed)
        cells = (rng.random(shape) < 0.35).astype(np.int32)
        kern, _, consts, per = Lf.KERNELS[kname]
        if kname == "bits":
            words = np.packbits(cells.astype(np.uint8), axis=1, bitorder="little").view(np.uint32)
            src = np.ascontiguousarray(words)
            ncols = src.shape[1]
        else:
            src = cells.copy()
            ncols = shape[1]
        dst = np.zeros_like(src)
        t = time.time()
        if kname == "tile":
            grid = (piton.cdiv(shape[0], consts["BLOCK_R"]) * piton.cdiv(ncols, consts["BLOCK_C"]),)
        else:
            grid = (piton.cdiv(ncols, consts["BLOCK"]), piton.cdiv(shape[0], consts["ROWS"]))
        kern[grid](src, dst, shape[0], ncols, ncols, **consts)
        save(name, dict(op="life", kernel=kname, shape=list(shape), constants=consts, grid=list(grid), ref=fp,
                        emu_seconds=time.time() - t), src=src, dst=dst)


def case_elem(fp, procs, big):
    import piton
    from elementwise import mul_kernel
    from primitive_kernels import fma_kernel
    from kernels import scaled_relu_kernel
    n = 1000
    x, y = W.vector_add(n, 77)
    for name, fn in (("elem_mul", lambda o: mul_kernel[(piton.cdiv(n, 64),)](x, y, o, n, BLOCK=64)),
                     ("elem_fma", lambda o: fma_kernel[(piton.cdiv(n, 64),)](x, y, o, n, 0.3, BLOCK=64)),
                     ("elem_scaled_relu", lambda o: scaled_relu_kernel[(piton.cdiv(n, 128),)](x, o, n, 0.5,
                                                                                                BLOCK=128))):
        if exists(name):
            continue
        out = np.zeros(n, np.float32)
        fn(out)
        save(name, dict(op=name, n=n, seed=77, ref=fp), x=x, y=y, out=out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PITON_REFERENCE", ""), required=False)
    ap.add_argument("--procs", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--big", action="store_true", help="also the multi-minute configuration sizes")
    ap.add_argument("--only", default="", help="comma list of add,softmax,matmul,dense,attention,idiv,life,elem,"
                                               "tinygpt,tinygpt_decode")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(args.ref):
        sys.exit("--ref must point at a PIton checkout")
    sys.path.insert(0, args.ref)
    sys.path.insert(0, os.path.join(args.ref, "examples"))
    os.environ.setdefault("PITON_PAIR", "0")      # same bits, faster compiles (tests/test_attention.py:4-8)
    fp = ref_fingerprint(args.ref)
    _STATE["ref"] = args.ref
    only = set(filter(None, args.only.split(",")))
    for name, fn in (("add", case_add), ("softmax", case_softmax), ("matmul", case_matmul),
                     ("dense", case_dense), ("attention", case_attention), ("idiv", case_idiv), ("life", case_life),
                     ("elem", case_elem), ("tinygpt", case_tinygpt),
                     ("tinygpt_decode", case_tinygpt_decode)):
        if not only or name in only:
            fn(fp, args.procs, args.big)


if __name__ == "__main__":
    main()
