"""Sharding of the hot-path operators across the GPUs of one node.

Every operator partitions into independent pieces (matmul: row blocks of A and
C with B replicated; softmax: rows; attention: batch x head; add: element
ranges; MLP / TinyGPT: batch rows), so a rank computes its piece with no
exchange, and the only collective is the final all-gather of the output
pieces over NVLink, which leaves the whole output on every rank: NCCL for most
operators, for matmul stores from the GEMM epilogue itself (NVSwitch multicast
or peer stores), and for attention peer stores from a gather warp of the
attention kernel.

Functions here are backend-agnostic (``torch.distributed`` with ``nccl`` on
GPUs or ``gloo`` on CPU), so the host-side logic is tested on CPU.
"""

from __future__ import annotations


def shard(n: int, world: int, rank: int, multiple: int = 1):
    """(start, count) of rank's equal piece of n items, piece sizes a multiple of
    `multiple`; the pieces cover ceil(n / world) rounded up, so the last may
    extend past n (the caller pads)."""
    per = -(-n // world)
    per = -(-per // multiple) * multiple
    return rank * per, per


def gather(dist, out, piece):
    """All-gather equal pieces (first dimension) into `out` on every rank."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        if out.data_ptr() != piece.data_ptr():
            out.copy_(piece)
        return out
    dist.all_gather_into_tensor(out, piece)
    return out


def batch_piece(batch, world: int, rank: int):
    """This rank's rows of a batch (numpy [n, ...]): the equal piece of ceil(n / world) rows
    starting at rank * ceil(n / world), with zero rows past the end of the batch (a zero image, a
    prompt of token 0), so that every rank runs the same shape.  Returns (piece, start)."""
    import numpy as np
    batch = np.asarray(batch)
    start, per = shard(batch.shape[0], world, rank)
    piece = np.zeros((per,) + batch.shape[1:], batch.dtype)
    mine = batch[start:start + per]
    piece[:len(mine)] = mine
    return piece, start


def run_batch_sharded(dist, fn, batch):
    """Data parallelism over independent batch rows, the sharding of the digits MLP's predict
    (examples/digits_model.py:137-139 runs every image through the same forward) and of
    batched TinyGPT decoding: each rank runs ``fn(piece)`` -> a torch tensor with one row per
    piece row on its own rows, the pieces are all-gathered and the first n rows (the whole
    batch's result, in batch order) are returned on every rank."""
    import torch
    world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
    rank = dist.get_rank() if world > 1 else 0
    n = len(batch)
    piece, _ = batch_piece(batch, world, rank)
    res = fn(piece)
    if not isinstance(res, torch.Tensor):
        res = torch.as_tensor(res)
    if res.shape[0] != piece.shape[0]:
        raise ValueError(f"fn returned {res.shape[0]} rows for a piece of {piece.shape[0]}")
    res = res.contiguous()
    out = torch.empty((res.shape[0] * world,) + tuple(res.shape[1:]), dtype=res.dtype, device=res.device)
    gather(dist, out, res)
    return out[:n]


def max_over_ranks(dist, value: float, device=None) -> float:
    """The maximum of a per-rank float (a timing) over all ranks."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class PeerOutput:
    """A full-size output buffer on every rank whose peers' copies this process
    can write: allocated with cudaMalloc (piton_b200_malloc), shared with CUDA
    IPC handles exchanged over `dist`, opened with peer access.  `peer_ptrs[r]`
    is rank r's buffer as an address valid in this process."""

    def __init__(self, dist, nbytes: int):
        import ctypes as C

        from .runtime.cuda import _lib
        lib = _lib.lib()
        self._lib = lib
        self.nbytes = nbytes
        self.world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
        self.rank = dist.get_rank() if self.world > 1 else 0
        ptr = C.c_uint64(0)
        _lib.check(lib.piton_b200_malloc(C.byref(ptr), nbytes), "malloc")
        self.ptr = ptr.value
        self.opened = []
        self.peer_ptrs = [0] * self.world
        self.peer_ptrs[self.rank] = self.ptr
        if self.world > 1:
            h = (C.c_uint8 * 64)()
            _lib.check(lib.piton_b200_ipc_handle(self.ptr, h), "ipc handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(h))
            for r, hb in enumerate(handles):
                if r == self.rank:
                    continue
                buf = (C.c_uint8 * 64).from_buffer_copy(hb)
                p = C.c_uint64(0)
                _lib.check(lib.piton_b200_ipc_open(buf, C.byref(p)), "ipc open")
                self.peer_ptrs[r] = p.value
                self.opened.append(p.value)

    def read(self, offset_bytes: int, nbytes: int):
        """Copy bytes of this rank's buffer to a new numpy uint8 array (synchronous)."""
        import ctypes as C

        import numpy as np
        out = np.empty(nbytes, np.uint8)
        from .runtime.cuda import _lib
        _lib.check(self._lib.piton_b200_memcpy_d2h(out.ctypes.data_as(C.c_void_p), self.ptr + offset_bytes, nbytes,
                                                   None), "d2h")
        _lib.check(self._lib.piton_b200_stream_wait(None, 60.0), "sync")
        return out

    def close(self):
        for p in self.opened:
            self._lib.piton_b200_ipc_close(p)
        self.opened = []
        if self.ptr:
            self._lib.piton_b200_free(self.ptr)
            self.ptr = 0


class SymmetricOutput:
    """A full-size output buffer on every rank in torch symmetric memory: the
    buffers are mapped into every rank (`peer_ptrs`) and, where the NVSwitch
    supports it, bound to one multicast address (`multicast_ptr`, else 0): a
    multimem store there is written by the switch into every rank's buffer, so
    each GPU sends its output once instead of once per peer."""

    def __init__(self, dist, nbytes: int, group=None):
        import torch
        import torch.distributed._symmetric_memory as symm
        self.nbytes = nbytes
        dev = torch.cuda.current_device()
        self.tensor = symm.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", dev))
        self.handle = symm.rendezvous(self.tensor, group if group is not None else dist.group.WORLD)
        self.world, self.rank = self.handle.world_size, self.handle.rank
        self.ptr = self.tensor.data_ptr()
        self.peer_ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.multicast_ptr = int(self.handle.multicast_ptr)

    @staticmethod
    def multicast_supported(device: int) -> bool:
        import torch
        import torch.distributed._symmetric_memory as symm
        try:
            return bool(symm._SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA, device))
        except (AttributeError, RuntimeError):
            return False

    def read(self, offset_bytes: int, nbytes: int):
        import torch
        torch.cuda.synchronize()
        return self.tensor[offset_bytes:offset_bytes + nbytes].cpu().numpy()

    def close(self):
        """Every rank calls this together: the buffers leave the multicast group only
        after all ranks are done with them."""
        if self.handle is not None:
            import torch
            torch.cuda.synchronize()
            self.handle.barrier()
            self.handle = None
            self.tensor = None


def matmul_allgather(a_piece, b, out, row_offset: int, ldc: int, stream=None, multicast: bool = True):
    """This rank's rows of C = A @ B (a_piece [m, K], b [K, N] CUDA float32 tensors),
    stored into every rank's full output by the fused all-gather epilogue: through the
    output's multicast address when it has one (and `multicast`), else with peer stores."""
    import ctypes as C

    import torch

    from .runtime.cuda import _lib
    lib = _lib.lib()
    m, K = a_piece.shape
    N = b.shape[1]
    a = _lib.MatmulArgs(a_piece.data_ptr(), b.data_ptr(), 0, m, N, K, a_piece.stride(0), a_piece.stride(1),
                        b.stride(0), b.stride(1), N, 1, 8, 64, 8, 8, -(-m // 8) * -(-N // 64), 0, 0, 0, 0)
    ws = lib.piton_b200_matmul_workspace_size(C.byref(a))
    key = (torch.cuda.current_device(), "allgather_ws")
    buf = _WS.get(key)
    if buf is None or buf.numel() < ws:
        buf = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
        _WS[key] = buf
    a.workspace, a.workspace_bytes = buf.data_ptr(), ws
    g = _lib.AllgatherArgs()
    for r, p in enumerate(out.peer_ptrs):
        g.peer_c[r] = p
    g.world, g.rank, g.row_offset, g.ldc = out.world, out.rank, row_offset, ldc
    if multicast and getattr(out, "multicast_ptr", 0):
        g.multicast_c = out.multicast_ptr
    s = stream if stream is not None else torch.cuda.current_stream()
    _lib.check(lib.piton_b200_matmul_allgather_f32(C.byref(a), C.byref(g), C.c_void_p(s.cuda_stream)),
               "matmul_allgather")


def attention_allgather(q, k, v, peer_ptrs, rank: int, head_offset: int, causal: bool = True, sm_scale=None,
                        stream=None):
    """This rank's heads of causal (or full) attention, q, k, v [heads, n_ctx, 64] contiguous
    CUDA float32 tensors, stored by the fused all-gather kernel into every rank's full output
    ([all heads, n_ctx, 64] float32) at heads [head_offset, head_offset + heads).  `peer_ptrs`:
    one device pointer per rank, valid in this process (PeerOutput.peer_ptrs), this rank's own
    output at index `rank`.  Every rank must pass a barrier before reading the outputs."""
    import ctypes as C

    import torch

    from .runtime.cuda import _lib
    lib = _lib.lib()
    heads, n, d = q.shape
    for t in (q, k, v):
        if not t.is_contiguous() or t.shape != (heads, n, d):
            raise ValueError("q, k, v must be contiguous [heads, n_ctx, head_dim] tensors")
    scale = float(sm_scale) if sm_scale is not None else 1.0 / float(d) ** 0.5
    sd = n * d
    a = _lib.AttentionArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, scale, sd, d, sd, d, 1, sd, d, sd, d, n, d,
                           64, 64, -(-n // 64), heads, 1 if causal else 0, 1 if n % 64 == 0 else 0, 0, 0, 0, 0)
    ws = lib.piton_b200_attention_workspace_size(C.byref(a))
    key = (torch.cuda.current_device(), "attn_allgather_ws")
    buf = _WS.get(key)
    if buf is None or buf.numel() < ws:
        buf = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
        _WS[key] = buf
    a.workspace, a.workspace_bytes = buf.data_ptr(), ws
    g = _lib.AllgatherArgs()
    for r, p in enumerate(peer_ptrs):
        g.peer_c[r] = p
    g.world, g.rank, g.row_offset = len(peer_ptrs), rank, head_offset
    s = stream if stream is not None else torch.cuda.current_stream()
    _lib.check(lib.piton_b200_attention_allgather_f32(C.byref(a), C.byref(g), C.c_void_p(s.cuda_stream)),
               "attention_allgather")


def softmax_allgather(x, peer_ptrs, rank: int, row_offset: int, ld: int, stream=None):
    """Row softmax of this rank's rows x ([rows, n] contiguous CUDA float32, n % 4 == 0, n <= 32768),
    stored by the fused all-gather kernel into rows [row_offset, row_offset + rows) (row stride `ld`
    floats) of every rank's full output.  `peer_ptrs`: one device pointer per rank valid in this
    process, this rank's own output at index `rank`.  Every rank must pass a barrier before
    reading the outputs."""
    import ctypes as C

    import torch

    from .runtime.cuda import _lib
    if x.dim() != 2 or not x.is_contiguous() or x.dtype != torch.float32:
        raise ValueError("x must be a contiguous float32 [rows, n_cols] tensor")
    rows, n = x.shape
    a = _lib.SoftmaxArgs(0, x.data_ptr(), n, n, n, n, rows, 0, 0)
    g = _lib.AllgatherArgs()
    for r, p in enumerate(peer_ptrs):
        g.peer_c[r] = p
    g.world, g.rank, g.row_offset, g.ldc = len(peer_ptrs), rank, row_offset, ld
    s = stream if stream is not None else torch.cuda.current_stream()
    _lib.check(_lib.lib().piton_b200_softmax_allgather_f32(C.byref(a), C.byref(g), C.c_void_p(s.cuda_stream)),
               "softmax_allgather")


def add_allgather(x, y, peer_ptrs, rank: int, offset: int, stream=None):
    """x + y for this rank's elements (contiguous CUDA float32 vectors of a multiple of 4 elements),
    stored by the fused all-gather kernel into elements [offset, offset + n) of every rank's full
    output.  Every rank must pass a barrier before reading the outputs."""
    import ctypes as C

    import torch

    from .runtime.cuda import _lib
    if x.shape != y.shape or x.dim() != 1 or not (x.is_contiguous() and y.is_contiguous()):
        raise ValueError("x and y must be contiguous float32 vectors of one length")
    n = x.numel()
    a = _lib.AddArgs(x.data_ptr(), y.data_ptr(), 0, n, 1024, -(-n // 1024), 0, 0)
    g = _lib.AllgatherArgs()
    for r, p in enumerate(peer_ptrs):
        g.peer_c[r] = p
    g.world, g.rank, g.row_offset = len(peer_ptrs), rank, offset
    s = stream if stream is not None else torch.cuda.current_stream()
    _lib.check(_lib.lib().piton_b200_add_allgather_f32(C.byref(a), C.byref(g), C.c_void_p(s.cuda_stream)),
               "add_allgather")


def allgather_pieces(piece, out, stream=None):
    """Store this rank's `piece` (a CUDA tensor) into every rank's full output `out`
    (PeerOutput or SymmetricOutput) at byte offset rank * piece.nbytes, with the library's
    peer-store all-gather (no NCCL).  Every rank must pass a barrier before reading `out`."""
    import ctypes as C

    import torch

    from .runtime.cuda import _lib
    lib = _lib.lib()
    if not piece.is_contiguous():
        raise ValueError("piece must be contiguous")
    nbytes = piece.numel() * piece.element_size()
    if (out.rank + 1) * nbytes > out.nbytes:
        raise ValueError(f"output holds {out.nbytes} bytes; rank {out.rank}'s piece ends at {(out.rank + 1) * nbytes}")
    g = _lib.AllgatherArgs()
    for r, p in enumerate(out.peer_ptrs):
        g.peer_c[r] = p
    g.world, g.rank = out.world, out.rank
    s = stream if stream is not None else torch.cuda.current_stream()
    _lib.check(lib.piton_b200_allgather(C.byref(g), piece.data_ptr(), nbytes, C.c_void_p(s.cuda_stream)), "allgather")


class HostShardedMatmul:
    """C = A @ B across the ranks with every operand in HOST memory: rank r holds its rows of
    A and of C (A_r [m, K], C_r [m, N]) and all of B [K, N].  Each call uploads A_r and only
    1/world of B's rows, completes B on every GPU with the peer-store all-gather over NVLink
    (each GPU's PCIe link carries K/world rows of B instead of all K), runs the GEMM and copies
    C_r back.  Host arrays should be page-locked (``runtime.cuda.pinned_empty``) for
    asynchronous copies; the call returns after C_r is on the host."""

    def __init__(self, dist, m: int, N: int, K: int):
        import torch
        self.dist = dist
        self.world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
        self.rank = dist.get_rank() if self.world > 1 else 0
        if K % self.world:
            raise ValueError(f"K = {K} must be a multiple of the {self.world} ranks")
        self.m, self.N, self.K = m, N, K
        self.kslice = K // self.world
        self.b_full = PeerOutput(dist, K * N * 4)
        dev = torch.cuda.current_device()
        self.b_piece = torch.empty(self.kslice * N, dtype=torch.float32, device=dev)
        self.done = torch.zeros(1, device=dev)

    def h2d_bytes(self) -> int:
        return 4 * (self.m * self.K + self.kslice * self.N)

    def d2h_bytes(self) -> int:
        return 4 * self.m * self.N

    def __call__(self, a_host, b_host, c_host):
        import ctypes as C

        import torch

        from .runtime.cuda import _lib
        lib = _lib.lib()
        s = torch.cuda.current_stream()
        if self.world > 1:
            self.dist.all_reduce(self.done)      # no rank still reads B from the previous call
        k0 = self.rank * self.kslice
        b_rows = torch.from_numpy(b_host.reshape(self.K, self.N)[k0:k0 + self.kslice].reshape(-1))
        self.b_piece.copy_(b_rows, non_blocking=True)
        allgather_pieces(self.b_piece, self.b_full, stream=s)
        if self.world > 1:
            self.dist.all_reduce(self.done)      # every rank's slice has landed in every B
        # host A and C, device-resident B: the library pipelines A's row blocks, the GEMM and C's
        M, N, K = self.m, self.N, self.K
        a = _lib.MatmulArgs(a_host.ctypes.data, self.b_full.ptr, c_host.ctypes.data, M, N, K, K, 1, N, 1, N, 1, 8,
                            64, 8, 8, -(-M // 8) * -(-N // 64), 0, 0, 0, 0)
        ws = lib.piton_b200_matmul_host_workspace_size(C.byref(a))
        if ws == 0:
            raise ValueError("the host-buffer matmul does not take this problem")
        key = (torch.cuda.current_device(), "host_sharded_ws")
        buf = _WS.get(key)
        if buf is None or buf.numel() < ws:
            buf = torch.empty(ws, dtype=torch.uint8, device="cuda")
            _WS[key] = buf
        a.workspace, a.workspace_bytes = buf.data_ptr(), ws
        _lib.check(lib.piton_b200_matmul_f32_host(C.byref(a), C.c_void_p(s.cuda_stream)), "matmul")
        s.synchronize()

    def close(self):
        self.b_full.close()


_WS = {}
