"""Sharding of the hot-path operators across the GPUs of one node.

Every operator partitions into independent pieces (matmul: row blocks of A and
C with B replicated; softmax: rows; attention: batch x head; add: element
ranges; MLP / TinyGPT: batch rows), so a rank computes its piece with no
exchange, and the only collective is the final all-gather of the output
pieces over NCCL (NVLink), which leaves the whole output on every rank.

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


def max_over_ranks(dist, value: float, device=None) -> float:
    """The maximum of a per-rank float (a timing) over all ranks."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
