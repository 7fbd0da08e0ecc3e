"""Split-KV decode across GPUs: the multi-GPU path of the 4-bit long-context decode.

The sequence axis is cut into contiguous, chunk-aligned token ranges, one per
rank (each rank's KV arena holds only its pages).  Every rank computes a
log-sum-exp partial (o/l, m, l) per (sequence, query head) over its range
with nyion_attn_decode_q4_partial, the partials are exchanged with one
all-gather (NCCL over NVLink on GPUs, gloo in the CPU tests), and every rank
merges them with nyion_attn_lse_combine.  There is no such path in the
reference (its long contexts rely on sparsity and an NVMe tier); the merge is
the same log-sum-exp identity the reference's Mojo kernel uses inside one
device (swamp-gpu/kernels/attention.mojo:89-96).
"""
from __future__ import annotations

from dataclasses import dataclass

CHUNK = 64   # token alignment of a rank's range (the Q4 kernel's stage)


def rank_range(rank: int, world: int, total_tokens: int, align: int = CHUNK) -> tuple[int, int]:
    """Even partition of [0, total_tokens) into `world` contiguous ranges whose
    interior boundaries are multiples of `align`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    units = (total_tokens + align - 1) // align
    lo_u = units * rank // world
    hi_u = units * (rank + 1) // world
    return min(lo_u * align, total_tokens), min(hi_u * align, total_tokens)


def exchange(partial, group=None):
    """All-gather this rank's partial [B, H, D+2] into [world, B, H, D+2]."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return partial.unsqueeze(0)
    b = partial.shape[0]
    out = torch.empty((world * b,) + tuple(partial.shape[1:]), dtype=partial.dtype, device=partial.device)
    dist.all_gather_into_tensor(out, partial.contiguous(), group=group)
    return out.view((world, b) + tuple(partial.shape[1:]))


@dataclass
class SplitKVDecoder:
    """One rank's share of a split-KV decode over `total_tokens` tokens.

    `pool` / `page_table` hold this rank's pages at absolute page indices
    (entries outside the rank's range are never read).
    """
    rank: int
    world: int
    total_tokens: int
    batch: int = 1
    n_heads: int = 32
    head_dim: int = 64
    group: object = None

    def __post_init__(self):
        self.lo, self.hi = rank_range(self.rank, self.world, self.total_tokens)
        self._ws = None
        self._part = None
        self._out = None

    def step(self, q, pool, page_table, stream=None):
        """Partial over [lo, hi), all-gather, combine; returns out [B, H, D] on every rank."""
        import torch
        from . import attn as A
        if self._ws is None:
            self._ws = A.Q4Workspace(self.batch, device=q.device)
            self._part = torch.empty(self.batch, self.n_heads, self.head_dim + 2, device=q.device)
            self._out = torch.empty(self.batch, self.n_heads, self.head_dim, device=q.device)
        A.decode_q4_partial(q, pool, page_table, u_begin=self.lo, u_end=self.hi, part=self._part,
                            workspace=self._ws, stream=stream)
        parts = exchange(self._part, self.group)
        return A.lse_combine(parts, out=self._out, stream=stream)
