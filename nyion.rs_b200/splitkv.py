"""Split-KV decode across GPUs: the multi-GPU path of the 4-bit long-context decode.

The sequence axis is cut into contiguous, chunk-aligned token ranges, one per
rank (each rank's KV arena holds only its pages).  Every rank computes a
log-sum-exp partial (o/l, m, l) per (sequence, query head) over its range and
the ranks' partials are merged on every rank.  Two exchanges:

  * "p2p" (the GPU path): nyion_attn_decode_q4_splitkv's decode launch
    writes each rank's merged rows straight into every rank's mailbox over
    peer memory (NVLink), and a second small kernel waits for the ranks' rows
    and combines them: no collective call.  The mailboxes are opened once
    through CUDA IPC handles exchanged with torch.distributed.
  * "collective": nyion_attn_decode_q4_partial, one all-gather (NCCL on GPUs,
    gloo in the CPU tests), nyion_attn_lse_combine — the library-collective
    baseline, and the host logic the CPU tests exercise.

There is no such path in the reference (its long contexts rely on sparsity
and an NVMe tier); the merge is the same log-sum-exp identity the reference's
Mojo kernel uses inside one device (swamp-gpu/kernels/attention.mojo:89-96).
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
    (entries outside the rank's range are never read).  mode "p2p" needs one
    GPU per rank on one node (CUDA IPC); "collective" works with any backend.
    """
    rank: int
    world: int
    total_tokens: int
    batch: int = 1
    n_heads: int = 32
    head_dim: int = 64
    group: object = None
    mode: str = "p2p"
    timeout_ms: int = 2000

    @property
    def launches_per_step(self) -> int:
        """Kernels one p2p step launches on each rank: the decode (whose merging
        CTAs send the rank's rows to every rank) and, with more than one rank,
        the exchange kernel that waits for the ranks' rows and combines them."""
        return 1 if self.world == 1 else 2

    def __post_init__(self):
        self.lo, self.hi = rank_range(self.rank, self.world, self.total_tokens)
        self._ws = None
        self._part = None
        self._out = None
        self._mbox = None
        self._peers = None

    def _setup(self, device):
        import torch
        from . import attn as A
        self._ws = A.Q4Workspace(self.batch, device=device)
        self._part = torch.empty(self.batch, self.n_heads, self.head_dim + 2, device=device)
        self._out = torch.empty(self.batch, self.n_heads, self.head_dim, device=device)
        if self.mode == "p2p":
            self._mbox = A.Mailbox(self.batch, self.n_heads)
            handles = [None] * self.world
            if self.world > 1:
                import torch.distributed as dist
                dist.all_gather_object(handles, self._mbox.ipc_handle(), group=self.group)
            self._peers = [self._mbox.ptr if r == self.rank else A.ipc_open(handles[r])
                           for r in range(self.world)]
            if self.world > 1:
                import torch.distributed as dist
                torch.cuda.synchronize()
                dist.barrier(group=self.group)    # every mailbox exists and is zeroed

    def step(self, q, pool, page_table, stream=None):
        """Partial over [lo, hi), exchange, combine; returns out [B, H, D] on every rank."""
        from . import attn as A
        if self._ws is None:
            self._setup(q.device)
        if self.mode == "p2p":
            return A.decode_q4_splitkv(q, pool, page_table, self.lo, self.hi, self._peers, self.rank,
                                       out=self._out, timeout_ms=self.timeout_ms, workspace=self._ws,
                                       stream=stream)
        import contextlib
        import torch
        A.decode_q4_partial(q, pool, page_table, u_begin=self.lo, u_end=self.hi, part=self._part,
                            workspace=self._ws, stream=stream)
        # the collective runs on torch's current stream: make it the caller's
        with torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext():
            parts = exchange(self._part, self.group)
            return A.lse_combine(parts, out=self._out, stream=stream)

    def close(self):
        """Unmap the peers' mailboxes and free this rank's (every rank calls it
        after its last step; a barrier keeps peers from writing into freed memory)."""
        if self._mbox is None:
            return
        import torch
        from . import attn as A
        torch.cuda.synchronize()
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)
        for r, ptr in enumerate(self._peers):
            if r != self.rank:
                A.ipc_close(ptr)
        self._mbox.free()
        self._mbox = None
