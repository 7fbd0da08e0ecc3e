"""BASELINE config 5 at its full size on one GPU: one sequence of 1,048,576
tokens of 4-bit KV (N(0,1) sources through the bit-exact quantizer, shuffled
16-token pages), 32 query heads over 4 KV heads, head_dim 64.

- the 4-bit decode (partial + combine) against the CPU oracle's
  decode_q4_partial + lse_combine over the whole context, max-abs 1e-3;
- the split-KV decode with the exchange fused in (one rank, its own mailbox)
  against the same oracle output;
- the 8-rank split of the sequence axis emulated on one GPU: partials over
  the eight rank ranges merged by the LSE combine equal the whole-context
  result (the computation an 8-GPU step performs).
The quantizer itself is checked byte for byte against the oracle on a slice
of the same pool.
"""
import os

import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import nyion_rs_b200.splitkv as S
import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
T = 1 << 20
H, N_KV, D, PT = 32, 4, 64, 16


@pytest.fixture(scope="module")
def full_case(cuda_device):
    dev = cuda_device
    gen = torch.Generator(device=dev).manual_seed(5)
    n_pages = T // PT
    pool = torch.empty(n_pages, N_KV, 2, PT, 40, dtype=torch.uint8, device=dev)
    order = torch.randperm(n_pages, device=dev, generator=gen)
    step = 4096
    first_src = None
    for p0 in range(0, n_pages, step):
        src = torch.randn(step * PT, N_KV, 2, D, device=dev, generator=gen)
        q4 = A.quantize_q4(src).reshape(step, PT, N_KV, 2, 40).permute(0, 2, 3, 1, 4)
        pool[order[p0:p0 + step]] = q4
        if first_src is None:
            first_src = (src[:2048].cpu().numpy(), A.quantize_q4(src[:2048]).cpu().numpy())
    table = order.to(torch.int32).reshape(1, n_pages)
    q = torch.randn(1, H, D, device=dev, generator=gen)
    pool_h = pool.cpu().numpy()
    table_h = table.cpu().numpy()
    ref = O.lse_combine(O.decode_q4_partial(q.cpu().numpy(), pool_h, table_h, 0, T, N_KV, D, PT,
                                            threads=os.cpu_count() or 8)[None])
    return q, pool, table, ref, first_src


def test_full_pool_quantizer_slice(full_case):
    _, _, _, _, (src, got) = full_case
    assert np.array_equal(got, O.q4_quantize_rows(src, D))


def test_config5_partial_vs_oracle(full_case):
    q, pool, table, ref, _ = full_case
    part = A.decode_q4_partial(q, pool, table, u_begin=0, u_end=T)
    out = A.lse_combine(part[None]).cpu().numpy()
    assert np.abs(out - ref).max() < TOL
    assert A.device_error() == 0


def test_config5_fused_exchange_one_rank_vs_oracle(full_case):
    q, pool, table, ref, _ = full_case
    dec = S.SplitKVDecoder(0, 1, T, mode="p2p")
    try:
        for _ in range(2):
            out = dec.step(q, pool, table).cpu().numpy()
            assert np.abs(out - ref).max() < TOL
    finally:
        dec.close()
    assert A.device_error() == 0


def test_config5_eight_rank_split_merges_to_whole(full_case):
    q, pool, table, ref, _ = full_case
    parts = torch.stack([A.decode_q4_partial(q, pool, table, u_begin=lo, u_end=hi)
                         for lo, hi in (S.rank_range(r, 8, T) for r in range(8))])
    out = A.lse_combine(parts).cpu().numpy()
    assert np.abs(out - ref).max() < TOL
    assert A.device_error() == 0
