"""GPU parity of the tensor-core chunked prefill against the CPU oracle.

The oracle restates the reference's prefill attention (executor.rs:106-138:
one ops::attention per prompt token with seq_len = position + 1) in double
precision on the same bf16 inputs; the kernel computes scores and the P.V
product as bf16 x bf16 -> f32 on tcgen05, so the bar is max-abs 2e-2.
"""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-2
D, PT = 64, 16


def _case(total, n_kv, gen, scale=0.5, extra_pages=7):
    """bf16 K/V for positions [0, total) in a shuffled 16-token page pool."""
    pages = (total + PT - 1) // PT
    n_pool = pages + extra_pages
    perm = torch.randperm(n_pool, generator=gen)[:pages].to(torch.int32)
    pool = (torch.randn(n_pool, n_kv, 2, PT, D, generator=gen) * scale).to(torch.bfloat16)
    return pool, perm


def _run(q, pool, table, q_start, dev, **kw):
    return A.prefill_paged_bf16(q.to(dev), pool.to(dev), table.to(dev), q_start, **kw).cpu().numpy()


def _oracle(q, pool, table, q_start, n_kv, scale=None):
    return O.prefill_paged_bf16(q.view(torch.uint16).numpy(), pool.view(torch.uint16).numpy(),
                                table.numpy(), q_start, n_kv, D, PT, scale=scale, threads=16)


@pytest.mark.parametrize("q_start,n_q,n_kv", [(0, 1, 1), (0, 16, 1), (0, 37, 4), (100, 200, 4),
                                              (13, 130, 2), (0, 300, 8), (255, 1, 4)])
def test_prefill_vs_oracle(cuda_device, q_start, n_q, n_kv):
    g = torch.Generator().manual_seed(q_start * 1000 + n_q + n_kv)
    pool, table = _case(q_start + n_q, n_kv, g)
    q = (torch.randn(n_q, n_kv * 8, D, generator=g) * 0.5).to(torch.bfloat16)
    got = _run(q, pool, table, q_start, cuda_device)
    ref = _oracle(q, pool, table, q_start, n_kv)
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() < TOL
    assert A.device_error() == 0


def test_prefill_scale_argument(cuda_device):
    g = torch.Generator().manual_seed(9)
    pool, table = _case(300, 4, g, scale=1.0)
    q = torch.randn(300, 32, D, generator=g).to(torch.bfloat16)
    got = _run(q, pool, table, 0, cuda_device, scale=0.05)
    ref = _oracle(q, pool, table, 0, 4, scale=0.05)
    assert np.abs(got - ref).max() < TOL


def test_prefill_nan_in_unwritten_slots(cuda_device):
    """Slots past the context in the last page hold NaN: they are never mixed in."""
    g = torch.Generator().manual_seed(10)
    pool, table = _case(200, 4, g)
    last = int(table[(200 - 1) // PT])
    pool[last, :, :, 200 % PT:] = float("nan")
    q = (torch.randn(200, 32, D, generator=g) * 0.5).to(torch.bfloat16)
    got = _run(q, pool, table, 0, cuda_device)
    ref = _oracle(q, pool, table, 0, 4)
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() < TOL


def test_config4_chunks(cuda_device):
    """2048 prompt tokens in 4 chunks of 512 against the growing paged cache
    (32 query heads, 4 KV heads, head_dim 64, N(0,1)*0.5)."""
    g = torch.Generator().manual_seed(4)
    T, CH, n_kv = 2048, 512, 4
    pool, table = _case(T, n_kv, g)
    q = (torch.randn(T, 32, D, generator=g) * 0.5).to(torch.bfloat16)
    dev_pool = torch.zeros_like(pool, device=cuda_device)
    dev_table = table.to(cuda_device)
    outs = []
    for c in range(T // CH):
        lo, hi = c * CH, (c + 1) * CH
        # the chunk's K/V are stored before its attention, as in the reference
        for pidx in range(lo // PT, hi // PT):
            p = int(table[pidx])
            dev_pool[p] = pool[p].to(cuda_device)
        outs.append(A.prefill_paged_bf16(q[lo:hi].to(cuda_device), dev_pool, dev_table, lo).cpu())
    got = torch.cat(outs).numpy()
    ref = _oracle(q, pool, table, 0, n_kv)
    assert np.abs(got - ref).max() < TOL
    assert A.device_error() == 0


def test_prefill_bad_page_id_sets_device_error(cuda_device):
    g = torch.Generator().manual_seed(11)
    pool, table = _case(100, 4, g)
    table[3] = pool.shape[0] + 5
    q = (torch.randn(100, 32, D, generator=g) * 0.5).to(torch.bfloat16)
    A.device_error()
    _run(q, pool, table, 0, cuda_device)
    assert A.device_error() & 1


def test_prefill_rejects_unsupported(cuda_device):
    pool = torch.zeros(4, 4, 2, PT, D, dtype=torch.bfloat16, device=cuda_device)
    table = torch.arange(4, dtype=torch.int32, device=cuda_device)
    q = torch.zeros(10, 64, D, dtype=torch.bfloat16, device=cuda_device)   # group 16
    with pytest.raises(A.NyionError):
        A.prefill_paged_bf16(q, pool, table, 0)
    q = torch.zeros(100, 32, D, dtype=torch.bfloat16, device=cuda_device)  # context > table
    with pytest.raises(A.NyionError):
        A.prefill_paged_bf16(q, pool, table, 0)
