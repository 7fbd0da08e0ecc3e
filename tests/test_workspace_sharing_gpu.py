"""Library-owned workspaces shared across entry points and batch sizes.

The fp32 paged decode keeps merge counters at the start of its workspace and
relies on them reading zero.  Calls that pass no workspace share the
library's buffers, so this runs, in one process: fp32 decode at batch 600
(two launches of at most 512 sequences), the position kernel (whose partials
use the scratch buffer), fp32 decode at batch 3, then batch 600 again, and
checks every result against the oracle (max-abs 1e-3).
"""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
N_KV, D, PT, H = 4, 64, 16, 32


def _f32_case(rng, B, max_len):
    lens = rng.integers(1, max_len + 1, B).astype(np.int32)
    mp = (max_len + PT - 1) // PT
    pool = rng.standard_normal((B * mp, N_KV, 2, PT, D), dtype=np.float32)
    table = rng.permutation(B * mp).astype(np.int32).reshape(B, mp)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    return q, pool, table, lens


def _run_f32(dev, case):
    q, pool, table, lens = case
    got = A.decode_paged_f32(*(torch.from_numpy(x).to(dev) for x in (q, pool, table, lens)))
    torch.cuda.synchronize()
    want = O.decode_paged_f32(q, pool, table, lens, N_KV, D, PT, threads=8)
    return np.abs(got.cpu().numpy() - want).max()


def test_internal_workspaces_across_entries_and_batches(cuda_device):
    rng = np.random.default_rng(77)
    big = _f32_case(rng, 600, 48)
    small = _f32_case(rng, 3, 3000)
    A.device_error()
    assert _run_f32(cuda_device, big) < 1e-3
    # the position kernel writes its partials at the start of its own buffer
    T = 700
    pool = rng.standard_normal((T // PT + 1, N_KV, 2, PT, D), dtype=np.float32)
    table = np.arange(T // PT + 1, dtype=np.int32)[None]
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    pos = rng.integers(0, T, (1, 600)).astype(np.int32)
    got = A.decode_positions(*(torch.from_numpy(x).to(cuda_device) for x in (q, pool, table, pos)),
                             torch.tensor([600], dtype=torch.int32, device=cuda_device))
    torch.cuda.synchronize()
    g = pool[pos[0] // PT, :, :, pos[0] % PT]                 # [600][n_kv][2][D]
    flat = np.zeros(((600 + PT - 1) // PT, N_KV, 2, PT, D), np.float32)
    for j in range(600):
        flat[j // PT, :, :, j % PT] = g[j]
    want = O.decode_paged_f32(q, flat, np.arange(flat.shape[0], dtype=np.int32)[None],
                              np.array([600], np.int32), N_KV, D, PT, threads=8)
    assert np.abs(got.cpu().numpy() - want).max() < 1e-3
    assert _run_f32(cuda_device, small) < 1e-3
    assert _run_f32(cuda_device, big) < 1e-3
    assert _run_f32(cuda_device, small) < 1e-3
    assert A.device_error() == 0
