"""The allocation-free decode entry point (nyion_attn_decode_paged_f32_noalloc).

Some callers cannot allocate device memory while they decode — a serving loop
that must not stall on cudaFree's device synchronisation, a host whose HBM is
fully owned by its own arena, a plugin host that forbids library allocations.
This variant keeps its split-KV scratch in a fixed device array inside the
library.  The test calls it through the C ABI twice in a row and checks both
results against the workspace-taking entry point (same tolerance as the other
decode tests), that 512 sequences of 4 KV heads (the whole-page kernel) fit,
and that an oversized call (8 KV heads, other kernel) is refused with an
error.  It lives in its own file so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A

pytestmark = pytest.mark.gpu
TOL = 1e-3
H, N_KV, D, PT = 32, 4, 64, 16


def _noalloc():
    f = A.lib().nyion_attn_decode_paged_f32_noalloc
    vp, i32, i64 = C.c_void_p, C.c_int32, C.c_int64
    f.restype = i32
    f.argtypes = [vp, vp, i64, vp, i32, vp, vp, i32, i32, i32, i32, i32, C.c_float, vp]
    return f


def _case(lens, max_pages, seed, dev, n_kv=N_KV):
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    n_pages = B * max_pages + 3
    pool = torch.randn(n_pages, n_kv, 2, PT, D, generator=g).to(dev)
    table = torch.randperm(n_pages, generator=g)[: B * max_pages].to(torch.int32).reshape(B, max_pages).to(dev)
    q = torch.randn(B, n_kv * 8, D, generator=g).to(dev)
    lt = torch.tensor(lens, dtype=torch.int32).to(dev)
    return q, pool, table, lt


def test_noalloc_matches_workspace_entry_twice(cuda_device):
    lens = [4096, 1, 700, 0, 33, 2048, 4000, 16] * 4       # 32 sequences, ragged
    q, pool, table, lt = _case(lens, 256, seed=11, dev=cuda_device)
    ref = A.decode_paged_f32(q, pool, table, lt, workspace=A.Workspace(len(lens), N_KV, H, D)).cpu().numpy()
    f = _noalloc()
    s = torch.cuda.current_stream()
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc = f(q.data_ptr(), pool.data_ptr(), pool.shape[0], table.data_ptr(), table.shape[1],
               lt.data_ptr(), out.data_ptr(), len(lens), H, N_KV, D, PT, 0.0, s.cuda_stream)
        assert rc == 0, A.last_error()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() < TOL


def test_noalloc_full_batch_with_four_kv_heads(cuda_device):
    lens = [64, 17, 1, 40] * 128                            # 512 sequences x 4 KV heads
    q, pool, table, lt = _case(lens, 4, seed=13, dev=cuda_device)
    ref = A.decode_paged_f32(q, pool, table, lt, workspace=A.Workspace(len(lens), N_KV, H, D)).cpu().numpy()
    out = torch.full_like(q, float("nan"))
    rc = _noalloc()(q.data_ptr(), pool.data_ptr(), pool.shape[0], table.data_ptr(), table.shape[1],
                    lt.data_ptr(), out.data_ptr(), len(lens), H, N_KV, D, PT, 0.0,
                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0, A.last_error()
    assert np.abs(out.cpu().numpy() - ref).max() < TOL


def test_noalloc_refuses_oversized_call(cuda_device):
    lens = [64] * 512                                       # 4096 (sequence, KV head) pairs
    q, pool, table, lt = _case(lens, 4, seed=12, dev=cuda_device, n_kv=8)
    out = torch.zeros_like(q)
    rc = _noalloc()(q.data_ptr(), pool.data_ptr(), pool.shape[0], table.data_ptr(), table.shape[1],
                    lt.data_ptr(), out.data_ptr(), len(lens), 64, 8, D, PT, 0.0,
                    torch.cuda.current_stream().cuda_stream)
    assert rc == -5 and "scratch" in A.last_error()
    assert torch.count_nonzero(out).item() == 0
