"""The allocation-free decode entry point (nyion_attn_decode_paged_f32_noalloc).

Some callers cannot allocate device memory while they decode — a serving loop
that must not stall on cudaFree's device synchronisation, a host whose HBM is
fully owned by its own arena, a plugin host that forbids library allocations.
This variant keeps its split-KV scratch in a fixed device array inside the
library.  The test calls it through the C ABI twice in a row and checks both
results against the workspace-taking entry point (same tolerance as the other
decode tests), that 512 sequences of 4 KV heads (the whole-page kernel) fit,
that 8 KV heads (the general kernel on the same scratch) match the CPU oracle
on two calls in a row, that an out-of-range page id is reported through
nyion_attn_device_error (and cleared by it), and that an oversized call is
refused with an error.  It lives in its own file so that pytest collects it
last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

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


def _call(q, pool, table, lt, out, n_heads, n_kv):
    return _noalloc()(q.data_ptr(), pool.data_ptr(), pool.shape[0], table.data_ptr(), table.shape[1],
                      lt.data_ptr(), out.data_ptr(), q.shape[0], n_heads, n_kv, D, PT, 0.0,
                      torch.cuda.current_stream().cuda_stream)


def test_noalloc_eight_kv_heads_vs_oracle(cuda_device):
    """8 KV heads take the general kernel on the static scratch (not the
    whole-page kernel): checked against the CPU oracle, two calls in a row."""
    lens = [700, 1, 0, 129, 2048, 16, 33, 1000] * 4        # 32 sequences x 8 KV heads
    q, pool, table, lt = _case(lens, 128, seed=17, dev=cuda_device, n_kv=8)
    ref = O.decode_paged_f32(q.cpu().numpy(), pool.cpu().numpy(), table.cpu().numpy(),
                             np.array(lens, np.int32), 8, D, PT, threads=8)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        assert _call(q, pool, table, lt, out, 64, 8) == 0, A.last_error()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() < TOL
    assert A.device_error() == 0


@pytest.mark.parametrize("n_kv", [4, 8])
def test_noalloc_page_error_reported(cuda_device, n_kv):
    """A page id past the pool is skipped and reported by nyion_attn_device_error,
    which clears it; the other sequences are unaffected."""
    A.device_error()                                        # start from a clear word
    lens = [300, 64, 500, 17]
    q, pool, table, lt = _case(lens, 32, seed=19, dev=cuda_device, n_kv=n_kv)
    bad = table.clone()
    bad[2, 3] = pool.shape[0] + 5
    ref = O.decode_paged_f32(q.cpu().numpy(), pool.cpu().numpy(), table.cpu().numpy(),
                             np.array(lens, np.int32), n_kv, D, PT, threads=4)
    out = torch.full_like(q, float("nan"))
    assert _call(q, pool, bad, lt, out, n_kv * 8, n_kv) == 0, A.last_error()
    assert A.device_error() & 1
    assert A.device_error() == 0
    got = out.cpu().numpy()
    keep = [0, 1, 3]
    assert np.abs(got[keep] - ref[keep]).max() < TOL


def test_noalloc_refuses_oversized_call(cuda_device):
    lens = [64] * 512                                       # 4096 (sequence, KV head) pairs
    q, pool, table, lt = _case(lens, 4, seed=12, dev=cuda_device, n_kv=8)
    out = torch.zeros_like(q)
    rc = _noalloc()(q.data_ptr(), pool.data_ptr(), pool.shape[0], table.data_ptr(), table.shape[1],
                    lt.data_ptr(), out.data_ptr(), len(lens), 64, 8, D, PT, 0.0,
                    torch.cuda.current_stream().cuda_stream)
    assert rc == -5 and "scratch" in A.last_error()
    assert torch.count_nonzero(out).item() == 0
