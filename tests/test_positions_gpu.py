"""GPU parity of position-list attention (ops::attention_sparse /
attention_fugu position sets, swamp-engine/src/ops.rs:85-168, 445-541) and
of ops::attention_sparse_q4 (ops.rs:597-723) against the CPU oracle.

* explicit lists over f32 and Q4 pools: the oracle is the contiguous decode
  over the listed rows gathered in list order (duplicates kept), which is
  what the reference's score / softmax / weighted-sum loops compute;
* attention_sparse_q4: oracle.attention_sparse_q4 on a ZonedPages store
  filled with the same tokens (writer-consistent nibble order), and the
  position kernel on oracle.sparse_positions' list;
* edges: empty lists, lists spanning several 128-position splits, ragged
  batches, shuffled page tables, a page-table hole (skipped, page-range bit).
Tolerance: max-abs 1e-3 (fp32 and 4-bit KV).
"""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
N_KV, D, PT, H = 4, 64, 16, 32


def _pool(src, fmt, rng, extra_pages=3):
    """src [B][T][n_kv][2][D] f32 -> (pool, table, per-token rows) with shuffled pages."""
    B, T = src.shape[:2]
    mp = (T + PT - 1) // PT
    n_pages = B * mp + extra_pages
    perm = rng.permutation(n_pages)[: B * mp].astype(np.int32).reshape(B, mp)
    if fmt == "q4":
        rows = O.q4_quantize_rows(src, D)                     # [B][T][n_kv][2][40]
        pool = np.zeros((n_pages, N_KV, 2, PT, 40), np.uint8)
    else:
        rows = src
        pool = np.zeros((n_pages, N_KV, 2, PT, D), np.float32)
    for b in range(B):
        for t in range(T):
            pool[perm[b, t // PT], :, :, t % PT] = rows[b, t]
    return pool, perm, rows


def _oracle_gathered(q, rows, pos_lists, fmt):
    """Contiguous oracle over rows[b][pos_lists[b]] in list order."""
    B = q.shape[0]
    out = np.zeros((B, H, D), np.float32)
    for b in range(B):
        idx = np.asarray(pos_lists[b], np.int64)
        n = len(idx)
        if n == 0:
            continue
        g = rows[b, idx]                                      # [n][n_kv][2][..]
        mp = (n + PT - 1) // PT
        shape = (mp, N_KV, 2, PT) + g.shape[3:]
        pool = np.zeros(shape, g.dtype)
        for j in range(n):
            pool[j // PT, :, :, j % PT] = g[j]
        table = np.arange(mp, dtype=np.int32)[None]
        if fmt == "q4":
            part = O.decode_q4_partial(q[b:b + 1], pool, table, 0, n, N_KV, D, PT, threads=8)
            out[b] = O.lse_combine(part[None])[0]
        else:
            out[b] = O.decode_paged_f32(q[b:b + 1], pool, table, np.array([n], np.int32), N_KV, D, PT,
                                        threads=8)[0]
    return out


def _lists(rng, B, T, sizes):
    lists = []
    for b in range(B):
        n = sizes[b % len(sizes)]
        lists.append(rng.integers(0, T, n).astype(np.int32))   # duplicates allowed
    return lists


def _pack(lists):
    mx = max(1, max(len(x) for x in lists))
    arr = np.zeros((len(lists), mx), np.int32)
    for b, x in enumerate(lists):
        arr[b, : len(x)] = x
    return arr, np.array([len(x) for x in lists], np.int32)


@pytest.mark.parametrize("fmt", ["f32", "q4"])
@pytest.mark.parametrize("B,T,sizes", [(1, 300, [37]), (3, 2000, [700, 0, 129]), (2, 5000, [1024, 257])])
def test_explicit_positions(cuda_device, fmt, B, T, sizes):
    rng = np.random.default_rng(B * 1000 + T + (fmt == "q4"))
    src = rng.standard_normal((B, T, N_KV, 2, D), dtype=np.float32)
    pool, table, rows = _pool(src, fmt, rng)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    lists = _lists(rng, B, T, sizes)
    pos, npos = _pack(lists)
    dev = cuda_device
    A.device_error()
    got = A.decode_positions(torch.from_numpy(q).to(dev), torch.from_numpy(pool).to(dev),
                             torch.from_numpy(table).to(dev), torch.from_numpy(pos).to(dev),
                             torch.from_numpy(npos).to(dev))
    torch.cuda.synchronize()
    want = _oracle_gathered(q, rows, lists, fmt)
    assert np.abs(got.cpu().numpy() - want).max() < TOL
    for b, x in enumerate(lists):
        if len(x) == 0:
            assert not got[b].abs().any()
    assert A.device_error() == 0


def test_positions_with_workspace_and_stream(cuda_device):
    rng = np.random.default_rng(5)
    B, T = 2, 900
    src = rng.standard_normal((B, T, N_KV, 2, D), dtype=np.float32)
    pool, table, rows = _pool(src, "f32", rng)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    lists = _lists(rng, B, T, [600, 300])
    pos, npos = _pack(lists)
    dev = cuda_device
    ws = A.positions_workspace(B, H, pos.shape[1], device=dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        args = [torch.from_numpy(x).to(dev) for x in (q, pool, table, pos, npos)]
        got = A.decode_positions(*args, workspace=ws, stream=s)
    s.synchronize()
    assert np.abs(got.cpu().numpy() - _oracle_gathered(q, rows, lists, "f32")).max() < TOL
    with pytest.raises(A.NyionError):
        A.decode_positions(*args, workspace=A.RawWorkspace(16, device=dev))


def test_page_hole_is_skipped_and_reported(cuda_device):
    rng = np.random.default_rng(9)
    T = 200
    src = rng.standard_normal((1, T, N_KV, 2, D), dtype=np.float32)
    pool, table, rows = _pool(src, "f32", rng)
    table[0, 3] = -1                                          # tokens 48..63 unmapped
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    lst = np.array([5, 50, 60, 100, 199], np.int32)
    dev = cuda_device
    A.device_error()
    got = A.decode_positions(torch.from_numpy(q).to(dev), torch.from_numpy(pool).to(dev),
                             torch.from_numpy(table).to(dev), torch.from_numpy(lst[None]).to(dev),
                             torch.tensor([5], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert A.device_error() & 1                               # page-range bit
    want = _oracle_gathered(q, rows, [np.array([5, 100, 199])], "f32")
    assert np.abs(got.cpu().numpy() - want).max() < TOL


def _zoned_and_pool(rng, T):
    """The same tokens in a reference-layout ZonedPages store and a 16-token Q4 pool."""
    src = rng.standard_normal((1, T, N_KV, 2, D), dtype=np.float32)
    zp = O.ZonedPages(1, N_KV, D, T + 64)
    for t in range(T):
        zp.save(0, t, src[0, t, :, 0], src[0, t, :, 1])
    pool, table, rows = _pool(src, "q4", rng)
    return zp, pool, table, rows


@pytest.mark.parametrize("T,q_pos,window,stride", [
    (100, 99, 512, 64),          # whole sequence inside the window: no global tokens
    (3000, 2999, 1024, 64),      # window + 30 global tokens
    (12000, 11999, 2048, 64),    # 155 candidates, capped at 128
    (5000, 3000, 1000, 7),       # q_pos inside the sequence, odd stride
    (4100, 4099, 4097, 64),      # valid_end - window == 2
])
def test_sparse_q4_matches_reference_rule(cuda_device, T, q_pos, window, stride):
    rng = np.random.default_rng(T + window + stride)
    zp, pool, table, rows = _zoned_and_pool(rng, T)
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    want = O.attention_sparse_q4(zp, q[0], 0, T, q_pos, H, window, stride, as_written=False)
    valid_end = min(q_pos, T - 1)
    dev = cuda_device
    dq, dp, dt = (torch.from_numpy(x).to(dev) for x in (q, pool, table))
    lens = torch.tensor([valid_end + 1], dtype=torch.int32, device=dev)
    A.device_error()
    got = A.sparse_q4(dq, dp, dt, lens, window, stride)
    torch.cuda.synchronize()
    assert np.abs(got[0].cpu().numpy() - want).max() < TOL
    # the same set through the explicit-list kernel
    lst = O.sparse_positions(T, q_pos, window, stride).astype(np.int32)
    got2 = A.decode_positions(dq, dp, dt, torch.from_numpy(lst[None]).to(dev),
                              torch.tensor([len(lst)], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert np.abs(got2[0].cpu().numpy() - want).max() < TOL
    assert A.device_error() == 0


def test_sparse_q4_batch_and_workspace(cuda_device):
    rng = np.random.default_rng(31)
    B, T = 3, 6000
    src = rng.standard_normal((B, T, N_KV, 2, D), dtype=np.float32)
    pool, table, rows = _pool(src, "q4", rng)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    lens = np.array([6000, 1, 2500], np.int32)
    window, stride = 1500, 32
    dev = cuda_device
    ws = A.sparse_q4_workspace(B, H, device=dev)
    args = [torch.from_numpy(x).to(dev) for x in (q, pool, table, lens)]
    for _ in range(2):                                        # workspace reuse
        got = A.sparse_q4(*args, window, stride, workspace=ws)
        torch.cuda.synchronize()
    lists = [O.sparse_positions(int(L), int(L) - 1, window, stride) for L in lens]
    want = _oracle_gathered(q, rows, lists, "q4")
    assert np.abs(got.cpu().numpy() - want).max() < TOL
    assert A.device_error() == 0
