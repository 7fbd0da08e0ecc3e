"""The HBM arena (nyion_attn_arena_*), the device side of the reference's
HeterogeneousMemoryAllocator (swamp-tensors/src/hma.rs:215-265), through the C
ABI: KV page pools, page tables, queries and outputs carved from one
reservation feed the fp32 and 4-bit decodes (checked against the CPU oracle);
freed blocks coalesce; a request larger than any free range and an unknown
handle are refused; a unified (managed) allocation is written from the host
and read by a kernel."""
import ctypes as C

import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
H, N_KV, D, PT = 32, 4, 64, 16
TOL = 1e-3


def _put(ar, arr):
    arr = np.ascontiguousarray(arr)
    h, p = ar.allocate(arr.nbytes)
    ar.upload(h, arr)
    return h, p


def test_decode_from_arena_blocks(cuda_device):
    rng = np.random.default_rng(5)
    lens = np.array([700, 1, 333, 64], np.int32)
    B, mp = len(lens), 44
    n_pages = B * mp + 3
    pool = rng.standard_normal((n_pages, N_KV, 2, PT, D), dtype=np.float32)
    table = rng.permutation(n_pages)[: B * mp].astype(np.int32).reshape(B, mp)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    ar = A.Arena(64 << 20)
    try:
        hp, pp = _put(ar, pool)
        ht, pt = _put(ar, table)
        hq, pq = _put(ar, q)
        hl, pl = _put(ar, lens)
        ho, po = ar.allocate(q.nbytes)
        assert all(x % 256 == 0 for x in (pp, pt, pq, pl, po))
        L = A.lib()
        st = L.nyion_attn_decode_paged_f32(pq, pp, n_pages, pt, mp, pl, po, B, H, N_KV, D, PT, 0.0, None, 0, None)
        assert st == 0, A.last_error()
        torch.cuda.synchronize()
        out = np.empty_like(q)
        ar.download(ho, out)
        ref = O.decode_paged_f32(q, pool, table, lens, N_KV, D, PT, threads=4)
        assert np.abs(out - ref).max() < TOL
        cap, used, free = ar.info()
        assert used == sum((x + 255) // 256 * 256 for x in (pool.nbytes, table.nbytes, q.nbytes, lens.nbytes, q.nbytes))
        assert cap == 64 << 20 and free == cap - used
    finally:
        ar.close()
    assert A.device_error() == 0


def test_q4_decode_from_arena(cuda_device):
    rng = np.random.default_rng(6)
    T = 1500
    src = rng.standard_normal((T, N_KV, 2, D), dtype=np.float32)
    q4 = O.q4_quantize_rows(src, D)
    mp = (T + PT - 1) // PT
    pool = np.zeros((mp, N_KV, 2, PT, 40), np.uint8)
    for t in range(T):
        pool[t // PT, :, :, t % PT] = q4[t]
    table = np.arange(mp, dtype=np.int32)[None]
    q = rng.standard_normal((1, H, D), dtype=np.float32)
    ar = A.Arena(32 << 20)
    try:
        _, pp = _put(ar, pool)
        _, pt = _put(ar, table)
        _, pq = _put(ar, q)
        hpart, ppart = ar.allocate(H * (D + 2) * 4)
        st = A.lib().nyion_attn_decode_q4_partial(pq, pp, mp, pt, mp, None, None, 0, T, ppart, 1, H, N_KV, D, PT,
                                                  0.0, None, 0, None)
        assert st == 0, A.last_error()
        torch.cuda.synchronize()
        part = np.empty((1, H, D + 2), np.float32)
        ar.download(hpart, part)
        ref = O.decode_q4_partial(q, pool, table, 0, T, N_KV, D, PT, threads=4)
        assert np.abs(part[0, :, :D] - ref[0, :, :D]).max() < TOL
    finally:
        ar.close()


def test_free_coalesces_and_refusals(cuda_device):
    ar = A.Arena(1 << 20)
    try:
        ha, pa = ar.allocate(1000)                 # 1024 bytes taken
        hb, pb = ar.allocate(300000)
        hc, pc = ar.allocate(5000)
        assert pb == pa + 1024 and pc == pb + 300032
        ar.free(hb)
        ar.free(ha)                                # coalesces with b's range
        hd, pd = ar.allocate(1024 + 300032)        # exactly the merged range (best fit)
        assert pd == pa
        with pytest.raises(A.NyionError) as e:
            ar.allocate(2 << 20)                   # larger than any free range
        assert e.value.status == -5
        with pytest.raises(A.NyionError) as e:
            ar.free(12345)
        assert e.value.status == -1
        ar.free(hd)
        ar.free(hc)
        cap, used, free = ar.info()
        assert used == 0 and free == cap           # everything coalesced back
    finally:
        ar.close()


def test_unified_allocation_written_from_host(cuda_device):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((4, D), dtype=np.float32)
    ar = A.Arena(1 << 20)
    try:
        hu, pu = ar.allocate(x.nbytes, unified=True)
        C.memmove(pu, x.ctypes.data, x.nbytes)      # host writes managed memory directly
        hq, pq = ar.allocate(4 * 40)
        assert A.lib().nyion_attn_quantize_q4(pu, pq, 4, D, None) == 0, A.last_error()
        torch.cuda.synchronize()
        got = np.empty((4, 40), np.uint8)
        ar.download(hq, got)
        assert np.array_equal(got, O.q4_quantize_rows(x, D))
        ar.free(hu)
    finally:
        ar.close()
