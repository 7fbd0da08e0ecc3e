"""The reference's cold-tier slot format (swamp-engine/src/cache.rs:251-276,
440-483, 485-529) moved into and out of the 16-token 4-bit page pools,
byte-exact:

  * slots cut from a reference-layout page store (oracle.ZonedPages, zones 0
    and 1, two layers) scatter into per-layer pools whose rows equal the
    oracle quantizer's rows of the same tokens, and gather back to the same
    slot bytes;
  * a zone-2 (1024-slot) slot of random bytes round-trips, from HBM and from
    mapped pinned host memory, with every row where the layout puts it;
  * the decode over a loaded pool equals the decode over a pool written
    directly;
  * pointers the device cannot reach are refused before any launch; page ids
    outside the pool raise the page-range bit.
"""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
N_KV, D, PT, ROW = 4, 64, 16, 40


def _expected_pool_rows(slot, bs, n_layers):
    """slot bytes -> [n_layers][bs][n_kv][2][40] (token-major) per the cache.rs layout."""
    half = n_layers * N_KV * bs * ROW
    k = slot[:half].reshape(n_layers, N_KV, bs, ROW)
    v = slot[half:2 * half].reshape(n_layers, N_KV, bs, ROW)
    return np.stack([k, v], axis=3).transpose(0, 2, 1, 3, 4)   # [L][bs][n_kv][2][40]


def _check_pools(pools, ids, rows, bs):
    for l, pool in enumerate(pools):
        p = pool.cpu().numpy()
        for j in range(bs // PT):
            got = p[ids[l, j]].transpose(2, 0, 1, 3)            # [16][n_kv][2][40]
            assert np.array_equal(got, rows[l, PT * j: PT * (j + 1)])


def test_zoned_store_slots_to_pools_and_back(cuda_device):
    rng = np.random.default_rng(1)
    n_layers, T = 2, 4096 + 200
    zp = O.ZonedPages(n_layers, N_KV, D, T)
    src = rng.standard_normal((T, n_layers, N_KV, 2, D), dtype=np.float32)
    for t in range(T):
        for l in range(n_layers):
            zp.save(l, t, src[t, l, :, 0], src[t, l, :, 1])
    dev = cuda_device
    n_pool = 40
    for pid, bs, start in [(3, 32, 96), (127, 32, 4064), (128, 128, 4096), (129, 128, 4224)]:
        assert O.page_id(start) == pid and O.block_size_for(start) == bs
        slot = np.concatenate([zp.k_q4[pid], zp.v_q4[pid]])
        assert slot.size == 2 * A.cold_q4_page_bytes(bs, n_layers, N_KV)
        ids = rng.permutation(n_pool)[: n_layers * bs // PT].astype(np.int32).reshape(n_layers, bs // PT)
        pools = [torch.zeros(n_pool, N_KV, 2, PT, ROW, dtype=torch.uint8, device=dev) for _ in range(n_layers)]
        dids = torch.from_numpy(ids).to(dev)
        A.cold_to_pool(torch.from_numpy(slot).to(dev), bs, pools, dids)
        torch.cuda.synchronize()
        rows = _expected_pool_rows(slot, bs, n_layers)
        _check_pools(pools, ids, rows, bs)
        # the rows are the oracle quantizer's rows of the tokens the page holds
        n = min(bs, T - start)
        want = O.q4_quantize_rows(src[start:start + n].transpose(1, 0, 2, 3, 4), D)   # [L][n][n_kv][2][40]
        assert np.array_equal(rows[:, :n], want)
        back = torch.zeros(slot.size, dtype=torch.uint8, device=dev)
        A.pool_to_cold(pools, dids, bs, back)
        torch.cuda.synchronize()
        assert np.array_equal(back.cpu().numpy(), slot)
    assert A.device_error() == 0


@pytest.mark.parametrize("pinned", [False, True])
def test_zone2_slot_round_trip(cuda_device, pinned):
    rng = np.random.default_rng(2 + pinned)
    n_layers, bs = 3, 1024
    nbytes = 2 * A.cold_q4_page_bytes(bs, n_layers, N_KV)
    slot = rng.integers(0, 256, nbytes, dtype=np.uint8)
    n_pool = n_layers * bs // PT + 9
    ids = rng.permutation(n_pool)[: n_layers * bs // PT].astype(np.int32).reshape(n_layers, bs // PT)
    dev = cuda_device
    pools = [torch.zeros(n_pool, N_KV, 2, PT, ROW, dtype=torch.uint8, device=dev) for _ in range(n_layers)]
    dids = torch.from_numpy(ids).to(dev)
    if pinned:
        hs = torch.from_numpy(slot).pin_memory()
        try:
            A.cold_to_pool(hs, bs, pools, dids)
        except A.NyionError as e:                 # pinned but not mapped on this system: refused, no launch
            assert "mapped pinned host memory" in str(e)
            pytest.skip("pinned host memory is not mapped into the device address space here")
    else:
        A.cold_to_pool(torch.from_numpy(slot).to(dev), bs, pools, dids)
    torch.cuda.synchronize()
    _check_pools(pools, ids, _expected_pool_rows(slot, bs, n_layers), bs)
    back = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    A.pool_to_cold(pools, dids, bs, back)
    torch.cuda.synchronize()
    assert np.array_equal(back.cpu().numpy(), slot)
    assert A.cold_q4_page_bytes(bs, n_layers, N_KV) * 2 * 7 == A.lib().nyion_attn_cold_slot_offset(7, bs, n_layers, N_KV, D)


def test_decode_over_loaded_pool(cuda_device):
    rng = np.random.default_rng(5)
    bs, T = 128, 128
    src = rng.standard_normal((1, T, N_KV, 2, D), dtype=np.float32)
    rows = O.q4_quantize_rows(src, D)[0]                           # [T][n_kv][2][40]
    slot = np.concatenate([rows[:, :, 0].transpose(1, 0, 2).reshape(-1), rows[:, :, 1].transpose(1, 0, 2).reshape(-1)])
    dev = cuda_device
    ids = np.array([[5, 2, 7, 0, 3, 6, 1, 4]], np.int32)
    pool = torch.zeros(8, N_KV, 2, PT, ROW, dtype=torch.uint8, device=dev)
    A.cold_to_pool(torch.from_numpy(slot).to(dev), bs, [pool], torch.from_numpy(ids).to(dev))
    direct = torch.zeros_like(pool)
    for t in range(T):
        direct[ids[0, t // PT], :, :, t % PT] = torch.from_numpy(rows[t]).to(dev)
    torch.cuda.synchronize()
    assert torch.equal(pool, direct)
    q = torch.from_numpy(rng.standard_normal((1, 32, D), dtype=np.float32)).to(dev)
    table = torch.from_numpy(ids).to(dev)
    a = A.lse_combine(A.decode_q4_partial(q, pool, table, u_begin=0, u_end=T)[None])
    want = O.lse_combine(O.decode_q4_partial(q.cpu().numpy(), direct.cpu().numpy(), ids, 0, T, N_KV, D, PT)[None])
    assert np.abs(a.cpu().numpy() - want).max() < 1e-3


def test_bad_pointers_and_page_ids(cuda_device):
    dev = cuda_device
    bs = 32
    pool = torch.zeros(4, N_KV, 2, PT, ROW, dtype=torch.uint8, device=dev)
    slot = torch.zeros(2 * A.cold_q4_page_bytes(bs, 1, N_KV), dtype=torch.uint8, device=dev)
    ids = torch.tensor([[0, 1]], dtype=torch.int32, device=dev)
    with pytest.raises(A.NyionError):
        A.cold_to_pool(slot, bs, [pool], torch.tensor([[0, 1]], dtype=torch.int32))       # host page ids
    with pytest.raises(A.NyionError):
        A.cold_to_pool(torch.zeros(slot.numel(), dtype=torch.uint8), bs, [pool], ids)     # pageable host slot
    with pytest.raises(A.NyionError):
        A.cold_to_pool(slot, 48, [pool], ids)                                              # not a zone size
    A.device_error()
    A.cold_to_pool(slot, bs, [pool], torch.tensor([[0, 9]], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert A.device_error() & 1
