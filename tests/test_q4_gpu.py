"""GPU parity of the 4-bit KV path against the CPU oracle (all through the C ABI).

- quantizer and dequant: bit-exact bytes / floats (cache.rs:637-663, 375-394);
- Q4 decode partials: o within max-abs 1e-3, (m, l) within 1e-3 relative;
- split-KV property: partials over [0,a), [a,b), [b,T) combine to the partial
  over [0,T) — the size-independent check used at full length;
- config 3 (B=16, window 4096 of 65536, fp32 ring of 128) at full shape, the
  oracle run on the window's pages.
"""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
H, N_KV, D, PT = 32, 4, 64, 16


def _rows(n, gen, scale=1.0):
    return (torch.randn(n, D, generator=gen) * scale).contiguous()


def test_quantizer_bit_exact(cuda_device):
    g = torch.Generator().manual_seed(21)
    x = torch.cat([_rows(5000, g), _rows(200, g, 1e-6), _rows(200, g, 300.0),
                   torch.zeros(3, D), torch.full((3, D), 42.0), torch.full((3, D), -7.5),
                   torch.arange(3 * D, dtype=torch.float32).reshape(3, D) - 50.0])
    want = O.q4_quantize_rows(x.numpy(), D)
    got = A.quantize_q4(x.to(cuda_device)).cpu().numpy()
    assert got.shape == want.shape
    assert np.array_equal(got, want)


def test_dequant_bit_exact(cuda_device):
    g = torch.Generator().manual_seed(22)
    x = torch.cat([_rows(3000, g), _rows(100, g, 1e-5), _rows(100, g, 1e3)])
    q4 = O.q4_quantize_rows(x.numpy(), D)
    want = O.q4_dequant_rows(q4, D)
    got = A.dequant_q4(torch.from_numpy(q4).to(cuda_device), D).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _q4_pool(B, T, max_pages, gen, dev, extra=5):
    """Random K/V [B][T][N_KV][2][D] quantized into a shuffled 16-token page pool."""
    src = torch.randn(B, T, N_KV, 2, D, generator=gen)
    q4 = O.q4_quantize_rows(src.numpy(), D)                       # [B][T][N_KV][2][40]
    n_pages = B * max_pages + extra
    perm = torch.randperm(n_pages, generator=gen)[: B * max_pages].numpy().astype(np.int32)
    table = perm.reshape(B, max_pages)
    pool = np.zeros((n_pages, N_KV, 2, PT, 40), np.uint8)
    for b in range(B):
        for t in range(T):
            pool[table[b, t // PT], :, :, t % PT] = q4[b, t]
    return src, pool, table


def _partial_ref(q, pool, table, b, lo, hi):
    return O.decode_q4_partial(q[b:b + 1], pool, table[b:b + 1], lo, hi, N_KV, D, PT)[0]


@pytest.mark.parametrize("ranges", [[(0, 700)], [(0, 700), (37, 500), (100, 101), (64, 64), (640, 700)],
                                    [(0, 64), (1, 2), (15, 17), (63, 129)]])
def test_q4_partial_vs_oracle(cuda_device, ranges):
    g = torch.Generator().manual_seed(len(ranges) * 31)
    B, T, mp = len(ranges), 700, 44
    _, pool, table = _q4_pool(B, T, mp, g, cuda_device)
    q = torch.randn(B, H, D, generator=g)
    tb = torch.tensor([r[0] for r in ranges], dtype=torch.int32)
    te = torch.tensor([r[1] for r in ranges], dtype=torch.int32)
    part = A.decode_q4_partial(q.to(cuda_device), torch.from_numpy(pool).to(cuda_device),
                               torch.from_numpy(table).to(cuda_device), tb.to(cuda_device),
                               te.to(cuda_device)).cpu().numpy()
    for b, (lo, hi) in enumerate(ranges):
        ref = _partial_ref(q.numpy(), pool, table, b, lo, hi)
        if hi <= lo:
            assert np.all(part[b, :, D + 1] == 0) and np.all(np.isneginf(part[b, :, D]))
            assert np.all(part[b, :, :D] == 0)
            continue
        assert np.abs(part[b, :, :D] - ref[:, :D]).max() < TOL
        assert np.allclose(part[b, :, D], ref[:, D], rtol=1e-3, atol=1e-4)
        assert np.allclose(part[b, :, D + 1], ref[:, D + 1], rtol=1e-3)
    assert A.device_error() == 0


def test_lse_combine_vs_oracle(cuda_device):
    g = torch.Generator().manual_seed(41)
    parts = torch.randn(3, 5, H, D + 2, generator=g)
    parts[..., D + 1] = parts[..., D + 1].abs() * 10
    parts[1, 2, :, D + 1] = 0.0            # an empty partial
    parts[1, 2, :, D] = -np.inf
    got = A.lse_combine(parts.to(cuda_device)).cpu().numpy()
    ref = O.lse_combine(parts.numpy())
    assert np.abs(got - ref).max() < 1e-5


def test_split_ranges_combine_to_whole(cuda_device):
    """Size-independent property of the split-KV path: partials over a split of
    [0, T) merge to the partial over [0, T)."""
    g = torch.Generator().manual_seed(43)
    B, T, mp = 2, 1000, 63
    _, pool, table = _q4_pool(B, T, mp, g, cuda_device)
    q = torch.randn(B, H, D, generator=g).to(cuda_device)
    dp, dt = torch.from_numpy(pool).to(cuda_device), torch.from_numpy(table).to(cuda_device)
    whole = A.decode_q4_partial(q, dp, dt, u_begin=0, u_end=T)
    pieces = torch.stack([A.decode_q4_partial(q, dp, dt, u_begin=a, u_end=b)
                          for a, b in [(0, 333), (333, 640), (640, T)]])
    merged = A.lse_combine(pieces)
    full = A.lse_combine(whole[None])
    assert (merged - full).abs().max().item() < 1e-4


def _window_ring_case(B, L, window, ring_tokens, seed, dev):
    g = torch.Generator().manual_seed(seed)
    T = max(L)
    mp = (T + PT - 1) // PT
    src, pool, table = _q4_pool(B, T, mp, g, dev)
    ring = np.zeros((B, N_KV, 2, ring_tokens, D), np.float32)
    srcn = src.numpy()
    for b in range(B):
        for t in range(max(0, L[b] - ring_tokens), L[b]):
            ring[b, :, :, t % ring_tokens] = srcn[b, t]
    q = torch.randn(B, H, D, generator=g)
    return q, pool, table, ring


@pytest.mark.parametrize("L,window,ring_tokens", [([1000, 300], 512, 128), ([130, 64, 1000], 4096, 128),
                                                  ([777], 100, 128), ([500, 60], 256, 64),
                                                  # 160 (sequence, KV head) ring units: some CTAs take two
                                                  ([3000 + 97 * i for i in range(40)], 1024, 100)])
def test_window_ring_vs_oracle(cuda_device, L, window, ring_tokens):
    B = len(L)
    q, pool, table, ring = _window_ring_case(B, L, window, ring_tokens, seed=sum(L), dev=cuda_device)
    lens = np.array(L, np.int32)
    out = A.decode_q4_window_ring(q.to(cuda_device), torch.from_numpy(pool).to(cuda_device),
                                  torch.from_numpy(table).to(cuda_device),
                                  torch.from_numpy(lens).to(cuda_device),
                                  torch.from_numpy(ring).to(cuda_device), window).cpu().numpy()
    ref = O.decode_q4_window_ring(q.numpy(), pool, table, lens, ring, ring_tokens, window, N_KV, D, PT,
                                  threads=8)
    assert np.abs(out - ref).max() < TOL


def test_config3_full_shape(cuda_device):
    """B=16, logical context 65536, window 4096, fp32 ring of the last 128
    tokens, K/V from N(0,1) quantized by the (bit-exact) GPU quantizer."""
    B, L, W, R = 16, 65536, 4096, 128
    mp = L // PT
    gd = torch.Generator(device=cuda_device).manual_seed(3)
    pool = torch.empty(B * mp, N_KV, 2, PT, 40, dtype=torch.uint8, device=cuda_device)
    table = torch.randperm(B * mp, device=cuda_device, generator=gd).to(torch.int32).reshape(B, mp)
    ring = torch.empty(B, N_KV, 2, R, D, device=cuda_device)
    for b in range(B):
        src = torch.randn(L, N_KV, 2, D, device=cuda_device, generator=gd)
        q4 = A.quantize_q4(src)                                  # [L][N_KV][2][40]
        pool[table[b].long()] = q4.reshape(mp, PT, N_KV, 2, 40).permute(0, 2, 3, 1, 4)
        tail = src[L - R:]                                        # slot = pos % R
        ring[b] = tail.permute(1, 2, 0, 3)[:, :, torch.arange(L - R, L, device=cuda_device) % R]
    q = torch.randn(B, H, D, device=cuda_device, generator=gd)
    lens = torch.full((B,), L, dtype=torch.int32, device=cuda_device)
    out = A.decode_q4_window_ring(q, pool, table, lens, ring, W, workspace=A.window_ring_workspace(B))
    # oracle on the window's pages only (remapped table)
    first = (L - W) // PT
    sub_pages = table[:, first:].reshape(-1).long()
    sub_pool = pool[sub_pages].cpu().numpy()
    sub_table = np.zeros((B, mp), np.int32)
    sub_table[:, first:] = np.arange(B * (mp - first), dtype=np.int32).reshape(B, mp - first)
    ref = O.decode_q4_window_ring(q.cpu().numpy(), sub_pool, sub_table, lens.cpu().numpy(),
                                  ring.cpu().numpy(), R, W, N_KV, D, PT, threads=8)
    assert np.abs(out.cpu().numpy() - ref).max() < TOL
    assert A.device_error() == 0
