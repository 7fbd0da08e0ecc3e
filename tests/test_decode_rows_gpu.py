"""GPU parity of the single-sequence row-cache decode (decode_contig.cu) at
sizes where every CTA refills its stage ring several times, for other KV-head
counts, and across all three zones of the reference arena.

The checker is attention in float64 over the same K/V rows (for f16 caches,
the f16 values), with the reference's masking (tokens [0, valid_end]); the
zone arena is filled through the oracle's restatement of the reference page
geometry (cache.rs page_id / slot_in_page).  Tolerance: max-abs 1e-3.
"""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
D = 64


def _attend(q, k, v, n):
    """q [H][D]; k, v [n_kv][>=n][D]; float64 softmax attention over tokens [0, n)."""
    H, n_kv = q.shape[0], k.shape[0]
    g = H // n_kv
    q64 = q.double().reshape(n_kv, g, D)
    k64, v64 = k[:, :n].double(), v[:, :n].double()
    s = torch.einsum("kgd,ktd->kgt", q64, k64) / np.sqrt(D)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("kgt,ktd->kgd", p, v64).reshape(H, D).float()


@pytest.mark.parametrize("n_kv,seq,stride", [(1, 5000, 5000), (2, 777, 800), (4, 20000, 20000),
                                             (4, 65536, 65536), (8, 20001, 20480), (16, 3000, 3000)])
def test_contiguous_f32_sizes_and_kv_heads(cuda_device, n_kv, seq, stride):
    g = torch.Generator().manual_seed(seq + n_kv)
    H = 8 * n_kv
    q = torch.randn(H, D, generator=g)
    k = torch.randn(n_kv, stride, D, generator=g)
    v = torch.randn(n_kv, stride, D, generator=g)
    want = _attend(q, k, v, seq)
    dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    out = torch.zeros(H, D, device=cuda_device)
    s = torch.cuda.Stream()
    assert A.lib().gpu_attention_streamed(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), H, n_kv,
                                          seq, D, stride, s.cuda_stream) == 0
    s.synchronize()
    assert (out.cpu() - want).abs().max().item() < TOL
    assert A.device_error() == 0


@pytest.mark.parametrize("seq,stride", [(40000, 40000), (100, 128), (4097, 5000)])
def test_contiguous_f16_long(cuda_device, seq, stride):
    g = torch.Generator().manual_seed(seq)
    H, n_kv = 32, 4
    q = torch.randn(H, D, generator=g)
    k = torch.randn(n_kv, stride, D, generator=g).half()
    v = torch.randn(n_kv, stride, D, generator=g).half()
    want = _attend(q, k.float(), v.float(), seq)
    out = A.decode_contig_f16(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), seq)
    torch.cuda.synchronize()
    assert (out.cpu() - want).abs().max().item() < TOL
    assert A.device_error() == 0


def test_contiguous_repeated_calls_share_counters(cuda_device):
    """Calls of different lengths and KV-head counts in a row on one stream:
    every call leaves the merge counters at zero for the next."""
    s = torch.cuda.Stream()
    for i, (n_kv, seq) in enumerate([(4, 9000), (2, 12000), (4, 300), (8, 9000), (4, 9000)]):
        g = torch.Generator().manual_seed(100 + i)
        H = 8 * n_kv
        q, k, v = (torch.randn(H, D, generator=g), torch.randn(n_kv, seq, D, generator=g),
                   torch.randn(n_kv, seq, D, generator=g))
        dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
        out = torch.zeros(H, D, device=cuda_device)
        for _ in range(2):
            assert A.lib().gpu_attention_streamed(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), H,
                                                  n_kv, seq, D, seq, s.cuda_stream) == 0
        s.synchronize()
        assert (out.cpu() - _attend(q, k, v, seq)).abs().max().item() < TOL, (n_kv, seq)


def _zone_arena(n_layers, n_kv, tokens, gen):
    """Token-major K/V [tokens][n_layers][n_kv][D] and the reference arena
    built from them: flat pages in page-id order, each [layer][kv][slot][D]."""
    ks = torch.randn(tokens, n_layers, n_kv, D, generator=gen)
    vs = torch.randn(tokens, n_layers, n_kv, D, generator=gen)
    pos = np.arange(tokens)
    pid = np.array([O.page_id(int(p)) for p in pos])
    slot = np.array([O.slot_in_page(int(p)) for p in pos])
    n_pages = int(pid.max()) + 1
    bs = np.array([32 if p < 128 else (128 if p < 1120 else 1024) for p in range(n_pages)])
    page_rows = n_layers * n_kv * bs
    page_off = np.concatenate([[0], np.cumsum(page_rows)[:-1]])
    k_ar = torch.zeros(int(page_rows.sum()), D)
    v_ar = torch.zeros(int(page_rows.sum()), D)
    for layer in range(n_layers):
        for h in range(n_kv):
            rows = torch.from_numpy(page_off[pid] + (layer * n_kv + h) * bs[pid] + slot)
            k_ar[rows] = ks[:, layer, h]
            v_ar[rows] = vs[:, layer, h]
    return ks, vs, k_ar, v_ar


@pytest.mark.parametrize("ctx,qpos", [(140000, 139999), (140000, 100000), (9000, 8999)])
def test_zoned_long_contexts_all_zones(cuda_device, ctx, qpos):
    """ops::attention over the zone arena above the short-context kernel's
    512 tokens: zone 0 (32-slot pages), zone 1 (128) and zone 2 (1024)."""
    gen = torch.Generator().manual_seed(ctx + qpos)
    n_layers, n_kv, H = 2, 4, 32
    ks, vs, k_ar, v_ar = _zone_arena(n_layers, n_kv, ctx, gen)
    q = torch.randn(H, D, generator=gen)
    layer = 1
    n = min(qpos, ctx - 1) + 1
    want = _attend(q, ks[:, layer].transpose(0, 1), vs[:, layer].transpose(0, 1), n)
    out = A.decode_zoned_f32(q.to(cuda_device), k_ar.to(cuda_device), v_ar.to(cuda_device), n_layers, layer, ctx,
                             qpos)
    torch.cuda.synchronize()
    assert (out.cpu() - want).abs().max().item() < TOL
    assert A.device_error() == 0


def test_ring_f16_empty_and_single_token(cuda_device):
    """Device length 0 attends nothing (zeros, no NaN); length 1 returns V of
    slot 0 for every head of the group."""
    H, n_kv, W = 32, 4, 256
    g = torch.Generator().manual_seed(9)
    q = torch.randn(H, D, generator=g)
    k = torch.randn(n_kv, W, D, generator=g).half()
    v = torch.randn(n_kv, W, D, generator=g).half()
    dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    ws = A.F16Workspace(H, W, device=cuda_device)
    for n in (0, 1):
        d_len = torch.full((1,), n, dtype=torch.int32, device=cuda_device)
        out = A.decode_ring_f16(dq, dk, dv, d_len, workspace=ws)
        torch.cuda.synchronize()
        o = out.cpu()
        assert torch.isfinite(o).all()
        if n == 0:
            assert (o == 0).all()
        else:
            want = v[:, 0].float().repeat_interleave(H // n_kv, dim=0)
            assert (o - want).abs().max().item() < TOL
    assert A.device_error() == 0


def test_zoned_long_context_missing_pages_report_error(cuda_device):
    """An arena that lacks zone pages the context needs: the missing tiles are
    skipped, the device error word reports a page outside the arena, and the
    call neither faults nor hangs."""
    gen = torch.Generator().manual_seed(21)
    n_layers, n_kv, H = 1, 4, 32
    ctx = 6000                                  # zone 0 (128 pages) + zone 1 pages
    ks, vs, k_ar, v_ar = _zone_arena(n_layers, n_kv, 4096, gen)   # only the 128 zone-0 pages exist
    q = torch.randn(H, D, generator=gen)
    A.device_error()                            # clear
    out = A.decode_zoned_f32(q.to(cuda_device), k_ar.to(cuda_device), v_ar.to(cuda_device), n_layers, 0, ctx,
                             ctx - 1)
    torch.cuda.synchronize()
    assert torch.isfinite(out.cpu()).all()
    assert A.device_error() & 1                 # page outside the arena
    # the attended tokens that do exist (zone 0) give the output
    want = _attend(q, ks[:, 0].transpose(0, 1), vs[:, 0].transpose(0, 1), 4096)
    assert (out.cpu() - want).abs().max().item() < TOL
