"""GPU parity of the fp32 decode kernels against the CPU oracle.

Tolerance: max-abs 1e-3 on attention outputs (fp32 KV), as the north star
states; the kernels use a different summation order (online softmax), so the
comparison is not bit-exact.  All calls go through the C ABI.
"""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
H, N_KV, D = 32, 4, 64


def _zoned_store(n_layers, tokens, gen, fill_layers=None):
    """Reference-layout pages filled with exact fp32 rows (ensure_pages_hot_f32
    then save, cache.rs:555-561 + 671-677)."""
    zp = O.ZonedPages(n_layers, N_KV, D, max(tokens, 1))
    ks = torch.randn(tokens, n_layers, N_KV, D, generator=gen).numpy()
    vs = torch.randn(tokens, n_layers, N_KV, D, generator=gen).numpy()
    for pos in range(tokens):
        for l in range(n_layers):
            zp.set_f32_exact(l, pos, ks[pos, l], vs[pos, l])
    return zp


def _arenas(zp, dev):
    n = max(zp.k_f32) + 1
    k = np.concatenate([zp.k_f32[i] for i in range(n)])
    v = np.concatenate([zp.v_f32[i] for i in range(n)])
    return torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev)


def test_config1_reference_layout(cuda_device):
    """Config 1: B=1, ctx 128, seed 0, reference PagedKVCache layout."""
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(H, D, generator=gen)
    zp = _zoned_store(1, 128, gen)
    k, v = _arenas(zp, cuda_device)
    out = A.decode_zoned_f32(q.to(cuda_device), k, v, 1, 0, 128, 127)
    ref = O.attention(zp, q.numpy(), 0, 128, 127, H)
    assert np.abs(out.cpu().numpy() - ref).max() < TOL
    assert A.device_error() == 0


@pytest.mark.parametrize("ctx,qpos", [(1, 0), (17, 16), (31, 30), (33, 32), (128, 60), (129, 128),
                                      (4096, 4095), (4200, 4199), (4200, 3000)])
def test_zoned_edges_multilayer(cuda_device, ctx, qpos):
    gen = torch.Generator().manual_seed(ctx)
    zp = _zoned_store(2, ctx, gen)
    q = torch.randn(H, D, generator=gen)
    k, v = _arenas(zp, cuda_device)
    out = A.decode_zoned_f32(q.to(cuda_device), k, v, 2, 1, ctx, qpos)
    ref = O.attention(zp, q.numpy(), 1, ctx, qpos, H)
    assert np.abs(out.cpu().numpy() - ref).max() < TOL


def _paged_case(lens, max_pages, seed, dev, extra_pages=7):
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    n_pages = B * max_pages + extra_pages
    pool = torch.randn(n_pages, N_KV, 2, 16, D, generator=g)
    perm = torch.randperm(n_pages, generator=g)[: B * max_pages].to(torch.int32).reshape(B, max_pages)
    q = torch.randn(B, H, D, generator=g)
    lens_t = torch.tensor(lens, dtype=torch.int32)
    return q, pool, perm, lens_t


@pytest.mark.parametrize("lens", [[100], [0, 1, 16, 17, 31, 32, 33, 1000], [4096] * 4,
                                  [5, 2000, 0, 4096, 77, 1, 640, 3333, 12, 1024]])
def test_paged_ragged_vs_oracle(cuda_device, lens):
    max_pages = 256
    q, pool, table, lens_t = _paged_case(lens, max_pages, seed=sum(lens) + len(lens), dev=cuda_device)
    out = A.decode_paged_f32(q.to(cuda_device), pool.to(cuda_device), table.to(cuda_device),
                             lens_t.to(cuda_device))
    ref = O.decode_paged_f32(q.numpy(), pool.numpy(), table.numpy(), lens_t.numpy(), N_KV, D, 16,
                             threads=8)
    assert np.abs(out.cpu().numpy() - ref).max() < TOL
    for b, L in enumerate(lens):
        if L == 0:
            assert torch.count_nonzero(out[b]).item() == 0
    assert A.device_error() == 0


def test_config2_shape_one_layer(cuda_device):
    """Config 2 geometry (B=32, ctx 4096, 16-token pages, shuffled table), one
    layer, against the oracle."""
    B, ctx, mp = 32, 4096, 256
    q, pool, table, lens_t = _paged_case([ctx] * B, mp, seed=2, dev=cuda_device, extra_pages=0)
    ws = A.Workspace(B, N_KV, H, D)
    dq, dp, dt, dl = (x.to(cuda_device) for x in (q, pool, table, lens_t))
    out1 = A.decode_paged_f32(dq, dp, dt, dl, workspace=ws).cpu().numpy()
    out2 = A.decode_paged_f32(dq, dp, dt, dl, workspace=ws).cpu().numpy()
    ref = O.decode_paged_f32(q.numpy(), pool.numpy(), table.numpy(), lens_t.numpy(), N_KV, D, 16,
                             threads=8)
    assert np.abs(out1 - ref).max() < TOL
    # the merge counters reset themselves: a second call on the same workspace agrees
    assert np.array_equal(out1, out2)
    # counters (first workspace region, one int32 per (sequence, KV head)) are back at zero
    assert int(ws.buf[:B * N_KV * 4].view(torch.int32).abs().sum().item()) == 0


def test_page_id_out_of_range_reports_error(cuda_device):
    q, pool, table, lens_t = _paged_case([64, 64], 8, seed=3, dev=cuda_device)
    table[1, 2] = pool.shape[0] + 5   # bad page id: zero-filled box + error bit, no fault
    out = A.decode_paged_f32(q.to(cuda_device), pool.to(cuda_device), table.to(cuda_device),
                             lens_t.to(cuda_device))
    bits = A.device_error()
    assert bits & 1
    good = O.decode_paged_f32(q.numpy()[:1], pool.numpy(), table.numpy()[:1], lens_t.numpy()[:1],
                              N_KV, D, 16)
    assert np.abs(out[:1].cpu().numpy() - good).max() < TOL
    assert A.device_error() == 0


def test_reference_abi_contiguous_and_graph(cuda_device):
    """gpu_attention_device / _streamed / _forward / graph API of
    fused_attention.cu, K/V [n_kv][kv_stride][hd]."""
    g = torch.Generator().manual_seed(5)
    seq, stride = 300, 512
    q = torch.randn(H, D, generator=g)
    k = torch.randn(N_KV, stride, D, generator=g)
    v = torch.randn(N_KV, stride, D, generator=g)
    # oracle: the same tokens as a zoned single-layer store
    zp = O.ZonedPages(1, N_KV, D, seq)
    for pos in range(seq):
        zp.set_f32_exact(0, pos, k[:, pos].numpy(), v[:, pos].numpy())
    ref = O.attention(zp, q.numpy(), 0, seq, seq - 1, H)
    L = A.lib()
    dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    out = torch.zeros(H, D, device=cuda_device)
    assert L.gpu_attention_device(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(),
                                  H, N_KV, seq, D, stride) == 0
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - ref).max() < TOL
    s = torch.cuda.Stream()
    out2 = torch.zeros(H, D, device=cuda_device)
    assert L.gpu_attention_streamed(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out2.data_ptr(),
                                    H, N_KV, seq, D, stride, s.cuda_stream) == 0
    s.synchronize()
    assert np.abs(out2.cpu().numpy() - ref).max() < TOL
    out3 = torch.zeros(H, D, device=cuda_device)
    handle = L.gpu_graph_create_attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), 0,
                                          out3.data_ptr(), H, N_KV, seq, D, stride)
    assert handle
    out3.zero_()
    for _ in range(3):
        assert L.gpu_graph_replay_attention(handle, s.cuda_stream) == 0
    s.synchronize()
    L.gpu_graph_destroy(handle)
    assert np.abs(out3.cpu().numpy() - ref).max() < TOL
    # host-pointer variant: contiguous [n_kv][seq][hd]
    kh = np.ascontiguousarray(k[:, :seq].numpy())
    vh = np.ascontiguousarray(v[:, :seq].numpy())
    qh = np.ascontiguousarray(q.numpy())
    oh = np.zeros((H, D), np.float32)
    f = lambda a: a.ctypes.data
    assert L.gpu_attention_forward(f(qh), f(kh), f(vh), f(oh), H, N_KV, seq, D) == 0
    assert np.abs(oh - ref).max() < TOL


def test_unsupported_shape_is_an_error(cuda_device):
    L = A.lib()
    x = torch.zeros(16, device=cuda_device)
    rc = L.gpu_attention_device(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                4, 4, 1, 96, 1)                   # head_dim 96: neither 64 nor 128
    assert rc == -1 and "head_dim" in A.last_error()
    rc = L.gpu_attention_device(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                64, 4, 1, 64, 1)                  # 16 query heads per KV head
    assert rc == -1


@pytest.mark.parametrize("ctx,qpos,prior", [(1, 0, 0.0), (128, 127, 0.0), (300, 200, 0.5), (512, 511, 0.0),
                                            (4200, 4199, 0.25)])
def test_attention_tracked_importance(cuda_device, ctx, qpos, prior):
    """ops::attention_tracked (ops.rs:283-401): same output as the decode, and
    importance[t] += sum over heads of the softmax weights (positions past
    q_pos keep their value); the oracle sums the f32 weights in double."""
    gen = torch.Generator().manual_seed(ctx + qpos)
    zp = _zoned_store(1, ctx, gen)
    q = torch.randn(H, D, generator=gen)
    k, v = _arenas(zp, cuda_device)
    imp = torch.full((ctx,), prior, dtype=torch.float64, device=cuda_device)
    out = A.decode_zoned_f32_tracked(q.to(cuda_device), k, v, 1, 0, ctx, qpos, imp)
    ref_out, ref_imp = O.attention(zp, q.numpy(), 0, ctx, qpos, H, tracked=True)
    assert np.abs(out.cpu().numpy() - ref_out).max() < TOL
    got = imp.cpu().numpy() - prior
    assert np.abs(got - ref_imp).max() < 1e-5
    assert abs(got.sum() - H) < 1e-4                        # each head's weights sum to 1
    assert not got[qpos + 1:].any()
    assert A.device_error() == 0
