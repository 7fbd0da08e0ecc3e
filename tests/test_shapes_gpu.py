"""Shapes beyond TinyLlama's (head_dim 64, GQA group 8): head_dim 64 and 128
with 1, 2, 4 and 8 query heads per KV head, as the reference's ops::attention
(swamp-engine/src/ops.rs:170-191) and its CUDA decode
(swamp-gpu/kernels/fused_attention.cu:20-68, 194-243) take them.  Every path is
checked against the CPU oracle (max-abs 1e-3 for fp32 / f16 / 4-bit KV, 2e-2
for the bf16 prefill); the contiguous fp32 and f16 decodes also against the
reference's own CUDA compiled here.  Shapes outside the supported set still
return NYION_ERR_UNSUPPORTED."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "libref_fused_attention.so")
PT = 16
TOL = 1e-3
SHAPES = [(hd, g) for hd in (64, 128) for g in (1, 2, 4, 8)]


@pytest.mark.parametrize("hd,g", SHAPES)
def test_paged_f32(cuda_device, hd, g):
    n_kv = 3 if g < 8 else 2
    H = n_kv * g
    rng = np.random.default_rng(hd * 10 + g)
    lens = np.array([1000, 1, 0, 333], np.int32)
    B, mp = len(lens), 63
    n_pages = B * mp + 2
    pool = rng.standard_normal((n_pages, n_kv, 2, PT, hd), dtype=np.float32)
    table = rng.permutation(n_pages)[: B * mp].astype(np.int32).reshape(B, mp)
    q = rng.standard_normal((B, H, hd), dtype=np.float32)
    dev = lambda a: torch.from_numpy(a).to(cuda_device)
    out = A.decode_paged_f32(dev(q), dev(pool), dev(table), dev(lens)).cpu().numpy()
    ref = O.decode_paged_f32(q, pool, table, lens, n_kv, hd, PT, threads=8)
    assert np.abs(out - ref).max() < TOL
    assert np.all(out[2] == 0)
    assert A.device_error() == 0


@pytest.mark.parametrize("hd,g", [(128, 4), (64, 1), (128, 8), (64, 2)])
def test_zoned_f32_across_zones(cuda_device, hd, g):
    n_kv = 2
    H = n_kv * g
    seq_len = 4300 if hd == 64 else 4200          # zone 0 (32-slot pages) and zone 1 (128-slot pages)
    rng = np.random.default_rng(seq_len + g)
    zp = O.ZonedPages(2, n_kv, hd, seq_len)
    k = rng.standard_normal((seq_len, n_kv, hd), dtype=np.float32)
    v = rng.standard_normal((seq_len, n_kv, hd), dtype=np.float32)
    last = O.page_id(seq_len - 1)
    zp.ensure_f32(last)
    for t in range(seq_len):
        pid, slot, bs = O.page_id(t), O.slot_in_page(t), O.block_size_for(t)
        for kh in range(n_kv):
            off = ((1 * n_kv + kh) * bs + slot) * hd     # layer 1
            zp.k_f32[pid][off:off + hd] = k[t, kh]
            zp.v_f32[pid][off:off + hd] = v[t, kh]
    q = rng.standard_normal((H, hd), dtype=np.float32)
    ref = O.attention(zp, q, 1, seq_len, seq_len - 1, H)
    ka = np.concatenate([zp.k_f32[p] for p in range(last + 1)])
    va = np.concatenate([zp.v_f32[p] for p in range(last + 1)])
    out = A.decode_zoned_f32(torch.from_numpy(q).to(cuda_device), torch.from_numpy(ka).to(cuda_device),
                             torch.from_numpy(va).to(cuda_device), 2, 1, seq_len, seq_len - 1,
                             n_kv=n_kv).cpu().numpy()
    assert np.abs(out - ref).max() < TOL


def _ref_lib():
    L = C.CDLL(REF)
    L.gpu_attention_device.restype = C.c_int
    L.gpu_attention_device.argtypes = [C.c_void_p] * 4 + [C.c_int] * 5
    L.gpu_attention_streamed_half.restype = C.c_int
    L.gpu_attention_streamed_half.argtypes = [C.c_void_p] * 4 + [C.c_int] * 5 + [C.c_void_p]
    return L


def _attend(q, k, v, n):
    """float64 attention of q [H, hd] over rows [n_kv][0, n)."""
    H, hd = q.shape
    n_kv = k.shape[0]
    g = H // n_kv
    out = np.zeros((H, hd))
    for h in range(H):
        kk, vv = k[h // g, :n].astype(np.float64), v[h // g, :n].astype(np.float64)
        s = kk @ q[h].astype(np.float64) / np.sqrt(hd)
        p = np.exp(s - s.max())
        out[h] = p @ vv / p.sum()
    return out


@pytest.mark.parametrize("hd,g", SHAPES)
@pytest.mark.parametrize("half", [False, True])
def test_contiguous_vs_reference_cuda(cuda_device, hd, g, half):
    n_kv, seq_len, stride = 2, 1500, 1536
    H = n_kv * g
    rng = np.random.default_rng(hd + g + half)
    q = rng.standard_normal((H, hd), dtype=np.float32)
    k = rng.standard_normal((n_kv, stride, hd), dtype=np.float32)
    v = rng.standard_normal((n_kv, stride, hd), dtype=np.float32)
    if half:
        k, v = k.astype(np.float16), v.astype(np.float16)
    dq, dk, dv = (torch.from_numpy(x).to(cuda_device) for x in (q, k, v))
    out = torch.zeros(H, hd, device=cuda_device)
    L = A.lib()
    fn = L.gpu_attention_streamed_half if half else L.gpu_attention_streamed
    assert fn(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), H, n_kv, seq_len, hd, stride, None) == 0, \
        A.last_error()
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want = _attend(q, k.astype(np.float32), v.astype(np.float32), seq_len)
    assert np.abs(got - want).max() < TOL
    if os.path.exists(REF):
        R = _ref_lib()
        rout = torch.zeros(H, hd, device=cuda_device)
        rf = R.gpu_attention_streamed_half if half else R.gpu_attention_device
        args = [dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), rout.data_ptr(), H, n_kv, seq_len, hd, stride]
        assert (rf(*args, None) if half else rf(*args)) == 0
        torch.cuda.synchronize()
        assert (rout - out).abs().max().item() < TOL


@pytest.mark.parametrize("hd,g", [(128, 4), (64, 2), (128, 1)])
def test_f16_ring_device_length(cuda_device, hd, g):
    n_kv, window = 2, 2048
    H = n_kv * g
    rng = np.random.default_rng(7 * hd + g)
    q = rng.standard_normal((H, hd), dtype=np.float32)
    k = rng.standard_normal((n_kv, window, hd)).astype(np.float16)
    v = rng.standard_normal((n_kv, window, hd)).astype(np.float16)
    dq, dk, dv = (torch.from_numpy(x).to(cuda_device) for x in (q, k, v))
    for n in (1, 700, 5000):                 # the length is clamped to the window
        d_len = torch.tensor([n], dtype=torch.int32, device=cuda_device)
        got = A.decode_ring_f16(dq, dk, dv, d_len).cpu().numpy()
        want = _attend(q, k.astype(np.float32), v.astype(np.float32), min(n, window))
        assert np.abs(got - want).max() < TOL


@pytest.mark.parametrize("hd,g", [(128, 4), (64, 1), (128, 8), (64, 4)])
def test_q4_partial(cuda_device, hd, g):
    n_kv, T = 2, 900
    H = n_kv * g
    rng = np.random.default_rng(hd * 3 + g)
    src = rng.standard_normal((T, n_kv, 2, hd), dtype=np.float32)
    q4 = O.q4_quantize_rows(src, hd)                       # [T][n_kv][2][hd / 32 * 20]
    rb = hd // 32 * 20
    mp = (T + PT - 1) // PT
    perm = rng.permutation(mp + 3)[:mp].astype(np.int32)
    pool = np.zeros((mp + 3, n_kv, 2, PT, rb), np.uint8)
    for t in range(T):
        pool[perm[t // PT], :, :, t % PT] = q4[t]
    table = perm[None]
    q = rng.standard_normal((1, H, hd), dtype=np.float32)
    dq, dp, dt = (torch.from_numpy(x).to(cuda_device) for x in (q, pool, table))
    for lo, hi in ((0, T), (37, 500), (100, 101), (64, 64)):
        part = A.decode_q4_partial(dq, dp, dt, u_begin=lo, u_end=hi).cpu().numpy()
        ref = O.decode_q4_partial(q, pool, table, lo, hi, n_kv, hd, PT, threads=4)
        if hi <= lo:
            assert np.all(part[0, :, hd + 1] == 0) and np.all(np.isneginf(part[0, :, hd]))
            continue
        assert np.abs(part[0, :, :hd] - ref[0, :, :hd]).max() < TOL
        assert np.allclose(part[0, :, hd], ref[0, :, hd], rtol=1e-3, atol=1e-4)
        assert np.allclose(part[0, :, hd + 1], ref[0, :, hd + 1], rtol=1e-3)
    # the LSE combine at this head_dim, and the split property
    pieces = torch.stack([A.decode_q4_partial(dq, dp, dt, u_begin=a, u_end=b) for a, b in ((0, 400), (400, T))])
    whole = A.lse_combine(A.decode_q4_partial(dq, dp, dt, u_begin=0, u_end=T)[None])
    assert (A.lse_combine(pieces) - whole).abs().max().item() < 1e-4
    assert A.device_error() == 0


@pytest.mark.parametrize("hd,g", [(128, 4), (64, 1), (128, 2)])
def test_prefill_bf16(cuda_device, hd, g):
    n_kv = 2
    H = n_kv * g
    rng = np.random.default_rng(hd + 100 * g)
    T, q_start = 300, 200                                   # a chunk of 100 after 200 cached tokens
    n_pages = (T + PT - 1) // PT
    pool = torch.from_numpy(rng.standard_normal((n_pages + 2, n_kv, 2, PT, hd), dtype=np.float32) * 0.5).to(torch.bfloat16)
    table = torch.from_numpy(rng.permutation(n_pages + 2)[:n_pages].astype(np.int32))
    q = torch.from_numpy(rng.standard_normal((T - q_start, H, hd), dtype=np.float32) * 0.5).to(torch.bfloat16)
    out = A.prefill_paged_bf16(q.to(cuda_device), pool.to(cuda_device), table.to(cuda_device), q_start).cpu().numpy()
    ref = O.prefill_paged_bf16(q.view(torch.int16).numpy().view(np.uint16), pool.view(torch.int16).numpy().view(np.uint16),
                               table.numpy(), q_start, n_kv, hd, PT, threads=8)
    assert np.abs(out - ref).max() < 2e-2


def test_unsupported_shapes_refused(cuda_device):
    L = A.lib()
    q = torch.zeros(16, 96, device=cuda_device)
    kv = torch.zeros(2, 64, 96, device=cuda_device)
    out = torch.zeros_like(q)
    f = L.gpu_attention_streamed
    assert f(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(), 16, 2, 10, 96, 64, None) == -1   # head_dim 96
    pool = torch.zeros(4, 1, 2, PT, 64, device=cuda_device)
    table = torch.zeros(1, 4, dtype=torch.int32, device=cuda_device)
    lens = torch.ones(1, dtype=torch.int32, device=cuda_device)
    with pytest.raises(A.NyionError) as e:                 # 16 query heads per KV head
        A.decode_paged_f32(torch.zeros(1, 16, 64, device=cuda_device), pool, table, lens)
    assert e.value.status == -3
