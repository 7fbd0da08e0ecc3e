"""GPU parity of the KV write path (RoPE + save into the caches) against the
CPU oracle, bit-exact:

  * the RoPE table (ops.rs:20-38) equals the oracle's, and rotated q / k equal
    apply_rope_ufc's (ops.rs:42-84), including the max_context clamp;
  * the 4-bit slot bytes equal the oracle quantizer on the rotated rows
    (cache.rs:637-663); f32 / bf16 pages, the bf16 q copy and the fp32 ring
    hold the rotated values (bf16 / f16 by round-to-nearest-even); every byte
    outside the written slots keeps its sentinel;
  * a prefill chunk written through the path feeds the bf16 prefill kernel
    (max-abs 2e-2 against the oracle on the same bf16 values);
  * the layer-graph f16 ring write (device seq_len / wpos);
  * the reference ABI copies (gpu_copy_kv_layer*) equal the reference CUDA
    library's same-named functions when oracle/_ref is built;
  * a row without a page raises the page-range bit and writes nothing.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
H, N_KV, D, PT = 32, 4, 64, 16
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "libref_fused_attention.so")


def _bits_bf16(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).bfloat16().view(torch.int16).numpy()


def test_rope_table_matches_oracle(cuda_device):
    for hd, ctx in [(64, 2048), (64, 70000), (128, 100)]:
        got = A.rope_table(hd, ctx, device=cuda_device).cpu().numpy()
        want = O.rope_lut(hd, ctx)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (hd, ctx)


def _decode_case(rng, B, max_ctx, n_pages_extra=5):
    mp = 400
    n_pages = B * mp + n_pages_extra
    table = rng.permutation(n_pages)[: B * mp].astype(np.int32).reshape(B, mp)
    pos = rng.integers(0, mp * PT, B).astype(np.int32)
    pos[0] = max_ctx + 123                       # RoPE clamps to max_context - 1, the save does not
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    k = rng.standard_normal((B, N_KV, D), dtype=np.float32)
    v = rng.standard_normal((B, N_KV, D), dtype=np.float32)
    return table, pos, q, k, v, n_pages


def test_decode_rows_all_destinations_bit_exact(cuda_device):
    rng = np.random.default_rng(11)
    B, max_ctx, ring_t = 9, 5000, 128
    table, pos, q, k, v, n_pages = _decode_case(rng, B, max_ctx)
    dev = cuda_device
    lut = O.rope_lut(D, max_ctx)
    rope = A.rope_table(D, max_ctx, device=dev)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    dq, dk, dv, dpos, dtab = t(q), t(k), t(v), t(pos), t(table)
    pool_q4 = torch.full((n_pages, N_KV, 2, PT, 40), 0xA5, dtype=torch.uint8, device=dev)
    pool_f32 = torch.full((n_pages, N_KV, 2, PT, D), -7.0, dtype=torch.float32, device=dev)
    pool_bf16 = torch.full((n_pages, N_KV, 2, PT, D), -7.0, dtype=torch.bfloat16, device=dev)
    q_bf16 = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev)
    ring = torch.full((B, N_KV, 2, ring_t, D), -7.0, dtype=torch.float32, device=dev)
    A.device_error()
    A.kv_write_paged(dk, dv, dpos, q=dq, rope=rope, page_table=dtab, pool_q4=pool_q4, pool_f32=pool_f32,
                     pool_bf16=pool_bf16, q_bf16=q_bf16, ring_f32=ring)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    gq, gk = dq.cpu().numpy(), dk.cpu().numpy()
    p4, pf, pb, rg = pool_q4.cpu().numpy(), pool_f32.cpu().numpy(), pool_bf16.cpu(), ring.cpu().numpy()
    written = np.zeros((n_pages, PT), bool)
    for b in range(B):
        wq, wk = O.apply_rope(q[b], k[b], int(pos[b]), max_ctx, lut)
        assert np.array_equal(gq[b].view(np.uint32), wq.view(np.uint32))
        assert np.array_equal(gk[b].view(np.uint32), wk.view(np.uint32))
        assert np.array_equal(q_bf16[b].cpu().view(torch.int16).numpy(), _bits_bf16(wq))
        page, slot = table[b, pos[b] // PT], pos[b] % PT
        written[page, slot] = True
        kv = np.stack([wk, v[b]], axis=1)                        # [n_kv][2][D]
        assert np.array_equal(p4[page, :, :, slot], O.q4_quantize_rows(kv, D))
        assert np.array_equal(pf[page, :, :, slot].view(np.uint32), kv.view(np.uint32))
        assert np.array_equal(pb[page, :, :, slot].view(torch.int16).numpy(), _bits_bf16(kv))
        assert np.array_equal(rg[b, :, :, pos[b] % ring_t], kv)
    untouched = ~written
    assert (p4.transpose(0, 3, 1, 2, 4)[untouched] == 0xA5).all()
    assert (pf.transpose(0, 3, 1, 2, 4)[untouched] == -7.0).all()
    ring_hit = np.zeros((B, ring_t), bool)
    ring_hit[np.arange(B), pos % ring_t] = True
    assert (rg.transpose(0, 3, 1, 2, 4)[~ring_hit] == -7.0).all()


def test_plain_save_without_rope_and_q(cuda_device):
    rng = np.random.default_rng(3)
    B = 4
    table, pos, q, k, v, n_pages = _decode_case(rng, B, 1000)
    dev = cuda_device
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    dk = t(k)
    pool_q4 = torch.zeros((n_pages, N_KV, 2, PT, 40), dtype=torch.uint8, device=dev)
    A.kv_write_paged(dk, t(v), t(pos), page_table=t(table), pool_q4=pool_q4)
    torch.cuda.synchronize()
    assert np.array_equal(dk.cpu().numpy(), k)                  # no rotation
    p4 = pool_q4.cpu().numpy()
    for b in range(B):
        kv = np.stack([k[b], v[b]], axis=1)
        assert np.array_equal(p4[table[b, pos[b] // PT], :, :, pos[b] % PT], O.q4_quantize_rows(kv, D))


def test_prefill_chunk_feeds_the_bf16_prefill(cuda_device):
    rng = np.random.default_rng(21)
    T, max_ctx = 300, 4096
    mp = (T + PT - 1) // PT + 2
    n_pages = mp + 3
    table = rng.permutation(n_pages)[:mp].astype(np.int32)
    q = (0.5 * rng.standard_normal((T, H, D))).astype(np.float32)
    k = (0.5 * rng.standard_normal((T, N_KV, D))).astype(np.float32)
    v = (0.5 * rng.standard_normal((T, N_KV, D))).astype(np.float32)
    dev = cuda_device
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    rope = A.rope_table(D, max_ctx, device=dev)
    pool = torch.zeros((n_pages, N_KV, 2, PT, D), dtype=torch.bfloat16, device=dev)
    q_bf16 = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)
    positions = torch.arange(T, dtype=torch.int32, device=dev)
    row_seq = torch.zeros(T, dtype=torch.int32, device=dev)
    A.kv_write_paged(t(k), t(v), positions, q=t(q), row_seq=row_seq, rope=rope, page_table=t(table[None]),
                     pool_bf16=pool, q_bf16=q_bf16)
    out = A.prefill_paged_bf16(q_bf16, pool, t(table), q_start=0)
    torch.cuda.synchronize()
    lut = O.rope_lut(D, max_ctx)
    qr = np.empty_like(q)
    pool_ref = np.zeros((n_pages, N_KV, 2, PT, D), np.float32)
    for i in range(T):
        qr[i], kr = O.apply_rope(q[i], k[i], i, max_ctx, lut)
        pool_ref[table[i // PT], :, 0, i % PT] = kr
        pool_ref[table[i // PT], :, 1, i % PT] = v[i]
    assert np.array_equal(pool.cpu().view(torch.int16).numpy(), _bits_bf16(pool_ref))
    qb = torch.from_numpy(qr).bfloat16().view(torch.int16).numpy().view(np.uint16)
    pb = torch.from_numpy(pool_ref).bfloat16().view(torch.int16).numpy().view(np.uint16)
    want = O.prefill_paged_bf16(qb, pb, table, 0, N_KV, D, PT, threads=8)
    assert np.abs(out.cpu().numpy() - want).max() < 2e-2


@pytest.mark.parametrize("pos,window,use_wpos", [(0, 4096, False), (5000, 4096, False), (77, 256, True)])
def test_layer_graph_f16_ring(cuda_device, pos, window, use_wpos):
    rng = np.random.default_rng(pos + window)
    max_ctx = 8192
    q = rng.standard_normal((H, D), dtype=np.float32)
    k = rng.standard_normal((N_KV, D), dtype=np.float32)
    v = rng.standard_normal((N_KV, D), dtype=np.float32)
    dev = cuda_device
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    rope = A.rope_table(D, max_ctx, device=dev)
    kr = torch.zeros(N_KV, window, D, dtype=torch.float16, device=dev)
    vr = torch.zeros_like(kr)
    seq_len = torch.tensor([pos + 1], dtype=torch.int32, device=dev)
    slot = (pos * 7 + 3) % window if use_wpos else pos % window
    wpos = torch.tensor([slot], dtype=torch.int32, device=dev) if use_wpos else None
    dq, dk = t(q), t(k)
    A.kv_write_ring_f16(dk, t(v), seq_len, kr, vr, q=dq, d_wpos=wpos, rope=rope)
    torch.cuda.synchronize()
    wq, wk = O.apply_rope(q, k, pos, max_ctx, O.rope_lut(D, max_ctx))
    assert np.array_equal(dq.cpu().numpy(), wq)
    assert np.array_equal(kr[:, slot].cpu().numpy(), wk.astype(np.float16))
    assert np.array_equal(vr[:, slot].cpu().numpy(), v.astype(np.float16))
    others = np.ones(window, bool)
    others[slot] = False
    assert not kr.cpu().numpy()[:, others].any()


def test_missing_page_reports_and_skips(cuda_device):
    dev = cuda_device
    k = torch.randn(2, N_KV, D, device=dev)
    v = torch.randn(2, N_KV, D, device=dev)
    table = torch.tensor([[0, 1], [2, -1]], dtype=torch.int32, device=dev)
    pool = torch.zeros(3, N_KV, 2, PT, 40, dtype=torch.uint8, device=dev)
    A.device_error()
    A.kv_write_paged(k, v, torch.tensor([5, 20], dtype=torch.int32, device=dev), page_table=table, pool_q4=pool)
    torch.cuda.synchronize()
    assert A.device_error() & 1
    p = pool.cpu().numpy()
    assert p[0, :, :, 5].any() and not p[1:].any()
    A.kv_write_paged(k[:0], v[:0], torch.zeros(0, dtype=torch.int32, device=dev), page_table=table,
                     pool_q4=pool)                               # rows == 0: nothing to do
    with pytest.raises(A.NyionError):
        A.kv_write_paged(k, v, torch.zeros(2, dtype=torch.int32, device=dev), pool_q4=pool)  # no page table


def _ref_lib():
    L = C.CDLL(REF)
    for n, args in [("gpu_copy_kv_layer", [C.c_void_p, C.c_void_p] + [C.c_int] * 4),
                    ("gpu_copy_kv_layer_async", [C.c_void_p, C.c_void_p] + [C.c_int] * 4 + [C.c_void_p]),
                    ("gpu_copy_kv_layer_async_half", [C.c_void_p, C.c_void_p] + [C.c_int] * 4 + [C.c_void_p]),
                    ("gpu_copy_kv_to_buffer", [C.c_void_p, C.c_void_p] + [C.c_int] * 5)]:
        getattr(L, n).restype = C.c_int
        getattr(L, n).argtypes = args
    return L


@pytest.mark.skipif(not os.path.exists(REF), reason="reference CUDA not built (make -C oracle ref)")
def test_reference_copy_abi_matches_reference_cuda(cuda_device):
    R, L = _ref_lib(), A.lib()
    rng = np.random.default_rng(4)
    n_kv, max_seq = N_KV, 300
    src = rng.standard_normal((n_kv, D), dtype=np.float32)
    row = rng.standard_normal(D, dtype=np.float32)
    sp = src.ctypes.data
    for kind in ("f32", "f32_async", "half", "row"):
        dt = torch.float16 if kind == "half" else torch.float32
        ours = torch.zeros(n_kv, max_seq, D, dtype=dt, device=cuda_device)
        theirs = torch.zeros_like(ours)
        for lib_, buf in ((L, ours), (R, theirs)):
            if kind == "f32":
                rc = lib_.gpu_copy_kv_layer(buf.data_ptr(), sp, 123, n_kv, max_seq, D)
            elif kind == "f32_async":
                rc = lib_.gpu_copy_kv_layer_async(buf.data_ptr(), sp, 299, n_kv, max_seq, D, None)
            elif kind == "half":
                rc = lib_.gpu_copy_kv_layer_async_half(buf.data_ptr(), sp, 7, n_kv, max_seq, D, None)
            else:
                rc = lib_.gpu_copy_kv_to_buffer(buf.data_ptr(), row.ctypes.data, 2, 45, n_kv, max_seq, D)
            assert rc == 0
            torch.cuda.synchronize()
        assert torch.equal(ours.view(torch.int16) if kind == "half" else ours.view(torch.int32),
                           theirs.view(torch.int16) if kind == "half" else theirs.view(torch.int32)), kind
        assert ours.any()
