"""Attention outputs pinned against the reference's own CUDA decode.

oracle/_ref/libref_fused_attention.so is swamp-gpu/kernels/fused_attention.cu
compiled from its source (oracle/Makefile, target `ref`).  Its
gpu_attention_device (fused_attention.cu:194-243: kernel_scores +
kernel_softmax_weighted_sum over a contiguous [n_kv][stride][64] fp32 cache)
is run on the same seeded inputs as

  - the CPU oracle (pages cut from the same cache): pins the oracle's
    attention output, which the reference's Rust tests never check;
  - this library's gpu_attention_device (same name and arguments): the
    drop-in itself.

The reference kernel keeps all scores in 48 KB of shared memory, so it is
only run for seq_len <= 12000 (longer contexts fail its launch).
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "libref_fused_attention.so")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(REF), reason="reference CUDA not built (make -C oracle ref)")]
H, N_KV, D, PT = 32, 4, 64, 16


def _ref():
    L = C.CDLL(REF)   # RTLD_LOCAL: its same-named exports never bind to ours
    L.gpu_attention_device.restype = C.c_int
    L.gpu_attention_device.argtypes = [C.c_void_p] * 4 + [C.c_int] * 5
    L.gpu_attention_streamed_half.restype = C.c_int
    L.gpu_attention_streamed_half.argtypes = [C.c_void_p] * 4 + [C.c_int] * 5 + [C.c_void_p]
    return L


def _pages(k, v, seq_len):
    """Cut a contiguous [n_kv][stride][D] cache into a 16-token page pool."""
    pages = (seq_len + PT - 1) // PT
    pool = np.zeros((pages, N_KV, 2, PT, D), np.float32)
    for t in range(seq_len):
        pool[t // PT, :, 0, t % PT] = k[:, t]
        pool[t // PT, :, 1, t % PT] = v[:, t]
    return pool, np.arange(pages, dtype=np.int32)[None]


@pytest.mark.parametrize("seq_len,stride", [(1, 1), (37, 64), (128, 128), (1000, 1024), (4096, 4096),
                                            (12000, 12000)])
def test_reference_cuda_pins_oracle_and_product(cuda_device, seq_len, stride):
    g = torch.Generator().manual_seed(seq_len)
    q = torch.randn(H, D, generator=g)
    k = torch.randn(N_KV, stride, D, generator=g)
    v = torch.randn(N_KV, stride, D, generator=g)
    dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    ref_out = torch.zeros(H, D, device=cuda_device)
    ours = torch.zeros(H, D, device=cuda_device)
    torch.cuda.synchronize()
    assert _ref().gpu_attention_device(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ref_out.data_ptr(),
                                       H, N_KV, seq_len, D, stride) == 0
    torch.cuda.synchronize()
    assert A.lib().gpu_attention_device(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ours.data_ptr(),
                                        H, N_KV, seq_len, D, stride) == 0
    torch.cuda.synchronize()
    pool, table = _pages(k.numpy(), v.numpy(), seq_len)
    want = O.decode_paged_f32(q.numpy()[None], pool, table, np.array([seq_len], np.int32), N_KV, D, PT,
                              threads=8)[0]
    ref_np, ours_np = ref_out.cpu().numpy(), ours.cpu().numpy()
    assert np.abs(ref_np - want).max() < 1e-4        # oracle == reference CUDA
    assert np.abs(ours_np - ref_np).max() < 1e-3     # product == reference CUDA
    assert np.abs(ours_np - want).max() < 1e-3


@pytest.mark.parametrize("seq_len,stride", [(1, 8), (300, 300), (4096, 4096), (12000, 12000)])
def test_reference_cuda_half_matches_product(cuda_device, seq_len, stride):
    """gpu_attention_streamed_half (fused_attention.cu:534-582) on an f16 cache."""
    g = torch.Generator().manual_seed(seq_len + 1)
    q = torch.randn(H, D, generator=g)
    k = torch.randn(N_KV, stride, D, generator=g).half()
    v = torch.randn(N_KV, stride, D, generator=g).half()
    dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    ref_out = torch.zeros(H, D, device=cuda_device)
    ours = torch.zeros(H, D, device=cuda_device)
    torch.cuda.synchronize()
    assert _ref().gpu_attention_streamed_half(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ref_out.data_ptr(),
                                              H, N_KV, seq_len, D, stride, None) == 0
    torch.cuda.synchronize()
    assert A.lib().gpu_attention_streamed_half(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ours.data_ptr(),
                                               H, N_KV, seq_len, D, stride, None) == 0
    torch.cuda.synchronize()
    pool, table = _pages(k.float().numpy(), v.float().numpy(), seq_len)
    want = O.decode_paged_f32(q.numpy()[None], pool, table, np.array([seq_len], np.int32), N_KV, D, PT,
                              threads=8)[0]
    ref_np, ours_np = ref_out.cpu().numpy(), ours.cpu().numpy()
    assert np.abs(ref_np - want).max() < 1e-4
    assert np.abs(ours_np - ref_np).max() < 1e-3
