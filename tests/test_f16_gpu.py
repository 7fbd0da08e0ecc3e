"""GPU parity of the f16-cache decode (contiguous half cache and the
layer-graph ring node) against the CPU oracle, at max-abs 1e-3.

f16 values are exact in f32, so the oracle runs on pages holding the same
values widened to f32 (the math of ops.rs:170-278 over tokens [0, n)).
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


def _oracle(q, k, v, n):
    """q [H][D]; k, v [n_kv][>=n][D] (any float dtype) -> oracle over tokens [0, n)."""
    k = k.float().numpy()[:, :n]
    v = v.float().numpy()[:, :n]
    pages = (n + PT - 1) // PT
    pool = np.zeros((pages, N_KV, 2, PT, D), np.float32)
    for t in range(n):
        pool[t // PT, :, 0, t % PT] = k[:, t]
        pool[t // PT, :, 1, t % PT] = v[:, t]
    table = np.arange(pages, dtype=np.int32)[None]
    return O.decode_paged_f32(q.numpy()[None], pool, table, np.array([n], np.int32), N_KV, D, PT, threads=8)[0]


def _case(stride, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(H, D, generator=g)
    k = torch.randn(N_KV, stride, D, generator=g).half()
    v = torch.randn(N_KV, stride, D, generator=g).half()
    return q, k, v


@pytest.mark.parametrize("seq_len,stride", [(1, 1), (31, 32), (33, 40), (256, 256), (257, 300), (4096, 4096),
                                            (20000, 20480)])
def test_contig_f16_vs_oracle(cuda_device, seq_len, stride):
    q, k, v = _case(stride, seq_len)
    got = A.decode_contig_f16(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), seq_len).cpu().numpy()
    assert np.abs(got - _oracle(q, k, v, seq_len)).max() < TOL


def test_reference_half_abi_and_graph(cuda_device):
    q, k, v = _case(1024, 7)
    dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    want = _oracle(q, k, v, 1000)
    out = torch.zeros(H, D, device=cuda_device)
    torch.cuda.synchronize()
    assert A.lib().gpu_attention_streamed_half(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(),
                                               H, N_KV, 1000, D, 1024, None) == 0
    torch.cuda.synchronize()
    assert np.abs(out.cpu().numpy() - want).max() < TOL
    out.zero_()
    gh = A.lib().gpu_graph_create_attention_half(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), None,
                                                 out.data_ptr(), H, N_KV, 1000, D, 1024)
    assert gh
    try:
        s = torch.cuda.Stream()
        for _ in range(3):
            assert A.lib().gpu_graph_replay_attention(gh, C.c_void_p(s.cuda_stream)) == 0
        s.synchronize()
    finally:
        A.lib().gpu_graph_destroy(gh)
    assert np.abs(out.cpu().numpy() - want).max() < TOL


def test_ring_f16_device_length_in_one_graph(cuda_device):
    """One captured graph, replayed while the device-side length grows past the
    window (the length is clamped to the window, every slot then valid)."""
    W = 512
    q, k, v = _case(W, 11)
    dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    d_len = torch.ones(1, dtype=torch.int32, device=cuda_device)
    out = torch.zeros(H, D, device=cuda_device)
    ws = A.F16Workspace(H, W, device=cuda_device)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        A.decode_ring_f16(dq, dk, dv, d_len, out=out, workspace=ws, stream=s)     # eager once
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            A.decode_ring_f16(dq, dk, dv, d_len, out=out, workspace=ws, stream=s)
    for n in [1, 7, 100, 511, 512, 513, 5000]:
        with torch.cuda.stream(s):
            d_len.fill_(n)                               # ordered before the replay on s
            g.replay()
        s.synchronize()
        assert np.abs(out.cpu().numpy() - _oracle(q, k, v, min(n, W))).max() < TOL, n
    del g
    assert A.device_error() == 0


def test_f16_rejects_bad_arguments(cuda_device):
    q, k, v = _case(600, 3)
    dq, dk, dv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
    with pytest.raises(A.NyionError):
        A.decode_contig_f16(dq, dk, dv, 601)           # seq_len > stride
    small = A.F16Workspace(H, 8, device=cuda_device)   # one 256-token split; 600 tokens need three
    with pytest.raises(A.NyionError):
        A.decode_contig_f16(dq, dk, dv, 600, workspace=small)
