"""Timing beside the reference's own CUDA decode (fused_attention.cu compiled
from its source into oracle/_ref): the same contiguous fp32 / f16 caches, each
side's CUDA-graph API (gpu_graph_create_attention[_half] + replay, scores
buffer preallocated for the reference), 50 replays queued behind a short spin so that the
events time the device, not the host's launch rate.
The outputs are checked against each other (1e-3); the times are printed
(`pytest -s`), not asserted."""
import ctypes as C
import os

import pytest
import torch

import nyion_rs_b200.attn as A

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "libref_fused_attention.so")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(REF), reason="reference CUDA not built (make -C oracle ref)")]
H, N_KV, D = 32, 4, 64


def _bind(L):
    for name in ("gpu_graph_create_attention", "gpu_graph_create_attention_half"):
        f = getattr(L, name)
        f.restype = C.c_void_p
        f.argtypes = [C.c_void_p] * 5 + [C.c_int] * 5
    L.gpu_graph_replay_attention.restype = C.c_int
    L.gpu_graph_replay_attention.argtypes = [C.c_void_p, C.c_void_p]
    L.gpu_graph_destroy.restype = None
    L.gpu_graph_destroy.argtypes = [C.c_void_p]
    return L


def _time(L, handle, stream, reps=50):
    for _ in range(3):
        assert L.gpu_graph_replay_attention(handle, stream.cuda_stream) == 0
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(4_000_000)   # ~2 ms: every replay is queued before the first runs
    e0.record(stream)
    for _ in range(reps):
        L.gpu_graph_replay_attention(handle, stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3


@pytest.mark.parametrize("half", [False, True])
@pytest.mark.parametrize("seq_len", [1024, 4096, 12000])
def test_graph_decode_time_beside_reference_cuda(cuda_device, half, seq_len):
    R, L = _bind(C.CDLL(REF)), _bind(A.lib())
    g = torch.Generator().manual_seed(seq_len)
    dt = torch.float16 if half else torch.float32
    q = torch.randn(H, D, generator=g).to(cuda_device)
    k = torch.randn(N_KV, seq_len, D, generator=g).to(dt).to(cuda_device)
    v = torch.randn(N_KV, seq_len, D, generator=g).to(dt).to(cuda_device)
    scores = torch.empty(H, seq_len, device=cuda_device)
    outs, times = {}, {}
    s = torch.cuda.Stream()
    for name, lib in (("reference", R), ("ours", L)):
        out = torch.zeros(H, D, device=cuda_device)
        create = lib.gpu_graph_create_attention_half if half else lib.gpu_graph_create_attention
        h = create(q.data_ptr(), k.data_ptr(), v.data_ptr(), scores.data_ptr(), out.data_ptr(), H, N_KV, seq_len, D,
                   seq_len)
        assert h
        try:
            times[name] = _time(lib, h, s)
        finally:
            lib.gpu_graph_destroy(h)
        outs[name] = out
    assert (outs["ours"] - outs["reference"]).abs().max().item() < 1e-3
    kv_bytes = 2 * N_KV * seq_len * D * (2 if half else 4)
    print(f"\n{'f16' if half else 'f32'} ctx {seq_len}: reference CUDA {times['reference']:.1f} us, "
          f"ours {times['ours']:.1f} us ({times['reference'] / times['ours']:.1f}x), "
          f"ours {kv_bytes / times['ours'] / 1e3:.0f} GB/s")
