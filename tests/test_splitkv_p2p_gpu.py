"""The fused split-KV exchange on one GPU (the multi-GPU run is
tests/test_splitkv_multi_gpu.py):

  * world 1: nyion_attn_decode_q4_splitkv equals partial + LSE combine, over
    consecutive steps (the mailbox halves alternate);
  * a rank whose peer never raises its flags: the bounded wait runs out
    (100 ms), the device error word reports a wait timeout, the call returns
    and the context stays usable.  Nothing else runs on the GPU meanwhile: the
    flag it waits for is simply never written.
"""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu
N_KV, D, PT, H = 4, 64, 16, 32


def _case(T, B, dev, seed):
    rng = np.random.default_rng(seed)
    src = rng.standard_normal((B, T, N_KV, 2, D), dtype=np.float32)
    q4 = O.q4_quantize_rows(src, D)
    mp = (T + PT - 1) // PT
    pool = np.zeros((B * mp, N_KV, 2, PT, 40), np.uint8)
    for b in range(B):
        for t in range(T):
            pool[b * mp + t // PT, :, :, t % PT] = q4[b, t]
    table = np.arange(B * mp, dtype=np.int32).reshape(B, mp)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    return (torch.from_numpy(q).to(dev), torch.from_numpy(pool).to(dev), torch.from_numpy(table).to(dev),
            q, pool, table)


@pytest.mark.parametrize("T,B", [(5000, 1), (1300, 3)])
def test_world1_equals_collective_path(cuda_device, T, B):
    dq, dp, dt, q, pool, table = _case(T, B, cuda_device, T + B)
    want = A.lse_combine(A.decode_q4_partial(dq, dp, dt, u_begin=0, u_end=T)[None])
    mb = A.Mailbox(B, H)
    try:
        ws = A.Q4Workspace(B, device=cuda_device)
        for _ in range(3):
            got = A.decode_q4_splitkv(dq, dp, dt, 0, T, [mb.ptr], 0, workspace=ws)
            torch.cuda.synchronize()
            assert (got - want).abs().max().item() < 1e-5
    finally:
        mb.free()
    ref = O.lse_combine(O.decode_q4_partial(q, pool, table, 0, T, N_KV, D, PT, threads=8)[None])
    assert np.abs(got.cpu().numpy() - ref).max() < 1e-3
    assert A.device_error() == 0


def test_peer_that_never_writes_times_out(cuda_device):
    dq, dp, dt, *_ = _case(2000, 1, cuda_device, 7)
    mine, silent = A.Mailbox(1, H), A.Mailbox(1, H)
    try:
        A.device_error()                       # clear
        A.decode_q4_splitkv(dq, dp, dt, 0, 1000, [mine.ptr, silent.ptr], 0, timeout_ms=100)
        torch.cuda.synchronize()
        assert A.device_error() & 2            # NYION_DEVERR_WAIT_TIMEOUT
        # the context is still usable
        x = torch.ones(4, device=cuda_device) * 2
        assert x.sum().item() == 8.0
    finally:
        mine.free()
        silent.free()
