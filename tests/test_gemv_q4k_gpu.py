"""The layer graph's Q4_K GEMV (swamp-gpu/kernels/fused_attention.cu:858-925)
against the oracle's restatement and, when oracle/_ref is built, the
reference's own gpu_gemv_q4k compiled from its source: relative error 1e-5
of the row norm (different summation order), batched and single-row forms,
row counts that are not multiples of 32, the O-projection shape (2048 x 2048)
and a wide FFN-down shape (n_blocks 22)."""
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


def _weights(rng, n_rows, n_blocks):
    w = rng.integers(0, 256, (n_blocks, n_rows, 144), dtype=np.uint8)
    d = (rng.random((n_blocks, n_rows)) * 0.02).astype(np.float16)
    dm = (rng.standard_normal((n_blocks, n_rows)) * 0.01).astype(np.float16)
    w[:, :, 0:2] = d.view(np.uint8).reshape(n_blocks, n_rows, 2)
    w[:, :, 2:4] = dm.view(np.uint8).reshape(n_blocks, n_rows, 2)
    return w


def _close(got, want):
    scale = np.abs(want).max() + 1e-6
    return np.abs(got - want).max() / scale < 1e-5


@pytest.mark.parametrize("n_rows,n_blocks,batch", [(2048, 8, 1), (2048, 8, 7), (100, 3, 2), (256, 22, 1)])
def test_gemv_q4k_matches_oracle(cuda_device, n_rows, n_blocks, batch):
    rng = np.random.default_rng(n_rows + n_blocks + batch)
    w = _weights(rng, n_rows, n_blocks)
    x = rng.standard_normal((batch, n_blocks * 256)).astype(np.float32)
    got = A.gemv_q4k(torch.from_numpy(w).to(cuda_device), torch.from_numpy(x).to(cuda_device), n_rows)
    torch.cuda.synchronize()
    for b in range(batch):
        assert _close(got[b].cpu().numpy(), O.gemv_q4k(w, x[b], n_rows, n_blocks))


@pytest.mark.skipif(not os.path.exists(REF), reason="reference CUDA not built (make -C oracle ref)")
def test_gemv_q4k_matches_reference_cuda(cuda_device):
    R = C.CDLL(REF)
    R.gpu_gemv_q4k.restype = None
    R.gpu_gemv_q4k.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    rng = np.random.default_rng(9)
    n_rows, n_blocks = 2048, 8
    w = torch.from_numpy(_weights(rng, n_rows, n_blocks)).to(cuda_device)
    x = torch.from_numpy(rng.standard_normal(n_blocks * 256).astype(np.float32)).to(cuda_device)
    ours = torch.zeros(n_rows, device=cuda_device)
    theirs = torch.zeros(n_rows, device=cuda_device)
    A.lib().gpu_gemv_q4k(w.data_ptr(), x.data_ptr(), ours.data_ptr(), n_rows, n_blocks, None)
    R.gpu_gemv_q4k(w.data_ptr(), x.data_ptr(), theirs.data_ptr(), n_rows, n_blocks, None)
    torch.cuda.synchronize()
    assert _close(ours.cpu().numpy(), theirs.cpu().numpy())
    assert _close(theirs.cpu().numpy(), O.gemv_q4k(w.cpu().numpy(), x.cpu().numpy(), n_rows, n_blocks))
