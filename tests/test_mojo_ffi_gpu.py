"""The Mojo FFI entry `sparse_attention_q4` (swamp-gpu/kernels/attention.mojo:
122-152, Rust binding swamp-gpu/src/mojo.rs:5, 65-97) on the GPU against the
oracle's restatement of the Mojo kernel as written (tiles of 64, earlier
tiles not rescaled, weights < 1e-8 skipped): max-abs 1e-4, host pointers in
and out, as the Rust caller passes them."""
import numpy as np
import pytest

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,hd,n", [(32, 64, 1), (32, 64, 64), (32, 64, 65), (8, 64, 4224), (4, 32, 300),
                                    (4, 96, 130)])
def test_sparse_attention_q4_ffi(cuda_device, H, hd, n):
    rng = np.random.default_rng(H * hd + n)
    T = max(500, n)
    kq = O.q4_quantize_rows(rng.standard_normal((T, hd)).astype(np.float32), hd)
    vq = O.q4_quantize_rows(rng.standard_normal((T, hd)).astype(np.float32), hd)
    km, vm = O.mojo_rows_from_q4(kq), O.mojo_rows_from_q4(vq)
    q = rng.standard_normal((H, hd)).astype(np.float32)
    pos = rng.integers(0, T, n).astype(np.int32)
    out = np.full((H, hd), np.nan, np.float32)
    A.lib().sparse_attention_q4(q.ctypes.data, km.ctypes.data, vm.ctypes.data, pos.ctypes.data, out.ctypes.data,
                                H, hd, n, 4096, H * hd * 4)
    want = O.mojo_sparse_attention_q4(q, km, vm, pos)
    assert np.abs(out - want).max() < 1e-4


def test_empty_position_set_gives_zeros(cuda_device):
    q = np.ones((2, 64), np.float32)
    out = np.full((2, 64), 7.0, np.float32)
    dummy = np.zeros(40, np.float32)
    pos = np.zeros(1, np.int32)
    A.lib().sparse_attention_q4(q.ctypes.data, dummy.ctypes.data, dummy.ctypes.data, pos.ctypes.data,
                                out.ctypes.data, 2, 64, 0, 0, 0)
    assert not out.any()
