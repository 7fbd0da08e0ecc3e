"""GPU versions of the swamp-kernels C ABIs on the attention path, against
the CPU oracle: the Q16.16 softmax (bit-exact, swamp-kernels/src/lib.rs:97-223)
and the Stokes KV store (contents after evictions, lib.rs:27-85)."""
import numpy as np
import pytest
import torch

import nyion_rs_b200.attn as A
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,T,scale", [(1, 1.0, 1.0), (15, 1.0, 3.0), (16, 0.7, 3.0), (17, 1.0, 3.0),
                                       (1000, 1.3, 5.0), (32000, 1.0, 8.0), (128257, 0.8, 10.0),
                                       (4096, 1e-9, 1.0), (500, 2.0, 1e-3)])
def test_softmax_padic_bit_exact(cuda_device, n, T, scale):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * scale).astype(np.float32)
    want = O.softmax_padic(x, T)
    got = A.softmax_padic(torch.from_numpy(x).to(cuda_device), T).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_exp_q16_16_whole_domain_bit_exact(cuda_device):
    """Every input of exp_q16_16 that is neither clamped to 0 (below -655360)
    nor to 65536 (>= 0), plus both clamps and the i32 extremes: the device
    function equals the oracle (glibc expf, as Rust's f32::exp) bit for bit."""
    x = np.concatenate([np.arange(-655362, 3, dtype=np.int32),
                        np.array([-(2 ** 31), 2 ** 31 - 1, -(2 ** 20), 1 << 20], np.int32)])
    want = O.exp_q16_16_many(x)
    got = A.exp_q16_16(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x = {x[bad[:5]]}"
    assert want[x == 0][0] == 65536 and want[x == -655361][0] == 0


@pytest.mark.parametrize("seed", [0, 1])
def test_softmax_padic_normalisation_small_n(cuda_device, seed):
    """Normalisation for every length 1..64 (both sides of the 16-wide block
    boundary and the tail rule), bit-exact."""
    rng = np.random.default_rng(100 + seed)
    for n in range(1, 65):
        x = (rng.standard_normal(n) * (1 + 4 * seed)).astype(np.float32)
        want = O.softmax_padic(x, 1.0)
        got = A.softmax_padic(torch.from_numpy(x).to(cuda_device), 1.0).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), n


def test_softmax_padic_extremes_and_host_abi(cuda_device):
    x = np.array([0.0, -1e30, 1e30, float("nan"), -5.0, 40000.0, -40000.0] * 5, np.float32)
    want = O.softmax_padic(x, 1.0)
    got = A.softmax_padic(torch.from_numpy(x).to(cuda_device), 1.0).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # reference-named host entry
    y = np.random.default_rng(3).standard_normal(777).astype(np.float32)
    out = np.zeros_like(y)
    A.lib().mojo_softmax_padic(y.ctypes.data, out.ctypes.data, y.size, 1.0)
    assert np.array_equal(out.view(np.uint32), O.softmax_padic(y, 1.0).view(np.uint32))
    A.lib().mojo_softmax_padic(None, None, 0, 1.0)     # silent, like the reference


def test_stokes_store_matches_oracle_after_evictions(cuda_device):
    hd, n = 64, 4500
    rng = np.random.default_rng(17)
    ks = rng.standard_normal((n, hd)).astype(np.float32)
    vs = rng.standard_normal((n, hd)).astype(np.float32)
    sc = rng.integers(0, 50, n).astype(np.float32)     # ties: the first minimum goes
    ref = O.Stokes(hd)
    st = A.StokesStore(hd)
    try:
        for i in range(n):
            ref.append(i, ks[i], vs[i], sc[i])
            st.append(i, ks[i], vs[i], sc[i])
        rk, rv, _ = ref.arrays()
        kp, vp, cnt = st.view()
        assert cnt == len(ref) == 4096
        k_dev = torch.empty(cnt * hd, device=cuda_device)
        v_dev = torch.empty(cnt * hd, device=cuda_device)
        torch.cuda.synchronize()
        _copy_from_ptr(k_dev, kp)
        _copy_from_ptr(v_dev, vp)
        assert np.array_equal(k_dev.cpu().numpy().reshape(cnt, hd), rk)
        assert np.array_equal(v_dev.cpu().numpy().reshape(cnt, hd), rv)
    finally:
        st.close()
        ref.close()


def _copy_from_ptr(dst, src_ptr):
    """Copy dst.numel() floats from a raw device pointer into dst."""
    import cuda.bindings.runtime as rt   # cuda-python
    err, = rt.cudaMemcpy(dst.data_ptr(), src_ptr, dst.numel() * 4, rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
    assert err == rt.cudaError_t.cudaSuccess
