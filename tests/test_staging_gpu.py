"""GPU checks of the host staging copies (staging.cu): pinned host -> device
-> pinned host round trips of aligned and ragged sizes and offsets, byte
exact; overlapping ranges and pageable memory are refused with an error
status, not run; copies captured in a CUDA graph replay correctly."""
import ctypes as C

import pytest
import torch

import nyion_rs_b200.attn as A

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,off", [(16, 0), (1, 0), (4097, 0), (262147, 0), (1000, 3), (65536, 5), (48, 16)])
def test_round_trip_bytes(cuda_device, n, off):
    g = torch.Generator().manual_seed(n + off)
    src = torch.randint(0, 256, (n + off,), dtype=torch.uint8, generator=g).pin_memory()
    back = torch.zeros(n + off, dtype=torch.uint8).pin_memory()
    dev = torch.zeros(n + 7, dtype=torch.uint8, device=cuda_device)
    s = torch.cuda.Stream()
    A.copy_async(dev[:n], src[off:], stream=s)
    A.copy_async(back[off:], dev[:n], stream=s)
    s.synchronize()
    assert torch.equal(back[off:], src[off:])
    assert torch.equal(dev[:n].cpu(), src[off:])
    assert (dev[n:].cpu() == 0).all()                   # nothing past the range


def test_refusals(cuda_device):
    L = A.lib()
    d = torch.zeros(1024, dtype=torch.uint8, device=cuda_device)
    s = torch.cuda.Stream()
    # overlapping ranges: refused before any launch (-1 = NYION_ERR_INVALID)
    assert L.nyion_attn_copy_async(d.data_ptr() + 8, d.data_ptr(), 64, s.cuda_stream) == -1
    assert L.nyion_attn_copy_async(0, d.data_ptr(), 64, s.cuda_stream) == -1
    assert L.nyion_attn_copy_async(0, 0, 0, s.cuda_stream) == 0            # empty copy
    pageable = torch.zeros(64, dtype=torch.uint8)
    out = C.c_void_p()
    assert L.nyion_attn_host_map(pageable.data_ptr(), C.byref(out)) != 0
    with pytest.raises(ValueError):
        A.device_address(pageable)


def test_graph_captured_copies(cuda_device):
    """Per-layer staging in a captured graph (the shape of the end-to-end
    bench leg): host rows in on one stream, device work, rows out on another."""
    layers, rows = 6, 32 * 32 * 64
    src = torch.randn(layers, rows).pin_memory()
    dst = torch.zeros(layers, rows).pin_memory()
    dev = torch.zeros(layers, rows, device=cuda_device)
    s, h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    sa, da = A.device_address(src), A.device_address(dst)
    rb = rows * 4

    def step():
        start = torch.cuda.Event()
        start.record(s)
        h2d.wait_event(start)
        d2h.wait_event(start)
        for l in range(layers):
            A.copy_async(dev[l], src[l], stream=h2d, src_addr=sa + l * rb)
            e = torch.cuda.Event()
            e.record(h2d)
            s.wait_event(e)
            with torch.cuda.stream(s):
                dev[l].mul_(2.0)
            e2 = torch.cuda.Event()
            e2.record(s)
            d2h.wait_event(e2)
            A.copy_async(dst[l], dev[l], stream=d2h, dst_addr=da + l * rb)
        end = torch.cuda.Event()
        end.record(d2h)
        s.wait_event(end)

    with torch.cuda.stream(s):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        step()
    dst.zero_()
    src.copy_(torch.randn(layers, rows))
    with torch.cuda.stream(s):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(dst, src * 2.0)
    del g
