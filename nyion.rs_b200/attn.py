"""Host-side binding of libnyion_attn.so (ctypes) with torch tensors as buffers.

This is the Python caller of the C ABI declared in include/nyion_attn.h.  It
owns no maths: every function checks shapes, passes raw device pointers and
the current torch stream to the library, and raises NyionError on a non-zero
status.  There is no CPU fallback: without the library or a CUDA device the
calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "libnyion_attn.so")
HEADER_DIR = os.path.join(ROOT, "include")

NYION_OK = 0
_lib = None


class NyionError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"nyion status {status}: {msg}")
        self.status = status


def lib() -> C.CDLL:
    """Loads the library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python nyion.rs_b200/build.py` "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        vp, i32, i64, f32, sz = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t
        sig = {
            "nyion_attn_version": (i32, []),
            "nyion_attn_last_error": (C.c_char_p, []),
            "nyion_attn_device_error": (i32, [vp, C.POINTER(i32)]),
            "nyion_attn_decode_workspace_size": (sz, [i32, i32, i32, i32]),
            "nyion_attn_workspace_reset": (i32, [vp, sz, vp]),
            "nyion_attn_host_map": (i32, [vp, C.POINTER(vp)]),
            "nyion_attn_copy_async": (i32, [vp, vp, sz, vp]),
            "nyion_attn_arena_create": (i32, [sz, C.POINTER(vp)]),
            "nyion_attn_arena_destroy": (i32, [vp]),
            "nyion_attn_arena_allocate_device": (i32, [vp, sz, C.POINTER(C.c_uint64), C.POINTER(vp)]),
            "nyion_attn_arena_allocate_unified": (i32, [vp, sz, C.POINTER(C.c_uint64), C.POINTER(vp)]),
            "nyion_attn_arena_free": (i32, [vp, C.c_uint64]),
            "nyion_attn_arena_upload": (i32, [vp, C.c_uint64, vp, sz, vp]),
            "nyion_attn_arena_download": (i32, [vp, C.c_uint64, vp, sz, vp]),
            "nyion_attn_arena_info": (i32, [vp, C.POINTER(sz), C.POINTER(sz), C.POINTER(sz)]),
            "nyion_attn_decode_paged_f32": (i32, [vp, vp, i64, vp, i32, vp, vp, i32, i32, i32, i32,
                                                  i32, f32, vp, sz, vp]),
            "nyion_attn_decode_zoned_f32": (i32, [vp, vp, vp, vp, i64, i32, i32, i64, i64, i32, i32,
                                                  i32, vp]),
            "nyion_attn_quantize_q4": (i32, [vp, vp, i64, i32, vp]),
            "nyion_attn_dequant_q4": (i32, [vp, vp, i64, i32, vp]),
            "nyion_attn_q4_workspace_size": (sz, [i32]),
            "nyion_attn_decode_q4_partial": (i32, [vp, vp, i64, vp, i32, vp, vp, i32, i32, vp, i32, i32,
                                                   i32, i32, i32, f32, vp, sz, vp]),
            "nyion_attn_lse_combine": (i32, [vp, i32, i64, i32, vp, vp]),
            "nyion_attn_decode_q4_window_ring": (i32, [vp, vp, i64, vp, i32, vp, vp, i32, i32, vp, i32,
                                                       i32, i32, i32, i32, f32, vp, sz, vp]),
            "nyion_attn_prefill_paged_bf16": (i32, [vp, vp, i64, vp, i32, i64, i64, vp, i32, i32, i32,
                                                    i32, f32, vp]),
            "gpu_attention_device": (C.c_int,[vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                               C.c_int]),
            "gpu_attention_streamed": (C.c_int, [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int,
                                                 C.c_int, C.c_int, vp]),
            "gpu_attention_forward": (C.c_int, [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int]),
            "gpu_graph_create_attention": (vp, [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int,
                                                C.c_int, C.c_int]),
            "gpu_graph_replay_attention": (C.c_int, [vp, vp]),
            "gpu_graph_destroy": (None, [vp]),
            "nyion_attn_f16_workspace_size": (sz, [i32, i32]),
            "nyion_attn_positions_workspace_size": (sz, [i32, i32, i32]),
            "nyion_attn_decode_zoned_f32_tracked": (i32, [vp, vp, vp, vp, i64, i32, i32, i64, i64, i32, i32, i32,
                                                          vp, vp]),
            "nyion_attn_cold_q4_page_bytes": (sz, [i32, i32, i32, i32]),
            "nyion_attn_cold_slot_offset": (i64, [i64, i32, i32, i32, i32]),
            "nyion_attn_cold_to_pool": (i32, [vp, i32, i32, i32, i32, vp, vp, i64, vp]),
            "nyion_attn_pool_to_cold": (i32, [vp, vp, i32, i32, i32, i32, i64, vp, vp]),
            "sparse_attention_q4": (None, [C.c_uint64] * 5 + [i32] * 5),
            "nyion_attn_gemv_q4k": (i32, [vp, vp, vp, i32, i32, i32, vp]),
            "gpu_gemv_q4k": (None, [vp, vp, vp, C.c_int, C.c_int, vp]),
            "nyion_attn_rope_table_bytes": (sz, [i32, i32]),
            "nyion_attn_rope_table": (i32, [vp, i32, i32, vp]),
            "nyion_attn_kv_write_paged": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, i32, vp, i32, i64, vp, vp,
                                                vp, vp, vp, i32, vp]),
            "nyion_attn_kv_write_ring_f16": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, i32, vp]),
            "gpu_alloc_kv_buffer": (vp, [C.c_int, C.c_int, C.c_int, C.POINTER(sz)]),
            "gpu_alloc_kv_buffer_half": (vp, [C.c_int, C.c_int, C.c_int, C.POINTER(sz)]),
            "gpu_copy_kv_to_buffer": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
            "gpu_copy_kv_layer": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, C.c_int]),
            "gpu_copy_kv_layer_async": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp]),
            "gpu_copy_kv_layer_async_half": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp]),
            "nyion_attn_decode_positions": (i32, [vp, vp, i32, i64, vp, i32, vp, vp, i32, vp, i32, i32, i32, i32,
                                                  i32, f32, vp, sz, vp]),
            "nyion_attn_sparse_q4_workspace_size": (sz, [i32, i32]),
            "nyion_attn_sparse_q4": (i32, [vp, vp, i64, vp, i32, vp, i32, i32, vp, i32, i32, i32, i32, i32, f32,
                                           vp, sz, vp]),
            "nyion_attn_softmax_padic": (i32, [vp, vp, i32, f32, vp]),
            "mojo_softmax_padic": (None, [vp, vp, C.c_int, f32]),
            "nyion_attn_exp_q16_16": (i32, [vp, vp, i64, vp]),
            "mojo_stokes_init": (vp, [C.c_int]),
            "mojo_stokes_append": (None, [vp, C.c_int, vp, vp, f32]),
            "mojo_stokes_free": (None, [vp]),
            "nyion_attn_stokes_view": (i32, [vp, C.POINTER(vp), C.POINTER(vp), C.POINTER(i32), C.POINTER(i32)]),
            "nyion_attn_splitkv_mailbox_bytes": (sz, [i32, i32]),
            "nyion_attn_mailbox_alloc": (i32, [sz, C.POINTER(vp)]),
            "nyion_attn_mailbox_free": (i32, [vp]),
            "nyion_attn_ipc_handle": (i32, [vp, C.c_char_p]),
            "nyion_attn_ipc_open": (i32, [C.c_char_p, C.POINTER(vp)]),
            "nyion_attn_ipc_close": (i32, [vp]),
            "nyion_attn_decode_q4_splitkv": (i32, [vp, vp, i64, vp, i32, i32, i32, vp, i32, i32, i32, i32, i32, f32,
                                                   C.POINTER(vp), i32, i32, i32, vp, sz, vp]),
            "nyion_attn_decode_contig_f16": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, vp, sz, vp]),
            "nyion_attn_decode_ring_f16": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, vp, sz, vp]),
            "gpu_attention_streamed_half": (C.c_int, [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                                      C.c_int, vp]),
            "gpu_graph_create_attention_half": (vp, [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int,
                                                     C.c_int, C.c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    m = lib().nyion_attn_last_error()
    return m.decode() if m else ""


def check(status: int) -> None:
    if status != NYION_OK:
        raise NyionError(status, last_error())


def declared_symbols() -> list[str]:
    """Function names declared in include/*.h (the exported ABI)."""
    names = []
    for fn in sorted(os.listdir(HEADER_DIR)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(HEADER_DIR, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", text):
            name = m.group(1)
            pre = text[max(0, m.start() - 40):m.start()]
            if name in ("if", "sizeof", "defined") or "#define" in pre.split("\n")[-1]:
                continue
            if re.search(r"(int32_t|int|void|size_t|char)\s*\**\s*$", pre):
                names.append(name)
    return sorted(set(names))


# ---------------------------------------------------------------------- torch glue
def _torch():
    import torch
    return torch


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream_ptr(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def device_address(t) -> int:
    """Address of tensor `t` as the device sees it: data_ptr() for a CUDA
    tensor, the mapped address (nyion_attn_host_map) for a pinned CPU tensor."""
    if t.is_cuda:
        return int(t.data_ptr())
    if not t.is_pinned():
        raise ValueError("device_address: a CPU tensor must be pinned (page-locked)")
    base = int(t.untyped_storage().data_ptr())
    d = C.c_void_p()
    check(lib().nyion_attn_host_map(base, C.byref(d)))
    return int(d.value) + (int(t.data_ptr()) - base)


def copy_async(dst, src, stream=None, dst_addr: int | None = None, src_addr: int | None = None) -> None:
    """dst <- src (same byte size, contiguous) by an SM kernel on `stream`;
    either may be a pinned CPU tensor.  dst_addr / src_addr: addresses from
    device_address() resolved beforehand (e.g. outside a CUDA graph capture)."""
    n = dst.numel() * dst.element_size()
    if n != src.numel() * src.element_size() or not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("copy_async: contiguous tensors of equal byte size required")
    check(lib().nyion_attn_copy_async(dst_addr if dst_addr is not None else device_address(dst),
                                      src_addr if src_addr is not None else device_address(src), n,
                                      _stream_ptr(stream)))


class Arena:
    """The HBM arena (nyion_attn_arena_*): the device side of the reference's
    HeterogeneousMemoryAllocator.  allocate() returns (handle, device address);
    upload / download move bytes between host numpy arrays and an allocation
    (synchronously unless a stream is given)."""

    def __init__(self, capacity: int):
        ptr = C.c_void_p()
        check(lib().nyion_attn_arena_create(capacity, C.byref(ptr)))
        self.ptr = ptr.value

    def allocate(self, size: int, unified: bool = False) -> tuple[int, int]:
        h, p = C.c_uint64(), C.c_void_p()
        fn = lib().nyion_attn_arena_allocate_unified if unified else lib().nyion_attn_arena_allocate_device
        check(fn(self.ptr, size, C.byref(h), C.byref(p)))
        return int(h.value), int(p.value)

    def free(self, handle: int) -> None:
        check(lib().nyion_attn_arena_free(self.ptr, handle))

    def upload(self, handle: int, data, stream=None) -> None:
        import numpy as np
        buf = np.ascontiguousarray(data)
        check(lib().nyion_attn_arena_upload(self.ptr, handle, buf.ctypes.data, buf.nbytes,
                                            _stream_ptr(stream) if stream is not None else None))

    def download(self, handle: int, out, stream=None) -> None:
        check(lib().nyion_attn_arena_download(self.ptr, handle, out.ctypes.data, out.nbytes,
                                              _stream_ptr(stream) if stream is not None else None))

    def info(self) -> tuple[int, int, int]:
        c, u, f = C.c_size_t(), C.c_size_t(), C.c_size_t()
        check(lib().nyion_attn_arena_info(self.ptr, C.byref(c), C.byref(u), C.byref(f)))
        return int(c.value), int(u.value), int(f.value)

    def close(self) -> None:
        if self.ptr:
            check(lib().nyion_attn_arena_destroy(self.ptr))
            self.ptr = None


class Workspace:
    """Device workspace for the decode entry points (zeroed once)."""

    def __init__(self, batch: int, n_kv_heads: int, n_heads: int, head_dim: int, device=None):
        torch = _torch()
        self.nbytes = int(lib().nyion_attn_decode_workspace_size(batch, n_kv_heads, n_heads, head_dim))
        self.buf = torch.zeros(self.nbytes, dtype=torch.uint8, device=device or "cuda")

    def ptr(self) -> int:
        return int(self.buf.data_ptr())


def decode_paged_f32(q, kv_pool, page_table, seq_lens, out=None, scale: float = 0.0,
                     workspace: Workspace | None = None, stream=None):
    """fp32 paged GQA decode (nyion_attn_decode_paged_f32).

    q [B, H, D] f32; kv_pool [P, n_kv, 2, 16, D] f32; page_table [B, max_pages]
    int32; seq_lens [B] int32 (device); returns out [B, H, D] f32.
    """
    torch = _torch()
    B, H, D = q.shape
    n_kv = kv_pool.shape[1]
    assert kv_pool.dtype == torch.float32 and q.dtype == torch.float32
    assert page_table.dtype == torch.int32 and seq_lens.dtype == torch.int32
    for t in (q, kv_pool, page_table, seq_lens):
        assert t.is_cuda and t.is_contiguous()
    if out is None:
        out = torch.empty_like(q)
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.ptr(), workspace.nbytes)
    check(lib().nyion_attn_decode_paged_f32(
        _ptr(q), _ptr(kv_pool), kv_pool.shape[0], _ptr(page_table), page_table.shape[1],
        _ptr(seq_lens), _ptr(out), B, H, n_kv, D, kv_pool.shape[3], float(scale), ws_ptr, ws_bytes,
        _stream_ptr(stream)))
    return out


def _zone_pages(k_arena, n_layers: int, n_kv: int, D: int) -> int:
    per_slot = n_layers * n_kv * D
    n = k_arena.numel()
    z0 = min(n // (per_slot * 32), 128)
    rest = n - z0 * per_slot * 32
    z1 = min(rest // (per_slot * 128), 992) if z0 == 128 else 0
    rest -= z1 * per_slot * 128
    z2 = rest // (per_slot * 1024) if z1 == 992 else 0
    return z0 + z1 + z2


def decode_zoned_f32(q, k_arena, v_arena, n_layers: int, layer: int, seq_len: int, q_pos: int,
                     out=None, stream=None, n_kv: int | None = None):
    """ops::attention over reference-layout zone pages (nyion_attn_decode_zoned_f32).

    q [H, D] f32; k_arena / v_arena: flat f32 arenas holding consecutive zone
    pages [n_layers][n_kv][slots][D]; returns out [H, D].  n_kv defaults to H / 8.
    """
    torch = _torch()
    H, D = q.shape
    n_kv = n_kv or H // 8
    if out is None:
        out = torch.empty_like(q)
    check(lib().nyion_attn_decode_zoned_f32(_ptr(out), _ptr(q), _ptr(k_arena), _ptr(v_arena),
                                            _zone_pages(k_arena, n_layers, n_kv, D), n_layers, layer, seq_len,
                                            q_pos, H, n_kv, D, _stream_ptr(stream)))
    return out


def decode_zoned_f32_tracked(q, k_arena, v_arena, n_layers: int, layer: int, seq_len: int, q_pos: int,
                             importance, out=None, stream=None):
    """ops::attention_tracked: decode_zoned_f32 plus importance[t] += sum_h p_h(t)
    (importance: float64 device tensor of seq_len)."""
    torch = _torch()
    H, D = q.shape
    n_kv = H // 8
    assert importance.dtype == torch.float64 and importance.numel() >= seq_len
    if out is None:
        out = torch.empty_like(q)
    check(lib().nyion_attn_decode_zoned_f32_tracked(
        _ptr(out), _ptr(q), _ptr(k_arena), _ptr(v_arena), _zone_pages(k_arena, n_layers, n_kv, D), n_layers,
        layer, seq_len, q_pos, H, n_kv, D, _ptr(importance), _stream_ptr(stream)))
    return out


def quantize_q4(src, stream=None):
    """Reference 4-bit quantizer (bit-exact): src [..., D] f32 -> [..., ceil(D/32)*20] uint8."""
    torch = _torch()
    D = src.shape[-1]
    nblk = (D + 31) // 32
    rows = src.numel() // D
    dst = torch.empty(src.shape[:-1] + (nblk * 20,), dtype=torch.uint8, device=src.device)
    check(lib().nyion_attn_quantize_q4(_ptr(src.contiguous()), _ptr(dst), rows, D, _stream_ptr(stream)))
    return dst


def dequant_q4(src, head_dim: int, stream=None):
    torch = _torch()
    rows = src.numel() // (((head_dim + 31) // 32) * 20)
    dst = torch.empty(src.shape[:-1] + (head_dim,), dtype=torch.float32, device=src.device)
    check(lib().nyion_attn_dequant_q4(_ptr(src.contiguous()), _ptr(dst), rows, head_dim, _stream_ptr(stream)))
    return dst


class Q4Workspace:
    def __init__(self, batch: int, extra: int = 0, device=None):
        torch = _torch()
        self.nbytes = int(lib().nyion_attn_q4_workspace_size(batch)) + extra
        self.buf = torch.zeros(self.nbytes, dtype=torch.uint8, device=device or "cuda")

    def ptr(self) -> int:
        return int(self.buf.data_ptr())


def decode_q4_partial(q, kv_pool, page_table, tok_begin=None, tok_end=None, u_begin=0, u_end=0,
                      part=None, scale: float = 0.0, workspace=None, stream=None):
    """Q4 paged decode partials [B, H, D+2] over per-sequence token ranges."""
    torch = _torch()
    B, H, D = q.shape
    if part is None:
        part = torch.empty(B, H, D + 2, dtype=torch.float32, device=q.device)
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.ptr(), workspace.nbytes)
    check(lib().nyion_attn_decode_q4_partial(
        _ptr(q), _ptr(kv_pool), kv_pool.shape[0], _ptr(page_table), page_table.shape[1],
        _ptr(tok_begin), _ptr(tok_end), u_begin, u_end, _ptr(part), B, H, kv_pool.shape[1], D,
        kv_pool.shape[3], float(scale), ws_ptr, ws_bytes, _stream_ptr(stream)))
    return part


def lse_combine(parts, out=None, stream=None):
    torch = _torch()
    G = parts.shape[0]
    D = parts.shape[-1] - 2
    rows = parts[0].numel() // (D + 2)
    if out is None:
        out = torch.empty(parts.shape[1:-1] + (D,), dtype=torch.float32, device=parts.device)
    check(lib().nyion_attn_lse_combine(_ptr(parts.contiguous()), G, rows, D, _ptr(out), _stream_ptr(stream)))
    return out


def decode_q4_window_ring(q, kv_pool, page_table, seq_lens, ring, window: int, out=None,
                          scale: float = 0.0, workspace=None, stream=None):
    """Config-3 decode: Q4 window + fp32 ring of the newest tokens."""
    torch = _torch()
    B, H, D = q.shape
    if out is None:
        out = torch.empty_like(q)
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.ptr(), workspace.nbytes)
    check(lib().nyion_attn_decode_q4_window_ring(
        _ptr(q), _ptr(kv_pool), kv_pool.shape[0], _ptr(page_table), page_table.shape[1],
        _ptr(seq_lens), _ptr(ring), ring.shape[3], window, _ptr(out), B, H, kv_pool.shape[1], D,
        kv_pool.shape[3], float(scale), ws_ptr, ws_bytes, _stream_ptr(stream)))
    return out


def window_ring_workspace(batch: int, n_heads: int = 32, head_dim: int = 64, device=None):
    return Q4Workspace(batch, extra=2 * batch * n_heads * (head_dim + 2) * 4 + 8 * batch + 256, device=device)


class RawWorkspace:
    """A zeroed device buffer of `nbytes` for the entries that take one."""

    def __init__(self, nbytes: int, device=None):
        torch = _torch()
        self.nbytes = int(nbytes)
        self.buf = torch.zeros(max(self.nbytes, 1), dtype=torch.uint8, device=device or "cuda")

    def ptr(self) -> int:
        return int(self.buf.data_ptr())


def decode_positions(q, kv_pool, page_table, positions, n_positions, out=None, scale: float = 0.0,
                     workspace=None, stream=None):
    """Attention over explicit per-sequence position lists (ops::attention_sparse /
    attention_fugu's position sets).  kv_pool is f32 [P, n_kv, 2, 16, D] or
    Q4 uint8 [P, n_kv, 2, 16, 40]; positions int32 [B, max_positions]."""
    torch = _torch()
    B, H, D = q.shape
    if out is None:
        out = torch.empty_like(q)
    fmt = 1 if kv_pool.dtype == torch.uint8 else 0
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.ptr(), workspace.nbytes)
    check(lib().nyion_attn_decode_positions(
        _ptr(q), _ptr(kv_pool), fmt, kv_pool.shape[0], _ptr(page_table), page_table.shape[1],
        _ptr(positions), _ptr(n_positions), positions.shape[1], _ptr(out), B, H, kv_pool.shape[1], D,
        kv_pool.shape[3], float(scale), ws_ptr, ws_bytes, _stream_ptr(stream)))
    return out


def positions_workspace(batch: int, n_heads: int, max_positions: int, device=None):
    return RawWorkspace(lib().nyion_attn_positions_workspace_size(batch, n_heads, max_positions), device)


def sparse_q4(q, kv_pool, page_table, seq_lens, window: int, global_stride: int, out=None,
              scale: float = 0.0, workspace=None, stream=None):
    """ops::attention_sparse_q4 on Q4 pages: window + every global_stride-th older token
    (at most 128); seq_lens[b] = min(q_pos, seq_len - 1) + 1."""
    torch = _torch()
    B, H, D = q.shape
    if out is None:
        out = torch.empty_like(q)
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.ptr(), workspace.nbytes)
    check(lib().nyion_attn_sparse_q4(
        _ptr(q), _ptr(kv_pool), kv_pool.shape[0], _ptr(page_table), page_table.shape[1], _ptr(seq_lens),
        int(window), int(global_stride), _ptr(out), B, H, kv_pool.shape[1], D, kv_pool.shape[3],
        float(scale), ws_ptr, ws_bytes, _stream_ptr(stream)))
    return out


def sparse_q4_workspace(batch: int, n_heads: int = 32, device=None):
    return RawWorkspace(lib().nyion_attn_sparse_q4_workspace_size(batch, n_heads), device)


def cold_to_pool(slot, block_slots: int, layer_pools, page_ids, stream=None):
    """Scatter one reference cold slot (uint8, HBM or pinned host) into per-layer
    4-bit pools (list of [P, n_kv, 2, 16, 40] uint8 tensors); page_ids int32
    [n_layers, block_slots / 16] on the device."""
    n_layers = len(layer_pools)
    n_kv = layer_pools[0].shape[1]
    ptrs = (C.c_void_p * n_layers)(*[p.data_ptr() for p in layer_pools])
    check(lib().nyion_attn_cold_to_pool(_ptr(slot), block_slots, n_layers, n_kv, 64, ptrs, _ptr(page_ids),
                                        layer_pools[0].shape[0], _stream_ptr(stream)))


def pool_to_cold(layer_pools, page_ids, block_slots: int, slot, stream=None):
    n_layers = len(layer_pools)
    n_kv = layer_pools[0].shape[1]
    ptrs = (C.c_void_p * n_layers)(*[p.data_ptr() for p in layer_pools])
    check(lib().nyion_attn_pool_to_cold(ptrs, _ptr(page_ids), block_slots, n_layers, n_kv, 64,
                                        layer_pools[0].shape[0], _ptr(slot), _stream_ptr(stream)))


def cold_q4_page_bytes(block_slots: int, n_layers: int, n_kv: int, head_dim: int = 64) -> int:
    return int(lib().nyion_attn_cold_q4_page_bytes(block_slots, n_layers, n_kv, head_dim))


def gemv_q4k(w, x, n_rows: int, out=None, stream=None):
    """Q4_K GEMV of the layer graph: w uint8 column-major super-blocks, x [B, n_cols] f32."""
    torch = _torch()
    x2 = x.reshape(-1, x.shape[-1])
    n_blocks = x2.shape[1] // 256
    if out is None:
        out = torch.empty(x2.shape[0], n_rows, dtype=torch.float32, device=x.device)
    check(lib().nyion_attn_gemv_q4k(_ptr(w), _ptr(x2), _ptr(out), n_rows, n_blocks, x2.shape[0],
                                    _stream_ptr(stream)))
    return out


def rope_table(head_dim: int, max_context: int, device=None, stream=None):
    """Device RoPE table [max_context][head_dim/2][2] (cos, sin) of the CPU engine
    (ops.rs:20-38), built on the host with libm and uploaded."""
    torch = _torch()
    t = torch.empty(max_context, head_dim // 2, 2, dtype=torch.float32, device=device or "cuda")
    check(lib().nyion_attn_rope_table(_ptr(t), head_dim, max_context, _stream_ptr(stream)))
    return t


def kv_write_paged(k, v, positions, q=None, row_seq=None, rope=None, page_table=None, n_pool_pages: int = 0,
                   pool_q4=None, pool_f32=None, pool_bf16=None, q_bf16=None, ring_f32=None, stream=None):
    """RoPE on q / k (in place) and the K / V save into the given caches (nyion_attn_kv_write_paged).
    k, v [rows, n_kv, D] f32; positions [rows] int32; rope = rope_table(...) or None."""
    rows, n_kv, D = k.shape
    n_heads = q.shape[1] if q is not None else 0
    pools = [x for x in (pool_q4, pool_f32, pool_bf16) if x is not None]
    if pools and not n_pool_pages:
        n_pool_pages = pools[0].shape[0]
    check(lib().nyion_attn_kv_write_paged(
        _ptr(q), _ptr(k), _ptr(v), _ptr(positions), _ptr(row_seq), rows, n_heads, n_kv, D, _ptr(rope),
        rope.shape[0] if rope is not None else 0, _ptr(page_table),
        page_table.shape[-1] if page_table is not None else 0, n_pool_pages, _ptr(pool_q4), _ptr(pool_f32),
        _ptr(pool_bf16), _ptr(q_bf16), _ptr(ring_f32), ring_f32.shape[3] if ring_f32 is not None else 0,
        _stream_ptr(stream)))


def kv_write_ring_f16(k, v, d_seq_len, k_ring, v_ring, q=None, d_wpos=None, rope=None, stream=None):
    """Layer-graph RoPE + f16 ring save of one sequence (nyion_attn_kv_write_ring_f16).
    k, v [n_kv, D] f32; k_ring / v_ring [n_kv, window, D] f16; d_seq_len int32 [1]."""
    n_kv, D = k.shape
    n_heads = q.shape[0] if q is not None else 0
    check(lib().nyion_attn_kv_write_ring_f16(
        _ptr(q), _ptr(k), _ptr(v), _ptr(d_seq_len), _ptr(d_wpos), _ptr(k_ring), _ptr(v_ring), n_heads, n_kv, D,
        k_ring.shape[1], _ptr(rope), rope.shape[0] if rope is not None else 0, _stream_ptr(stream)))


def prefill_paged_bf16(q, kv_pool, page_table, q_start: int, out=None, scale: float = 0.0,
                       stream=None):
    """Causal chunked prefill (nyion_attn_prefill_paged_bf16).

    q [n_q, H, D] bf16 at positions q_start..; kv_pool [pages, n_kv, 2, 16, D]
    bf16; page_table [max_pages] int32; returns out [n_q, H, D] f32.
    """
    torch = _torch()
    n_q, H, D = q.shape
    if out is None:
        out = torch.empty(n_q, H, D, dtype=torch.float32, device=q.device)
    check(lib().nyion_attn_prefill_paged_bf16(
        _ptr(q), _ptr(kv_pool), kv_pool.shape[0], _ptr(page_table), page_table.numel(), q_start, n_q,
        _ptr(out), H, kv_pool.shape[1], D, kv_pool.shape[3], float(scale), _stream_ptr(stream)))
    return out


class F16Workspace:
    def __init__(self, n_heads: int, max_tokens: int, device=None):
        torch = _torch()
        self.nbytes = int(lib().nyion_attn_f16_workspace_size(n_heads, max_tokens))
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device or "cuda")
        check(lib().nyion_attn_workspace_reset(self.ptr(), self.nbytes, None))   # merge counters start at 0

    def ptr(self) -> int:
        return int(self.buf.data_ptr())


def decode_contig_f16(q, k_cache, v_cache, seq_len: int, out=None, scale: float = 0.0, workspace=None,
                      stream=None):
    """q [H, D] f32; k/v_cache [n_kv, stride, D] f16; attends tokens [0, seq_len)."""
    torch = _torch()
    H, D = q.shape
    if out is None:
        out = torch.empty(H, D, dtype=torch.float32, device=q.device)
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.ptr(), workspace.nbytes)
    check(lib().nyion_attn_decode_contig_f16(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), H,
                                             k_cache.shape[0], seq_len, D, k_cache.shape[1], float(scale),
                                             ws_ptr, ws_bytes, _stream_ptr(stream)))
    return out


def decode_ring_f16(q, k_ring, v_ring, d_seq_len, out=None, scale: float = 0.0, workspace=None,
                    stream=None):
    """Layer-graph node: q [H, D] f32; rings [n_kv, window, D] f16; length read on device."""
    torch = _torch()
    H, D = q.shape
    if out is None:
        out = torch.empty(H, D, dtype=torch.float32, device=q.device)
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.ptr(), workspace.nbytes)
    check(lib().nyion_attn_decode_ring_f16(_ptr(q), _ptr(k_ring), _ptr(v_ring), _ptr(d_seq_len), _ptr(out), H,
                                           k_ring.shape[0], D, k_ring.shape[1], float(scale), ws_ptr, ws_bytes,
                                           _stream_ptr(stream)))
    return out


class Mailbox:
    """A split-KV mailbox in device memory (library-allocated so CUDA IPC maps
    exactly this allocation)."""

    def __init__(self, batch: int, n_heads: int = 32):
        self.nbytes = int(lib().nyion_attn_splitkv_mailbox_bytes(batch, n_heads))
        ptr = C.c_void_p()
        check(lib().nyion_attn_mailbox_alloc(self.nbytes, C.byref(ptr)))
        self.ptr = ptr.value

    def ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        check(lib().nyion_attn_ipc_handle(C.c_void_p(self.ptr), buf))
        return buf.raw

    def free(self):
        if self.ptr:
            check(lib().nyion_attn_mailbox_free(C.c_void_p(self.ptr)))
            self.ptr = None


def ipc_open(handle: bytes) -> int:
    ptr = C.c_void_p()
    check(lib().nyion_attn_ipc_open(handle, C.byref(ptr)))
    return ptr.value


def ipc_close(ptr: int) -> None:
    check(lib().nyion_attn_ipc_close(C.c_void_p(ptr)))


def decode_q4_splitkv(q, kv_pool, page_table, u_begin: int, u_end: int, mailboxes, rank: int, out=None,
                      scale: float = 0.0, timeout_ms: int = 0, workspace=None, stream=None):
    """Rank `rank`'s share of a split-KV decode, the ranks' rows exchanged over
    peer memory: returns the combined attention out [B, H, D] (same on every rank)."""
    torch = _torch()
    B, H, D = q.shape
    if out is None:
        out = torch.empty(B, H, D, dtype=torch.float32, device=q.device)
    world = len(mailboxes)
    arr = (C.c_void_p * world)(*[C.c_void_p(m) for m in mailboxes])
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.ptr(), workspace.nbytes)
    check(lib().nyion_attn_decode_q4_splitkv(
        _ptr(q), _ptr(kv_pool), kv_pool.shape[0], _ptr(page_table), page_table.shape[1], u_begin, u_end, _ptr(out),
        B, H, kv_pool.shape[1], D, kv_pool.shape[3], float(scale), arr, world, rank, timeout_ms, ws_ptr, ws_bytes,
        _stream_ptr(stream)))
    return out


def exp_q16_16(x_fixed, out=None, stream=None):
    """exp_q16_16 of a device int32 vector (nyion_attn_exp_q16_16)."""
    import torch
    assert x_fixed.is_cuda and x_fixed.dtype == torch.int32 and x_fixed.is_contiguous()
    if out is None:
        out = torch.empty_like(x_fixed)
    check(lib().nyion_attn_exp_q16_16(_ptr(x_fixed), _ptr(out), x_fixed.numel(), _stream_ptr(stream)))
    return out


def softmax_padic(logits, temperature: float = 1.0, out=None, stream=None):
    """Q16.16 softmax of a device f32 vector (nyion_attn_softmax_padic)."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(logits)
    check(lib().nyion_attn_softmax_padic(_ptr(logits), _ptr(out), logits.numel(), float(temperature),
                                         _stream_ptr(stream)))
    return out


class StokesStore:
    """The reference's Stokes KV store, rows in HBM (mojo_stokes_*)."""

    def __init__(self, head_dim: int):
        self.hd = head_dim
        self.h = lib().mojo_stokes_init(head_dim)
        if not self.h:
            raise NyionError(-1, last_error())

    def append(self, token_id: int, key, value, score: float) -> None:
        import numpy as np
        k = np.ascontiguousarray(key, dtype=np.float32)
        v = np.ascontiguousarray(value, dtype=np.float32)
        lib().mojo_stokes_append(self.h, token_id, k.ctypes.data, v.ctypes.data, float(score))

    def view(self):
        """(keys, values) device pointers, token count."""
        k, v, n, hd = C.c_void_p(), C.c_void_p(), C.c_int32(), C.c_int32()
        check(lib().nyion_attn_stokes_view(self.h, C.byref(k), C.byref(v), C.byref(n), C.byref(hd)))
        return k.value, v.value, n.value

    def close(self):
        if self.h:
            lib().mojo_stokes_free(self.h)
            self.h = None


def device_error(stream=None) -> int:
    bits = C.c_int32(0)
    st = lib().nyion_attn_device_error(_stream_ptr(stream), C.byref(bits))
    if st not in (NYION_OK, -4):
        check(st)
    return int(bits.value)
