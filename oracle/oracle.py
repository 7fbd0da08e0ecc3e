"""ctypes wrapper over liboracle.so — the CPU restatement of the reference.

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline legs use it as the checker.  The product path (nyion.rs_b200)
never imports it.  Every function mirrors one C entry point of
nyion_oracle.c, which cites the reference file:line it restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "nyion_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB_PATH)
        i64, i32, f32 = C.c_int64, C.c_int, C.c_float
        sig = {
            "or_f16_from_f32": (C.c_uint16, [f32]),
            "or_f16_to_f32": (f32, [C.c_uint16]),
            "or_f16c_available": (i32, []),
            "or_f16_from_f32_f16c": (C.c_uint16, [f32]),
            "or_zone_index": (i64, [i64]),
            "or_block_size_for": (i64, [i64]),
            "or_page_id": (i64, [i64]),
            "or_slot_in_page": (i64, [i64]),
            "or_page_start_for": (i64, [i64]),
            "or_zone_page_count": (i64, [i32, i64]),
            "or_total_pages": (i64, [i64]),
            "or_q4_quantize_block": (None, [f32p, i32, u8p]),
            "or_q4_dequant_block": (None, [u8p, i32, f32p]),
            "or_q4_quantize_rows": (None, [f32p, i64, i32, u8p]),
            "or_q4_dequant_rows": (None, [u8p, i64, i32, f32p]),
            "or_dot_product_raw": (f32, [f32p, f32p, i32]),
            "or_weighted_sum_raw": (None, [f32p, f32p, f32, i32]),
            "or_avx512_available": (i32, []),
            "or_attention": (None, [f32p, f32p, C.c_void_p, C.c_void_p, i32, i32, i64, i64, i32, i32, i32]),
            "or_attention_tracked": (None, [f32p, f32p, C.c_void_p, C.c_void_p, i32, i32, i64, i64, i32, i32, i32, f64p]),
            "or_attention_sparse_q4": (None, [f32p, f32p, C.c_void_p, C.c_void_p, i32, i32, i64, i64, i32, i32, i32, i64, i64, i32]),
            "or_sparse_positions": (i64, [i64, i64, i64, i64, i64p, i64]),
            "or_exp_q16_16": (C.c_int32, [C.c_int32]),
            "or_exp_q16_16_many": (None, [i32p, i32p, i64]),
            "or_rope_lut": (None, [f32p, i32, i64]),
            "or_gemv_q4k": (None, [u8p, f32p, f32p, i32, i32]),
            "or_mojo_sparse_attention_q4": (None, [f32p, f32p, f32p, i32p, f32p, i32, i32, i32]),
            "or_apply_rope": (None, [f32p, f32p, i64, i32, i32, i32, i64, f32p]),
            "or_softmax_padic": (None, [f32p, f32p, i32, f32]),
            "or_stokes_init": (C.c_void_p, [i32]),
            "or_stokes_append": (None, [C.c_void_p, i32, f32p, f32p, f32]),
            "or_stokes_free": (None, [C.c_void_p]),
            "or_stokes_len": (i64, [C.c_void_p]),
            "or_stokes_keys": (C.POINTER(f32), [C.c_void_p]),
            "or_stokes_values": (C.POINTER(f32), [C.c_void_p]),
            "or_stokes_scores": (C.POINTER(f32), [C.c_void_p]),
            "or_decode_paged_f32": (None, [f32p, f32p, f32p, i32p, i32p, i32, i32, i32, i32, i32, i32, f32, i32]),
            "or_decode_q4_window_ring": (None, [f32p, f32p, u8p, i32p, i32p, f32p, i32, i64, i32, i32, i32, i32, i32, i32, f32, i32]),
            "or_decode_q4_partial": (None, [f32p, f32p, u8p, i32p, i64, i64, i32, i32, i32, i32, i32, i32, f32, i32]),
            "or_lse_combine": (None, [f32p, f32p, i32, i64, i32]),
            "or_prefill_paged_bf16": (None, [f32p, u16p, u16p, i32p, i32, i64, i64, i32, i32, i32, i32, f32, i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- f16 / zones
def f16_from_f32(x: float) -> int:
    return int(lib().or_f16_from_f32(float(x)))


def f16_to_f32(h: int) -> float:
    return float(lib().or_f16_to_f32(int(h)))


def page_id(pos: int) -> int:
    return int(lib().or_page_id(pos))


def slot_in_page(pos: int) -> int:
    return int(lib().or_slot_in_page(pos))


def block_size_for(pos: int) -> int:
    return int(lib().or_block_size_for(pos))


def page_start_for(pos: int) -> int:
    return int(lib().or_page_start_for(pos))


def total_pages(max_seq_len: int) -> int:
    return int(lib().or_total_pages(max_seq_len))


# ---------------------------------------------------------------- Q4 blocks
def q4_quantize_rows(src: np.ndarray, head_dim: int) -> np.ndarray:
    """src [..., head_dim] f32 -> [..., nblk*20] u8 (cache.rs:637-663 per row)."""
    src = _c(src, np.float32)
    nblk = (head_dim + 31) // 32
    rows = src.size // head_dim
    dst = np.zeros(rows * nblk * 20, dtype=np.uint8)
    lib().or_q4_quantize_rows(src.reshape(-1), rows, head_dim, dst)
    return dst.reshape(src.shape[:-1] + (nblk * 20,))


def q4_dequant_rows(src: np.ndarray, head_dim: int) -> np.ndarray:
    src = _c(src, np.uint8)
    nblk = (head_dim + 31) // 32
    rows = src.size // (nblk * 20)
    dst = np.zeros(rows * head_dim, dtype=np.float32)
    lib().or_q4_dequant_rows(src.reshape(-1), rows, head_dim, dst)
    if src.ndim == 1:
        return dst.reshape(rows, head_dim)
    return dst.reshape(src.shape[:-1] + (head_dim,))


def q4_quantize_block_into(src: np.ndarray, blk: np.ndarray) -> None:
    """OR-into quantization of one block (cache.rs:659 semantics)."""
    lib().or_q4_quantize_block(_c(src, np.float32), int(src.size), blk)


# ---------------------------------------------------------------- simd
def dot_product_raw(a: np.ndarray, b: np.ndarray) -> float:
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    return float(lib().or_dot_product_raw(a, b, a.size))


def weighted_sum_raw(out: np.ndarray, v: np.ndarray, score: float) -> None:
    lib().or_weighted_sum_raw(out, _c(v, np.float32), float(score), out.size)


# ---------------------------------------------------------------- reference-layout cache
class ZonedPages:
    """Host copy of the reference PagedKVCache page set (cache.rs), f32 and Q4.

    Pages are allocated per flat page id exactly as cache.rs does, laid out
    [layer][kv_head][slot][head_dim] (f32) and [layer][kv_head][slot][blk*20] (Q4).
    ``save(layer, pos, k, v)`` follows PagedKVCache::save: Q4 always, f32 only
    if that page's f32 copy exists (cache.rs:613-679).  ``ensure_f32(end)``
    follows ensure_pages_hot_f32 (dequantize pages lacking f32).
    """

    def __init__(self, n_layers: int, n_kv: int, head_dim: int, max_seq_len: int):
        self.n_layers, self.n_kv, self.hd, self.max_seq_len = n_layers, n_kv, head_dim, max_seq_len
        self.nblk = (head_dim + 31) // 32
        self.k_q4, self.v_q4, self.k_f32, self.v_f32 = {}, {}, {}, {}

    def _bs(self, pid: int) -> int:
        return 32 if pid < 128 else (128 if pid < 1120 else 1024)

    def _ensure(self, pid: int) -> None:
        if pid not in self.k_q4:
            n = self.n_layers * self.n_kv * self._bs(pid) * self.nblk * 20
            self.k_q4[pid] = np.zeros(n, np.uint8)
            self.v_q4[pid] = np.zeros(n, np.uint8)

    def save(self, layer: int, pos: int, k: np.ndarray, v: np.ndarray) -> None:
        pid, slot = page_id(pos), slot_in_page(pos)
        self._ensure(pid)
        bs = self._bs(pid)
        k = _c(k, np.float32).reshape(self.n_kv, self.hd)
        v = _c(v, np.float32).reshape(self.n_kv, self.hd)
        row = self.nblk * 20
        for kv_h in range(self.n_kv):
            off = ((layer * self.n_kv + kv_h) * bs + slot) * row
            for b in range(self.nblk):
                s, e = b * 32, min(b * 32 + 32, self.hd)
                kb = self.k_q4[pid][off + b * 20: off + b * 20 + 20]
                vb = self.v_q4[pid][off + b * 20: off + b * 20 + 20]
                q4_quantize_block_into(k[kv_h, s:e], kb)
                q4_quantize_block_into(v[kv_h, s:e], vb)
                self.k_q4[pid][off + b * 20: off + b * 20 + 20] = kb
                self.v_q4[pid][off + b * 20: off + b * 20 + 20] = vb
            if pid in self.k_f32:
                foff = ((layer * self.n_kv + kv_h) * bs + slot) * self.hd
                self.k_f32[pid][foff: foff + self.hd] = k[kv_h]
                self.v_f32[pid][foff: foff + self.hd] = v[kv_h]

    def ensure_f32(self, end_page: int) -> None:
        for pid in range(end_page + 1):
            self._ensure(pid)
            if pid not in self.k_f32:
                self.k_f32[pid] = q4_dequant_rows(self.k_q4[pid], self.hd).reshape(-1)
                self.v_f32[pid] = q4_dequant_rows(self.v_q4[pid], self.hd).reshape(-1)

    def set_f32_exact(self, layer: int, pos: int, k: np.ndarray, v: np.ndarray) -> None:
        """Exact-fp32 fill: ensure_pages_hot_f32 then save (cache.rs:555-561, 671-677)."""
        pid = page_id(pos)
        self.ensure_f32(pid)
        self.save(layer, pos, k, v)

    def ptr_arrays(self, kind: str):
        store_k, store_v = (self.k_f32, self.v_f32) if kind == "f32" else (self.k_q4, self.v_q4)
        n = max(store_k) + 1 if store_k else 0
        kp = (C.c_void_p * n)()
        vp = (C.c_void_p * n)()
        for pid in range(n):
            if pid in store_k:
                kp[pid] = store_k[pid].ctypes.data
                vp[pid] = store_v[pid].ctypes.data
        return kp, vp


def attention(zp: ZonedPages, q: np.ndarray, layer: int, seq_len: int, q_pos: int, n_heads: int,
              tracked: bool = False):
    """ops::attention / attention_tracked over a ZonedPages store (f32 pages)."""
    out = np.zeros(n_heads * zp.hd, np.float32)
    kp, vp = zp.ptr_arrays("f32")
    q = _c(q, np.float32).reshape(-1)
    if tracked:
        imp = np.zeros(seq_len, np.float64)
        lib().or_attention_tracked(out, q, kp, vp, zp.n_layers, layer, seq_len, q_pos, n_heads,
                                   zp.n_kv, zp.hd, imp)
        return out.reshape(n_heads, zp.hd), imp
    lib().or_attention(out, q, kp, vp, zp.n_layers, layer, seq_len, q_pos, n_heads, zp.n_kv, zp.hd)
    return out.reshape(n_heads, zp.hd)


def attention_sparse_q4(zp: ZonedPages, q, layer, seq_len, q_pos, n_heads, window, global_stride,
                        as_written: bool):
    out = np.zeros(n_heads * zp.hd, np.float32)
    kp, vp = zp.ptr_arrays("q4")
    lib().or_attention_sparse_q4(out, _c(q, np.float32).reshape(-1), kp, vp, zp.n_layers, layer,
                                 seq_len, q_pos, n_heads, zp.n_kv, zp.hd, window, global_stride,
                                 1 if as_written else 0)
    return out.reshape(n_heads, zp.hd)


def sparse_positions(seq_len, q_pos, window, global_stride) -> np.ndarray:
    cap = window + 130
    buf = np.zeros(cap, np.int64)
    n = lib().or_sparse_positions(seq_len, q_pos, window, global_stride, buf, cap)
    return buf[:n].copy()


# ---------------------------------------------------------------- rope
def rope_lut(head_dim: int, max_seq_len: int) -> np.ndarray:
    """[max_seq_len][head_dim/2][2] (cos, sin), ops.rs:20-38."""
    lut = np.zeros((max_seq_len, head_dim // 2, 2), np.float32)
    lib().or_rope_lut(lut.reshape(-1), head_dim, max_seq_len)
    return lut


def apply_rope(q, k, pos: int, max_context: int, lut: np.ndarray):
    """Rotated copies of q [n_q][hd] and k [n_kv][hd] (ops.rs:42-84)."""
    q = _c(q, np.float32).copy()
    k = _c(k, np.float32).copy()
    hd = q.shape[-1]
    lib().or_apply_rope(q.reshape(-1), k.reshape(-1), int(pos), q.size // hd, k.size // hd, hd, int(max_context),
                        _c(lut, np.float32).reshape(-1))
    return q, k


def gemv_q4k(w, x, n_rows: int, n_blocks: int) -> np.ndarray:
    """fused_attention.cu:858-914 Q4_K GEMV (column-major super-blocks)."""
    out = np.zeros(n_rows, np.float32)
    lib().or_gemv_q4k(_c(w, np.uint8).reshape(-1), _c(x, np.float32).reshape(-1), out, n_rows, n_blocks)
    return out


def mojo_sparse_attention_q4(q, k_rows, v_rows, positions):
    """attention.mojo:40-152 as written: q [H][hd]; k_rows / v_rows [n][blocks*20] f32."""
    q = _c(q, np.float32)
    H, hd = q.shape
    out = np.zeros((H, hd), np.float32)
    pos = _c(positions, np.int32)
    lib().or_mojo_sparse_attention_q4(q.reshape(-1), _c(k_rows, np.float32).reshape(-1),
                                      _c(v_rows, np.float32).reshape(-1), pos, out.reshape(-1), H, hd, pos.size)
    return out


def mojo_rows_from_q4(rows_u8: np.ndarray) -> np.ndarray:
    """20-byte blocks [f16 d][f16 dmin][16 B] -> the Mojo kernel's 20-float blocks."""
    r = _c(rows_u8, np.uint8)
    nblk = r.shape[-1] // 20
    b = r.reshape(r.shape[:-1] + (nblk, 20))
    out = np.zeros(b.shape, np.float32)
    out[..., 0] = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    out[..., 1] = b[..., 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    out[..., 2:18] = b[..., 4:20].astype(np.float32)
    return out.reshape(r.shape[:-1] + (nblk * 20,))


# ---------------------------------------------------------------- softmax / stokes
def exp_q16_16(x: int) -> int:
    return int(lib().or_exp_q16_16(int(x)))


def exp_q16_16_many(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.int32)
    out = np.zeros_like(x)
    lib().or_exp_q16_16_many(x, out, x.size)
    return out


def softmax_padic(logits: np.ndarray, temperature: float = 1.0) -> np.ndarray:
    logits = _c(logits, np.float32)
    probs = np.zeros_like(logits)
    lib().or_softmax_padic(logits, probs, logits.size, float(temperature))
    return probs


class Stokes:
    def __init__(self, head_dim: int):
        self.hd = head_dim
        self.h = lib().or_stokes_init(head_dim)

    def append(self, token_id: int, k, v, score: float) -> None:
        lib().or_stokes_append(self.h, token_id, _c(k, np.float32), _c(v, np.float32), float(score))

    def __len__(self):
        return int(lib().or_stokes_len(self.h))

    def arrays(self):
        n = len(self)
        k = np.ctypeslib.as_array(lib().or_stokes_keys(self.h), shape=(n * self.hd,)).copy()
        v = np.ctypeslib.as_array(lib().or_stokes_values(self.h), shape=(n * self.hd,)).copy()
        s = np.ctypeslib.as_array(lib().or_stokes_scores(self.h), shape=(n,)).copy()
        return k.reshape(n, self.hd), v.reshape(n, self.hd), s

    def close(self):
        if self.h:
            lib().or_stokes_free(self.h)
            self.h = None


# ---------------------------------------------------------------- new layouts
def decode_paged_f32(q, pool, page_table, seq_lens, n_kv, head_dim, page_tokens, scale=None, threads=1):
    q = _c(q, np.float32)
    B, H = q.shape[0], q.shape[1]
    out = np.zeros((B, H, head_dim), np.float32)
    scale = 1.0 / np.sqrt(head_dim) if scale is None else scale
    pt = _c(page_table, np.int32)
    lib().or_decode_paged_f32(out.reshape(-1), q.reshape(-1), _c(pool, np.float32).reshape(-1),
                              pt.reshape(-1), _c(seq_lens, np.int32), B, pt.shape[1], H, n_kv,
                              head_dim, page_tokens, float(scale), threads)
    return out


def decode_q4_window_ring(q, pool_q4, page_table, seq_lens, ring, ring_tokens, window, n_kv,
                          head_dim, page_tokens, scale=None, threads=1):
    q = _c(q, np.float32)
    B, H = q.shape[0], q.shape[1]
    out = np.zeros((B, H, head_dim), np.float32)
    scale = 1.0 / np.sqrt(head_dim) if scale is None else scale
    pt = _c(page_table, np.int32)
    lib().or_decode_q4_window_ring(out.reshape(-1), q.reshape(-1), _c(pool_q4, np.uint8).reshape(-1),
                                   pt.reshape(-1), _c(seq_lens, np.int32), _c(ring, np.float32).reshape(-1),
                                   ring_tokens, window, B, pt.shape[1], H, n_kv, head_dim, page_tokens,
                                   float(scale), threads)
    return out


def decode_q4_partial(q, pool_q4, page_table, tok_begin, tok_end, n_kv, head_dim, page_tokens,
                      scale=None, threads=1):
    q = _c(q, np.float32)
    B, H = q.shape[0], q.shape[1]
    part = np.zeros((B, H, head_dim + 2), np.float32)
    scale = 1.0 / np.sqrt(head_dim) if scale is None else scale
    pt = _c(page_table, np.int32)
    lib().or_decode_q4_partial(part.reshape(-1), q.reshape(-1), _c(pool_q4, np.uint8).reshape(-1),
                               pt.reshape(-1), tok_begin, tok_end, B, pt.shape[1], H, n_kv, head_dim,
                               page_tokens, float(scale), threads)
    return part


def lse_combine(parts: np.ndarray) -> np.ndarray:
    parts = _c(parts, np.float32)
    G = parts.shape[0]
    hd = parts.shape[-1] - 2
    rows = parts[0].size // (hd + 2)
    out = np.zeros(rows * hd, np.float32)
    lib().or_lse_combine(out, parts.reshape(-1), G, rows, hd)
    return out.reshape(parts.shape[1:-1] + (hd,))


def prefill_paged_bf16(q_bf16, pool_bf16, page_table, q_start, n_kv, head_dim, page_tokens,
                       scale=None, threads=1):
    q = _c(q_bf16, np.uint16)
    n_q, H = q.shape[0], q.shape[1]
    out = np.zeros((n_q, H, head_dim), np.float32)
    scale = 1.0 / np.sqrt(head_dim) if scale is None else scale
    pt = _c(page_table, np.int32).reshape(-1)
    lib().or_prefill_paged_bf16(out.reshape(-1), q.reshape(-1), _c(pool_bf16, np.uint16).reshape(-1),
                                pt, pt.size, q_start, n_q, H, n_kv, head_dim, page_tokens,
                                float(scale), threads)
    return out
