"""Pins the CPU oracle to the reference's own known-answer tests.

Each test cites the reference test it ports (bmcc-DEV/Nyion.rs paths).  The
oracle is the checker for every GPU parity test, so it is pinned first:
zone page ids, Q4 round trips, dot/AXPY, exp/softmax Q16.16, f16 rounding.
"""
import os
import struct
import subprocess
import sys

import numpy as np
import pytest

import oracle as O


# ----------------------------------------------------------------- zone geometry
def test_zone_boundaries_golden():
    """swamp-engine/src/cache.rs:1000-1029 test_zone_boundaries (exact ids)."""
    assert O.block_size_for(0) == 32
    assert O.block_size_for(4095) == 32
    assert O.block_size_for(4096) == 128
    assert O.block_size_for(131071) == 128
    assert O.block_size_for(131072) == 1024
    golden = {0: 0, 31: 0, 32: 1, 4095: 127, 4096: 128, 4223: 128, 4224: 129,
              131071: 128 + 991, 131072: 128 + 992, 132095: 128 + 992, 132096: 128 + 993}
    for pos, pid in golden.items():
        assert O.page_id(pos) == pid, pos


def test_zone_slots_and_starts():
    """cache.rs:599-610: slot = (pos-zone_start) % bs, page start = pos - slot."""
    for pos in [0, 1, 31, 32, 4095, 4096, 4097, 4223, 4224, 131071, 131072, 131073, 1048575]:
        bs = O.block_size_for(pos)
        zs = 0 if pos < 4096 else (4096 if pos < 131072 else 131072)
        assert O.slot_in_page(pos) == (pos - zs) % bs
        assert O.page_start_for(pos) == pos - (pos - zs) % bs
    # build_zones (cache.rs:185-200): 128 + 992 + ceil((max-131072)/1024)
    assert O.total_pages(140000) == 128 + 992 + 9
    assert O.total_pages(128) == 128 + 992


# ----------------------------------------------------------------- f16
def _py_f16(x: np.float32) -> int:
    # struct 'e' packs IEEE binary16 with round-half-even (independent of the oracle)
    return struct.unpack("<H", struct.pack("<e", float(x)))[0]


def test_f16_rne_matches_independent_statement():
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32),
        (rng.standard_normal(5000) * 1e-5).astype(np.float32),   # subnormal f16 range
        (rng.standard_normal(2000) * 3e4).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-10, 2.0 ** -25, 2.0 ** -24,
                  3 * 2.0 ** -26, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11], np.float32),
    ])
    for v in vals:
        v = np.float32(v)
        try:
            want = _py_f16(v)
        except OverflowError:
            want = 0x7C00 | (0x8000 if v < 0 else 0)
        assert O.f16_from_f32(v) == want, float(v)


@pytest.mark.skipif(not O.lib().or_f16c_available(), reason="host has no F16C")
def test_f16_rne_matches_f16c_hardware():
    rng = np.random.default_rng(2)
    vals = np.concatenate([rng.standard_normal(20000), rng.standard_normal(5000) * 1e-6,
                           rng.standard_normal(2000) * 7e4]).astype(np.float32)
    L = O.lib()
    for v in vals:
        assert L.or_f16_from_f32(float(v)) == L.or_f16_from_f32_f16c(float(v)), float(v)


def test_f16_to_f32_exact_all_finite():
    for h in range(0, 0x10000, 7):
        if (h & 0x7C00) == 0x7C00:
            continue
        want = struct.unpack("<e", struct.pack("<H", h))[0]
        assert O.f16_to_f32(h) == np.float32(want)


# ----------------------------------------------------------------- Q4 quantizer
def _numpy_quantize_block(x: np.ndarray) -> bytes:
    """Independent numpy statement of cache.rs:637-663 for one block."""
    x = x.astype(np.float32)
    mx = np.float32(0.0)
    mn = np.float32(np.finfo(np.float32).max)
    for v in x:
        mx = np.float32(max(mx, abs(v)))
        mn = np.float32(min(mn, v))
    d = np.float32(mx / np.float32(7.0)) if mx > np.float32(1e-10) else np.float32(0.0)
    out = bytearray(20)
    out[0:2] = struct.pack("<H", _py_f16(d))
    out[2:4] = struct.pack("<H", _py_f16(mn))
    for i, v in enumerate(x):
        q = 0
        if d > np.float32(1e-10):
            r = np.float32(np.float32(v - mn) / d)
            r = np.floor(np.float64(r) + 0.5)          # round half away from zero (r >= 0)
            q = int(min(max(r, 0.0), 15.0))
        out[4 + i // 2] |= (q << (0 if i % 2 == 0 else 4))
    return bytes(out)


def test_q4_quantizer_bytes_match_independent_statement():
    rng = np.random.default_rng(3)
    blocks = [rng.standard_normal(32), rng.standard_normal(32) * 100, np.zeros(32),
              np.full(32, 42.0), np.arange(32, dtype=np.float64), -np.arange(32, dtype=np.float64),
              rng.standard_normal(32) * 1e-6, np.concatenate([np.zeros(31), [1e-12]])]
    blocks += [rng.standard_normal(32) for _ in range(300)]
    for x in blocks:
        x = x.astype(np.float32)
        got = O.q4_quantize_rows(x[None, :], 32)[0].tobytes()
        assert got == _numpy_quantize_block(x)


def test_q4_nibble_order_and_dequant_formula():
    """F6: element i in byte i/2, low nibble for even i; dequant = f32(d)*q + f32(dmin)."""
    x = np.arange(32, dtype=np.float32)
    blk = O.q4_quantize_rows(x[None, :], 32)[0]
    d = O.f16_to_f32(int(blk[0]) | int(blk[1]) << 8)
    dmin = O.f16_to_f32(int(blk[2]) | int(blk[3]) << 8)
    deq = O.q4_dequant_rows(blk[None, :], 32)[0]
    for i in range(32):
        nib = (blk[4 + i // 2] >> (0 if i % 2 == 0 else 4)) & 0xF
        want = np.float32(np.float32(d) * np.float32(nib)) + np.float32(dmin)
        assert deq[i] == np.float32(want)
    assert abs(deq - x).max() <= 31.0 / 7.0


def _fill_cache(zp, tokens, make_kv, layers):
    for pos in range(tokens):
        k, v = make_kv(pos)
        for l in range(layers):
            zp.save(l, pos, k, v)


def test_paged_cache_basic_rw():
    """cache.rs:853-890: 2 layers, 4 kv heads, hd 64, Q4 round trip within 1.0."""
    zp = O.ZonedPages(2, 4, 64, 128)

    def kv(pos):
        k = np.zeros((4, 64), np.float32)
        v = np.zeros((4, 64), np.float32)
        for h in range(4):
            k[h, 0] = pos * 100 + h
            v[h, 0] = pos * 1000 + h
        return k, v

    _fill_cache(zp, 3, kv, 2)
    zp.ensure_f32(0)
    for l in range(2):
        for h in range(4):
            for pos in range(3):
                off = ((l * 4 + h) * 32 + pos) * 64
                assert abs(zp.k_f32[0][off] - (pos * 100 + h)) < 1.0
                assert abs(zp.v_f32[0][off] - (pos * 1000 + h)) < 1.0


def test_paged_cache_multiple_pages_exact():
    """cache.rs:892-926: constant rows survive Q4 exactly; page starts via k_page_ptr."""
    zp = O.ZonedPages(1, 1, 64, 1024)
    _fill_cache(zp, 32, lambda p: (np.full(64, p, np.float32), np.full(64, 2 * p, np.float32)), 1)
    zp.ensure_f32(O.page_id(31))
    for pos in range(32):
        pid, slot = O.page_id(pos), O.slot_in_page(pos)
        assert zp.k_f32[pid][slot * 64] == pos
        assert zp.v_f32[pid][slot * 64] == 2 * pos
        bs = O.block_size_for(pos)
        assert abs(zp.k_f32[pid][0] - (pos - pos % bs)) < 0.5


def test_paged_cache_reset_rewrite():
    """cache.rs:928-949: after reset, slot 0 rewritten with 42 reads back 42 (fresh page)."""
    zp = O.ZonedPages(1, 1, 64, 1024)
    zp.save(0, 0, np.full(64, 42.0, np.float32), np.full(64, 42.0, np.float32))
    zp.ensure_f32(0)
    assert abs(zp.k_f32[0][0] - 42.0) < 0.5


def test_zone_read_write_cross_zone():
    """cache.rs:1031-1068: writes across zones 0/1 read back within 10."""
    zp = O.ZonedPages(2, 2, 64, 200000)
    for pos in list(range(0, 100)) + list(range(4090, 4200)):
        k = np.full(128, pos, np.float32)
        v = np.full(128, pos * 3, np.float32)
        for l in range(2):
            zp.save(l, pos, k, v)
    zp.ensure_f32(O.page_id(4199))
    for pos in [0, 99, 4096, 4198]:
        pid, slot, bs = O.page_id(pos), O.slot_in_page(pos), O.block_size_for(pos)
        k0 = zp.k_f32[pid][((0 * 2 + 0) * bs + slot) * 64]
        v1 = zp.v_f32[pid][((0 * 2 + 1) * bs + slot) * 64]
        assert abs(k0 - pos) < 10.0
        assert abs(v1 - pos * 3) < 10.0


def test_reresave_ors_nibbles():
    """cache.rs:659 ORs nibbles into existing bytes (quirk kept, not fixed)."""
    blk = np.zeros(20, np.uint8)
    O.q4_quantize_block_into(np.arange(32, dtype=np.float32), blk)
    first = blk.copy()
    O.q4_quantize_block_into(np.arange(32, dtype=np.float32)[::-1].copy(), blk)
    assert np.all((blk[4:] & first[4:]) == first[4:])


# ----------------------------------------------------------------- simd
def test_dot_product_known_answers():
    """swamp-kernels/src/simd.rs:190-229."""
    a = np.array([1, 2, 3, 4, 5, 6, 7, 8], np.float32)
    b = np.array([8, 7, 6, 5, 4, 3, 2, 1], np.float32)
    assert abs(O.dot_product_raw(a, b) - 120.0) < 1e-6
    a = np.array([1, 2, 3, 5, 7, 9], np.float32)
    b = np.array([2, 3, 5, 7, 11, 13], np.float32)
    assert abs(O.dot_product_raw(a, b) - float(np.dot(a, b))) < 1e-6
    a = (np.arange(64) * 0.5).astype(np.float32)
    b = (np.arange(64) * 0.25).astype(np.float32)
    assert abs(O.dot_product_raw(a, b) - float(np.dot(a.astype(np.float64), b))) < 1e-4


def test_weighted_sum_known_answer():
    out = np.array([1, 2, 3, 4], np.float32)
    O.weighted_sum_raw(out, np.array([5, 6, 7, 8], np.float32), 2.0)
    assert np.allclose(out, [11, 14, 17, 20], atol=1e-6)


def _numpy_dot_avx512_order(a, b):
    lanes = np.zeros(16, np.float32)
    n = a.size
    i = 0
    while i + 16 <= n:
        for j in range(16):
            lanes[j] = np.float32(np.float64(a[i + j]) * np.float64(b[i + j]) + np.float64(lanes[j]))
        i += 16
    s = [np.float32(np.float32(lanes[j] + lanes[4 + j]) + np.float32(lanes[8 + j] + lanes[12 + j]))
         for j in range(4)]
    return np.float32(np.float32(s[0] + s[1]) + np.float32(s[2] + s[3]))


def test_dot_product_reduction_order():
    """simd.rs:37-68 order: 16-lane FMA, quarters (l0+l1)+(l2+l3), two hadds.
    The float64 product+add then one rounding equals a single-rounded FMA."""
    rng = np.random.default_rng(4)
    for _ in range(200):
        a = rng.standard_normal(64).astype(np.float32)
        b = rng.standard_normal(64).astype(np.float32)
        assert O.dot_product_raw(a, b) == _numpy_dot_avx512_order(a, b)


def test_isa_paths_bit_identical():
    """The AVX-512, AVX2 and scalar oracle paths give identical bits."""
    code = ("import numpy as np, oracle as O\n"
            "rng=np.random.default_rng(5)\n"
            "a=rng.standard_normal((50,64)).astype(np.float32); b=rng.standard_normal((50,64)).astype(np.float32)\n"
            "print(','.join(repr(float(O.dot_product_raw(a[i],b[i]))) for i in range(50)))\n")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle")
    fast = subprocess.check_output([sys.executable, "-c", code], env=env)
    env["NYION_ORACLE_SCALAR"] = "1"
    scalar = subprocess.check_output([sys.executable, "-c", code], env=env)
    assert fast == scalar


# ----------------------------------------------------------------- softmax Q16.16
def test_exp_q16_16_accuracy():
    """swamp-kernels/src/lib.rs:629-656: < 0.8 % relative error on [-6, 0]."""
    worst = 0.0
    x = -6 * 65536
    while x <= 0:
        got = O.exp_q16_16(x) / 65536.0
        want = np.exp(x / 65536.0)
        worst = max(worst, abs(got - want) / want)
        x += 65536 // 64
    assert worst < 0.008


def test_exp_q16_16_edges():
    assert O.exp_q16_16(0) == 65536
    assert O.exp_q16_16(5) == 65536
    assert O.exp_q16_16(-655361) == 0
    assert O.exp_q16_16(-655360) > 0


def test_softmax_padic_normalization():
    """swamp-kernels/src/lib.rs:658-684."""
    logits = np.array([1.0, 2.0, 3.0, 0.5, -1.0, 4.0, 2.5, 1.5], np.float32)
    p = O.softmax_padic(logits, 1.0)
    assert abs(p.sum() - 1.0) < 0.01
    assert int(np.argmax(p)) == 5


def test_softmax_padic_simd_wrap_quirk():
    """AVX-512 blocks wrap p*inv at 2^32: a lone survivor in a 16-block reads 0."""
    logits = np.full(16, -100.0, np.float32)
    logits[3] = 10.0
    p = O.softmax_padic(logits, 1.0)
    assert p[3] == 0.0
    p8 = O.softmax_padic(logits[:8].copy(), 1.0)   # scalar tail keeps it
    assert p8[3] == 1.0


def test_softmax_padic_null_and_temperature():
    assert O.softmax_padic(np.zeros(0, np.float32)).size == 0
    x = np.linspace(-3, 3, 40).astype(np.float32)
    hot = O.softmax_padic(x, 10.0)
    cold = O.softmax_padic(x, 0.5)
    assert hot.max() < cold.max()


# ----------------------------------------------------------------- stokes
def test_stokes_append_and_evict():
    """swamp-kernels/src/lib.rs:36-85: above 4096 tokens the min-score row goes."""
    st = O.Stokes(4)
    for t in range(4097):
        st.append(t, np.full(4, t, np.float32), np.full(4, -t, np.float32), float(t if t != 10 else -5.0))
    assert len(st) == 4096
    k, v, s = st.arrays()
    assert 10.0 not in k[:, 0]
    assert k[10, 0] == 11.0 and s.min() == 0.0
    st.close()


# ----------------------------------------------------------------- attention maths
def _fp64_attention(q, K, V, scale):
    s = (K.astype(np.float64) @ q.astype(np.float64)) * scale
    p = np.exp(s - s.max())
    p /= p.sum()
    return p @ V.astype(np.float64)


def test_attention_zoned_against_fp64():
    """ops.rs:170-278 restated over reference-layout pages vs an fp64 statement."""
    rng = np.random.default_rng(0)
    L, n_kv, hd, H = 2, 4, 64, 32
    zp = O.ZonedPages(L, n_kv, hd, 4200)
    ks = rng.standard_normal((150, n_kv, hd)).astype(np.float32)
    vs = rng.standard_normal((150, n_kv, hd)).astype(np.float32)
    for pos in range(150):
        for l in range(L):
            zp.set_f32_exact(l, pos, ks[pos], vs[pos])
    q = rng.standard_normal((H, hd)).astype(np.float32)
    out = O.attention(zp, q, 1, 150, 149, H)
    for h in range(H):
        ref = _fp64_attention(q[h], ks[:, h // 8], vs[:, h // 8], 0.125)
        assert np.abs(out[h] - ref).max() < 1e-5
    # causal truncation: q_pos < seq_len - 1 sees only [0, q_pos]
    out2 = O.attention(zp, q, 1, 150, 99, H)
    ref2 = _fp64_attention(q[0], ks[:100, 0], vs[:100, 0], 0.125)
    assert np.abs(out2[0] - ref2).max() < 1e-5
    out3, imp = O.attention(zp, q, 1, 150, 99, H, tracked=True)
    assert np.array_equal(out3, out2)
    assert abs(imp.sum() - H) < 1e-4 and np.all(imp[100:] == 0)


def test_paged_f32_equals_zoned_on_same_rows():
    """The 16-token page-table reference runs the same per-head algorithm as
    ops::attention, so identical rows in identical order give identical bits."""
    rng = np.random.default_rng(7)
    n_kv, hd, H, T, pt = 4, 64, 32, 96, 16
    ks = rng.standard_normal((T, n_kv, hd)).astype(np.float32)
    vs = rng.standard_normal((T, n_kv, hd)).astype(np.float32)
    zp = O.ZonedPages(1, n_kv, hd, 4096)
    for pos in range(T):
        zp.set_f32_exact(0, pos, ks[pos], vs[pos])
    q = rng.standard_normal((H, hd)).astype(np.float32)
    zoned = O.attention(zp, q, 0, T, T - 1, H)
    n_pages = T // pt
    perm = rng.permutation(n_pages).astype(np.int32)
    pool = np.zeros((n_pages, n_kv, 2, pt, hd), np.float32)
    for p in range(n_pages):
        for s in range(pt):
            pool[perm[p], :, 0, s] = ks[p * pt + s]
            pool[perm[p], :, 1, s] = vs[p * pt + s]
    paged = O.decode_paged_f32(q[None], pool, perm[None], np.array([T], np.int32), n_kv, hd, pt)
    assert np.array_equal(paged[0], zoned)


def test_sparse_positions_and_q4_pairing():
    """ops.rs:597-723 positions; as-written vs writer-consistent pairing (F9)."""
    pos = O.sparse_positions(5000, 4999, 256, 64)
    assert pos[0] == 0 and pos[1] == 64 and pos[-1] == 4999
    assert len(pos) == min((4999 - 256 + 1) // 64, 128) + 256
    rng = np.random.default_rng(9)
    n_kv, hd, H = 4, 64, 32
    zp = O.ZonedPages(1, n_kv, hd, 400)
    ks = rng.standard_normal((300, n_kv, hd)).astype(np.float32)
    vs = rng.standard_normal((300, n_kv, hd)).astype(np.float32)
    for p in range(300):
        zp.save(0, p, ks[p], vs[p])
    q = rng.standard_normal((H, hd)).astype(np.float32)
    consistent = O.attention_sparse_q4(zp, q, 0, 300, 299, H, 256, 16, as_written=False)
    written = O.attention_sparse_q4(zp, q, 0, 300, 299, H, 256, 16, as_written=True)
    # writer-consistent equals fp64 attention over dequantized rows on the same positions
    sel = O.sparse_positions(300, 299, 256, 16)
    kd = O.q4_dequant_rows(O.q4_quantize_rows(ks[sel], hd), hd)
    vd = O.q4_dequant_rows(O.q4_quantize_rows(vs[sel], hd), hd)
    for h in range(H):
        ref = _fp64_attention(q[h], kd[:, h // 8], vd[:, h // 8], 0.125)
        assert np.abs(consistent[h] - ref).max() < 1e-4
    assert np.abs(written - consistent).max() > 1e-2


def test_lse_combine_matches_full():
    rng = np.random.default_rng(11)
    n_kv, hd, H, T, pt = 4, 64, 32, 256, 16
    src = rng.standard_normal((T, n_kv, 2, hd)).astype(np.float32)
    q4 = O.q4_quantize_rows(src, hd)                       # [T][n_kv][2][40]
    pool = np.ascontiguousarray(q4.reshape(T // pt, pt, n_kv, 2, 40).transpose(0, 2, 3, 1, 4))
    table = np.arange(T // pt, dtype=np.int32)[None]
    q = rng.standard_normal((1, H, hd)).astype(np.float32)
    parts = np.stack([O.decode_q4_partial(q, pool, table, a, b, n_kv, hd, pt)
                      for a, b in [(0, 100), (100, 101), (101, 256), (256, 256)]])
    merged = O.lse_combine(parts)
    full = O.decode_q4_window_ring(q, pool, table, np.array([T], np.int32),
                                   np.zeros((1, n_kv, 2, 1, hd), np.float32), 1, T, n_kv, hd, pt)
    # ring of 1 token reads the last position exactly; compare against partial of all tokens
    whole = O.lse_combine(O.decode_q4_partial(q, pool, table, 0, T, n_kv, hd, pt)[None])
    assert np.abs(merged - whole).max() < 1e-5
    assert full.shape == merged.shape


def test_rope_restatement_properties():
    """ops.rs:20-84: position 0 is the identity, positions past max_context use
    max_context - 1, the table equals cos / sin of the f32 angle m * freq to a
    few f32 ulps, and a rotation keeps every pair's norm."""
    hd, ctx = 64, 3000
    lut = O.rope_lut(hd, ctx)
    rng = np.random.default_rng(5)
    q = rng.standard_normal((32, hd)).astype(np.float32)
    k = rng.standard_normal((4, hd)).astype(np.float32)
    q0, k0 = O.apply_rope(q, k, 0, ctx, lut)
    assert np.array_equal(q0, q) and np.array_equal(k0, k)
    qa, _ = O.apply_rope(q, k, 10 ** 7, ctx, lut)
    qb, _ = O.apply_rope(q, k, ctx - 1, ctx, lut)
    assert np.array_equal(qa, qb)
    kk = np.arange(hd // 2, dtype=np.float32)
    freq = (np.float32(1.0) / np.power(np.float32(10000.0), (2 * kk) / np.float32(hd))).astype(np.float32)
    ang = (np.arange(ctx, dtype=np.float32)[:, None] * freq[None]).astype(np.float32).astype(np.float64)
    # freq may differ from numpy's power by an ulp, which moves large angles by ulps of the angle
    tol = 1e-6 + 4 * np.spacing(ang.astype(np.float32)).astype(np.float64)
    assert (np.abs(lut[..., 0] - np.cos(ang)) <= tol).all()
    assert (np.abs(lut[..., 1] - np.sin(ang)) <= tol).all()
    qr, _ = O.apply_rope(q, k, 1234, ctx, lut)
    n0 = np.hypot(q[:, 0::2].astype(np.float64), q[:, 1::2])
    n1 = np.hypot(qr[:, 0::2].astype(np.float64), qr[:, 1::2])
    assert np.abs(n0 - n1).max() < 1e-5


def _mojo_quirk_f64(q, k, v, positions):
    """attention.mojo:40-118 in float64 from dequantized rows k, v [n][hd]."""
    H, hd = q.shape
    out = np.zeros((H, hd))
    for h in range(H):
        m, d = -1e10, 0.0
        for t0 in range(0, len(positions), 64):
            idx = positions[t0:t0 + 64]
            s = (k[idx] @ q[h].astype(np.float64)) / np.sqrt(hd)
            mx = max(-1e10, s.max())
            td = np.exp(s - mx).sum()
            nm = max(m, mx)
            d = d * np.exp(m - nm) + td * np.exp(mx - nm)
            m = nm
            w = np.exp(s - m) / d
            keep = w >= 1e-8
            out[h] += (w[keep, None] * v[idx][keep]).sum(0)
    return out


@pytest.mark.parametrize("hd,n", [(64, 1), (64, 64), (64, 65), (32, 300), (96, 130)])
def test_mojo_sparse_attention_restatement(hd, n):
    """The Mojo kernel as written (tiles of 64, earlier tiles not rescaled):
    the C restatement equals a float64 statement of the same recurrence, and a
    single tile is plain softmax attention."""
    rng = np.random.default_rng(hd + n)
    T = 400
    kf = rng.standard_normal((T, hd)).astype(np.float32)
    vf = rng.standard_normal((T, hd)).astype(np.float32)
    kq, vq = O.q4_quantize_rows(kf, hd), O.q4_quantize_rows(vf, hd)
    kd, vd = O.q4_dequant_rows(kq, hd), O.q4_dequant_rows(vq, hd)
    q = rng.standard_normal((4, hd)).astype(np.float32)
    pos = rng.integers(0, T, n).astype(np.int32)
    got = O.mojo_sparse_attention_q4(q, O.mojo_rows_from_q4(kq), O.mojo_rows_from_q4(vq), pos)
    want = _mojo_quirk_f64(q, kd.astype(np.float64), vd.astype(np.float64), pos)
    assert np.abs(got - want).max() < 1e-4
    if n <= 64:
        for h in range(4):
            ref = _fp64_attention(q[h], kd[pos], vd[pos], 1 / np.sqrt(hd))
            assert np.abs(got[h] - ref).max() < 1e-4
