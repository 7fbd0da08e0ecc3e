/*
 * nyion_oracle.c — CPU restatement of the reference attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see nyion_oracle.h).  Compiled with
 * -ffp-contract=off so that every multiply and add that the reference writes
 * separately stays separate; fused multiply-adds appear only where the
 * reference itself uses an FMA intrinsic (simd.rs, ops.rs:650-717).
 */
#include "nyion_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ======================================================================= */
/* half precision                                                           */
/* ======================================================================= */

/* IEEE binary16 round-to-nearest-even; the behaviour of half 2.7.1
 * f16::from_f32 (used by cache.rs:651-652 and 779-780), including subnormals,
 * overflow to infinity and quiet NaNs. */
uint16_t or_f16_from_f32(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t exp = (u >> 23) & 0xffu;
    uint32_t man = u & 0x7fffffu;
    if (exp == 0xffu) {
        if (man) return (uint16_t)(sign | 0x7c00u | 0x0200u | (man >> 13));
        return (uint16_t)(sign | 0x7c00u);
    }
    int e = (int)exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t hm = man >> shift;
        uint32_t rb = 1u << (shift - 1);
        if ((man & rb) && (man & (3u * rb - 1u))) hm += 1u;
        return (uint16_t)(sign | hm);
    }
    uint32_t r = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rb = 0x1000u;
    if ((man & rb) && (man & (3u * rb - 1u))) r += 1u;
    return (uint16_t)r;
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else {
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            man &= 0x3ffu;
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

int or_f16c_available(void) {
#if defined(__x86_64__)
    return __builtin_cpu_supports("f16c");
#else
    return 0;
#endif
}

#if defined(__x86_64__)
__attribute__((target("f16c")))
static uint16_t f16c_cvt(float x) {
    return (uint16_t)_cvtss_sh(x, _MM_FROUND_TO_NEAREST_INT);
}
#endif

uint16_t or_f16_from_f32_f16c(float x) {
#if defined(__x86_64__)
    if (or_f16c_available()) return f16c_cvt(x);
#endif
    return or_f16_from_f32(x);
}

/* ======================================================================= */
/* zone geometry — cache.rs:17-21 (constants), 185-237, 593-611             */
/* ======================================================================= */

static const int64_t ZONE_STARTS[3] = {0, 4096, 131072};
static const int64_t ZONE_BLOCK[3] = {32, 128, 1024};

int64_t or_zone_index(int64_t pos) {              /* cache.rs:211-215 */
    if (pos < ZONE_STARTS[1]) return 0;
    if (pos < ZONE_STARTS[2]) return 1;
    return 2;
}

int64_t or_block_size_for(int64_t pos) {          /* cache.rs:233-235 */
    return ZONE_BLOCK[or_zone_index(pos)];
}

/* build_zones (cache.rs:185-200): zones 0 and 1 always span up to the next
 * zone start; zone 2 spans up to max_seq_len. */
int64_t or_zone_page_count(int zone, int64_t max_seq_len) {
    int64_t start = ZONE_STARTS[zone];
    int64_t end = zone + 1 < 3 ? ZONE_STARTS[zone + 1] : max_seq_len;
    int64_t cov = end > start ? end - start : 0;
    return cov > 0 ? (cov + ZONE_BLOCK[zone] - 1) / ZONE_BLOCK[zone] : 0;
}

int64_t or_total_pages(int64_t max_seq_len) {
    return or_zone_page_count(0, max_seq_len) + or_zone_page_count(1, max_seq_len) +
           or_zone_page_count(2, max_seq_len);
}

/* zone_page_offsets (cache.rs:202-209) do not depend on max_seq_len for the
 * first two zones: {0, 128, 1120}. */
static int64_t zone_offset(int zone) {
    int64_t acc = 0;
    for (int z = 0; z < zone; z++) acc += or_zone_page_count(z, ZONE_STARTS[2]);
    return acc;
}

int64_t or_page_id(int64_t pos) {                 /* cache.rs:593-597 */
    int zi = (int)or_zone_index(pos);
    int64_t local = (pos - ZONE_STARTS[zi]) / ZONE_BLOCK[zi];
    return zone_offset(zi) + local;
}

int64_t or_slot_in_page(int64_t pos) {            /* cache.rs:604-610 */
    int zi = (int)or_zone_index(pos);
    return (pos - ZONE_STARTS[zi]) % ZONE_BLOCK[zi];
}

int64_t or_page_start_for(int64_t pos) {          /* cache.rs:599-602 */
    return pos - or_slot_in_page(pos);
}

int64_t or_resolve_flat(int64_t flat_id, int* zone) {   /* cache.rs:221-228 */
    for (int zi = 2; zi >= 0; zi--) {
        if (flat_id >= zone_offset(zi)) {
            if (zone) *zone = zi;
            return ZONE_BLOCK[zi];
        }
    }
    if (zone) *zone = -1;
    return -1;
}

/* ======================================================================= */
/* Q4 block — quantizer cache.rs:637-663 (save) / 768-807 (save_at),        */
/* dequant cache.rs:375-394                                                  */
/* ======================================================================= */

void or_q4_quantize_block(const float* src, int len, uint8_t* blk) {
    float mx = 0.0f, mn = 3.40282347e+38f;           /* f32::MAX */
    for (int i = 0; i < len; i++) {
        mx = fmaxf(mx, fabsf(src[i]));
        mn = fminf(mn, src[i]);
    }
    float d = mx > 1e-10f ? mx / 7.0f : 0.0f;
    float dmin = mn;
    uint16_t hd = or_f16_from_f32(d), hm = or_f16_from_f32(dmin);
    blk[0] = (uint8_t)(hd & 0xff);
    blk[1] = (uint8_t)(hd >> 8);
    blk[2] = (uint8_t)(hm & 0xff);
    blk[3] = (uint8_t)(hm >> 8);
    for (int i = 0; i < len; i++) {
        uint8_t q = 0;
        if (d > 1e-10f) {
            float r = roundf((src[i] - dmin) / d);
            r = fminf(fmaxf(r, 0.0f), 15.0f);
            q = (uint8_t)r;                     /* saturating `as u8`; r in [0,15] */
        }
        int shift = (i % 2 == 0) ? 0 : 4;
        blk[4 + i / 2] = (uint8_t)(blk[4 + i / 2] | (uint8_t)(q << shift));
    }
}

void or_q4_dequant_block(const uint8_t* blk, int len, float* dst) {
    float d = or_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    float dmin = or_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
    for (int i = 0; i < len; i++) {
        uint8_t b = blk[4 + i / 2];
        uint8_t nib = (i % 2 == 0) ? (b & 0x0f) : (b >> 4);
        float prod = d * (float)nib;            /* separate mul and add */
        dst[i] = prod + dmin;
    }
}

void or_q4_quantize_rows(const float* src, int64_t n_rows, int head_dim, uint8_t* dst) {
    int nblk = (head_dim + 31) / 32;
    for (int64_t r = 0; r < n_rows; r++) {
        uint8_t* row = dst + r * nblk * 20;
        memset(row, 0, (size_t)nblk * 20);
        for (int b = 0; b < nblk; b++) {
            int start = b * 32;
            int end = start + 32 < head_dim ? start + 32 : head_dim;
            or_q4_quantize_block(src + r * head_dim + start, end - start, row + b * 20);
        }
    }
}

void or_q4_dequant_rows(const uint8_t* src, int64_t n_rows, int head_dim, float* dst) {
    int nblk = (head_dim + 31) / 32;
    for (int64_t r = 0; r < n_rows; r++) {
        for (int b = 0; b < nblk; b++) {
            int start = b * 32;
            int end = start + 32 < head_dim ? start + 32 : head_dim;
            or_q4_dequant_block(src + (r * nblk + b) * 20, end - start, dst + r * head_dim + start);
        }
    }
}

/* ======================================================================= */
/* dot / AXPY — simd.rs:37-68 (dot_product_avx512), 108-121                 */
/* ======================================================================= */

/* Scalar statement of the AVX-512 order: 16 independent lanes of fmaf over
 * full 16-wide chunks, an 8-wide chunk into lanes 0..7, a scalar mul-add tail,
 * then (q0+q1)+(q2+q3) over 128-bit quarters followed by two hadds. */
static float dot_scalar(const float* a, const float* b, int n) {
    float lane[16] = {0};
    int i = 0;
    while (i + 16 <= n) {
        for (int j = 0; j < 16; j++) lane[j] = fmaf(a[i + j], b[i + j], lane[j]);
        i += 16;
    }
    float tail = 0.0f;
    if (i + 8 <= n) {
        for (int j = 0; j < 8; j++) lane[j] = fmaf(a[i + j], b[i + j], lane[j]);
        i += 8;
    }
    while (i < n) {
        float p = a[i] * b[i];
        tail = tail + p;
        i++;
    }
    float s[4];
    for (int j = 0; j < 4; j++) {
        float s1 = lane[j] + lane[4 + j];
        float s2 = lane[8 + j] + lane[12 + j];
        s[j] = s1 + s2;
    }
    float h0 = s[0] + s[1], h1 = s[2] + s[3];
    float r = h0 + h1;
    return r + tail;
}

static void axpy_scalar(float* out, const float* v, float score, int n) {
    int i = 0;
    while (i + 16 <= n) {
        for (int j = 0; j < 16; j++) out[i + j] = fmaf(score, v[i + j], out[i + j]);
        i += 16;
    }
    while (i < n) {
        float p = score * v[i];
        out[i] = out[i] + p;
        i++;
    }
}

#if defined(__x86_64__)
__attribute__((target("avx512f")))
static float dot_avx512(const float* a, const float* b, int n) {
    __m512 sum = _mm512_setzero_ps();
    int i = 0;
    while (i + 16 <= n) {
        sum = _mm512_fmadd_ps(_mm512_loadu_ps(a + i), _mm512_loadu_ps(b + i), sum);
        i += 16;
    }
    float tail = 0.0f;
    if (i + 8 <= n) {
        __m512 va = _mm512_zextps256_ps512(_mm256_loadu_ps(a + i));
        __m512 vb = _mm512_zextps256_ps512(_mm256_loadu_ps(b + i));
        sum = _mm512_fmadd_ps(va, vb, sum);
        i += 8;
    }
    while (i < n) {
        float p = a[i] * b[i];
        tail = tail + p;
        i++;
    }
    __m128 lo = _mm512_extractf32x4_ps(sum, 0);
    __m128 hi = _mm512_extractf32x4_ps(sum, 1);
    __m128 hi2 = _mm512_extractf32x4_ps(sum, 2);
    __m128 hi3 = _mm512_extractf32x4_ps(sum, 3);
    __m128 s = _mm_add_ps(_mm_add_ps(lo, hi), _mm_add_ps(hi2, hi3));
    s = _mm_hadd_ps(s, s);
    s = _mm_hadd_ps(s, s);
    return _mm_cvtss_f32(s) + tail;
}

__attribute__((target("avx512f")))
static void axpy_avx512(float* out, const float* v, float score, int n) {
    __m512 sb = _mm512_set1_ps(score);
    int i = 0;
    while (i + 16 <= n) {
        _mm512_storeu_ps(out + i, _mm512_fmadd_ps(sb, _mm512_loadu_ps(v + i), _mm512_loadu_ps(out + i)));
        i += 16;
    }
    while (i < n) {
        float p = score * v[i];
        out[i] = out[i] + p;
        i++;
    }
}

/* AVX2 emulation of the same 16-lane order (two 8-lane accumulators). */
__attribute__((target("avx2,fma")))
static float dot_avx2_16lane(const float* a, const float* b, int n) {
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    int i = 0;
    while (i + 16 <= n) {
        acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc0);
        acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), acc1);
        i += 16;
    }
    float tail = 0.0f;
    if (i + 8 <= n) {
        acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc0);
        i += 8;
    }
    while (i < n) {
        float p = a[i] * b[i];
        tail = tail + p;
        i++;
    }
    __m128 lo = _mm256_castps256_ps128(acc0), hi = _mm256_extractf128_ps(acc0, 1);
    __m128 hi2 = _mm256_castps256_ps128(acc1), hi3 = _mm256_extractf128_ps(acc1, 1);
    __m128 s = _mm_add_ps(_mm_add_ps(lo, hi), _mm_add_ps(hi2, hi3));
    s = _mm_hadd_ps(s, s);
    s = _mm_hadd_ps(s, s);
    return _mm_cvtss_f32(s) + tail;
}

__attribute__((target("avx2,fma")))
static void axpy_avx2(float* out, const float* v, float score, int n) {
    __m256 sb = _mm256_set1_ps(score);
    int i = 0;
    while (i + 16 <= n) {
        _mm256_storeu_ps(out + i, _mm256_fmadd_ps(sb, _mm256_loadu_ps(v + i), _mm256_loadu_ps(out + i)));
        _mm256_storeu_ps(out + i + 8, _mm256_fmadd_ps(sb, _mm256_loadu_ps(v + i + 8), _mm256_loadu_ps(out + i + 8)));
        i += 16;
    }
    while (i < n) {
        float p = score * v[i];
        out[i] = out[i] + p;
        i++;
    }
}
#endif

static int g_isa = -1;   /* 2 = avx512, 1 = avx2+fma, 0 = scalar */

static int isa(void) {
    if (g_isa < 0) {
#if defined(__x86_64__)
        if (getenv("NYION_ORACLE_SCALAR")) g_isa = 0;
        else if (__builtin_cpu_supports("avx512f")) g_isa = 2;
        else if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) g_isa = 1;
        else g_isa = 0;
#else
        g_isa = 0;
#endif
    }
    return g_isa;
}

int or_avx512_available(void) { return isa() == 2; }

float or_dot_product_raw(const float* a, const float* b, int n) {
#if defined(__x86_64__)
    int k = isa();
    if (k == 2) return dot_avx512(a, b, n);
    if (k == 1) return dot_avx2_16lane(a, b, n);
#endif
    return dot_scalar(a, b, n);
}

void or_weighted_sum_raw(float* out, const float* v, float score, int n) {
#if defined(__x86_64__)
    int k = isa();
    if (k == 2) { axpy_avx512(out, v, score, n); return; }
    if (k == 1) { axpy_avx2(out, v, score, n); return; }
#endif
    axpy_scalar(out, v, score, n);
}

/* ======================================================================= */
/* per-head attention — ops.rs:192-276 (body of the par_chunks_mut closure)  */
/* ======================================================================= */

/* One query head over n_valid key/value rows; the masked tail of the
 * reference (positions valid_end+1 .. seq_len-1, ops.rs:233-235) contributes
 * exp(-inf) = 0 to the sum and is skipped by the AXPY loop, so it needs no
 * explicit representation.  `scores` is caller scratch of n_valid floats. */
static void attend_head(float* out, const float* q, const float* const* k_rows,
                        const float* const* v_rows, int64_t n_valid, int head_dim,
                        float scale, float* scores, double* importance, const int64_t* imp_pos) {
    float max_score = -INFINITY;
    for (int64_t t = 0; t < n_valid; t++) {
        float s = or_dot_product_raw(q, k_rows[t], head_dim) * scale;
        scores[t] = s;
        if (s > max_score) max_score = s;
    }
    float sum_exp = 0.0f;
    for (int64_t t = 0; t < n_valid; t++) {
        float e = expf(scores[t] - max_score);
        scores[t] = e;
        sum_exp += e;
    }
    float inv_sum = 1.0f / sum_exp;
    for (int64_t t = 0; t < n_valid; t++) scores[t] *= inv_sum;
    if (importance) {
        for (int64_t t = 0; t < n_valid; t++)
            importance[imp_pos ? imp_pos[t] : t] += (double)scores[t];
    }
    memset(out, 0, sizeof(float) * (size_t)head_dim);
    for (int64_t t = 0; t < n_valid; t++) or_weighted_sum_raw(out, v_rows[t], scores[t], head_dim);
}

static void zoned_rows(const float* const* pages, int n_layers, int layer, int n_kv, int kv_h,
                       int head_dim, int64_t n, const float** rows) {
    (void)n_layers;
    for (int64_t t = 0; t < n; t++) {
        int zone;
        int64_t pid = or_page_id(t);
        int64_t bs = or_resolve_flat(pid, &zone);
        int64_t slot = or_slot_in_page(t);
        rows[t] = pages[pid] + (((int64_t)layer * n_kv + kv_h) * bs + slot) * head_dim;
    }
}

/* ops.rs:170-278 */
void or_attention(float* out, const float* q, const float* const* k_pages,
                  const float* const* v_pages, int n_layers, int layer_idx, int64_t seq_len,
                  int64_t q_pos, int n_heads, int n_kv_heads, int head_dim) {
    or_attention_tracked(out, q, k_pages, v_pages, n_layers, layer_idx, seq_len, q_pos, n_heads,
                         n_kv_heads, head_dim, NULL);
}

/* ops.rs:283-401 (importance summed over heads in head order) */
void or_attention_tracked(float* out, const float* q, const float* const* k_pages,
                          const float* const* v_pages, int n_layers, int layer_idx,
                          int64_t seq_len, int64_t q_pos, int n_heads, int n_kv_heads,
                          int head_dim, double* importance) {
    float scale = 1.0f / sqrtf((float)head_dim);
    int n_rep = n_heads / n_kv_heads;
    int64_t valid_end = q_pos < seq_len - 1 ? q_pos : seq_len - 1;
    int64_t n_valid = valid_end + 1;
    const float** kr = (const float**)malloc(sizeof(float*) * (size_t)n_valid);
    const float** vr = (const float**)malloc(sizeof(float*) * (size_t)n_valid);
    float* scores = (float*)malloc(sizeof(float) * (size_t)n_valid);
    for (int h = 0; h < n_heads; h++) {
        int kv_h = h / n_rep;
        zoned_rows(k_pages, n_layers, layer_idx, n_kv_heads, kv_h, head_dim, n_valid, kr);
        zoned_rows(v_pages, n_layers, layer_idx, n_kv_heads, kv_h, head_dim, n_valid, vr);
        attend_head(out + (int64_t)h * head_dim, q + (int64_t)h * head_dim, kr, vr, n_valid,
                    head_dim, scale, scores, importance, NULL);
    }
    free(kr);
    free(vr);
    free(scores);
}

/* ops.rs:101-113 / 614-622 */
int64_t or_sparse_positions(int64_t seq_len, int64_t q_pos, int64_t window,
                            int64_t global_stride, int64_t* positions, int64_t cap) {
    int64_t valid_end = q_pos < seq_len - 1 ? q_pos : seq_len - 1;
    int64_t window_start = valid_end > window ? valid_end - window + 1 : 0;
    int64_t global_count = window_start / global_stride;
    if (global_count > 128) global_count = 128;
    int64_t n = 0;
    for (int64_t gi = 0; gi < global_count; gi++) {
        if (n < cap) positions[n] = global_stride * gi;
        n++;
    }
    for (int64_t t = window_start; t <= valid_end; t++) {
        if (n < cap) positions[n] = t;
        n++;
    }
    return n;
}

/* ops.rs:597-723.  as_written pairs the 16 even-element nibbles with q[0..16)
 * and the odd ones with q[16..32) (and scatters V the same way), exactly as the
 * reference's lane layout does; writer-consistent pairs element i with q[i]. */
void or_attention_sparse_q4(float* out, const float* q, const uint8_t* const* k_q4_pages,
                            const uint8_t* const* v_q4_pages, int n_layers, int layer_idx,
                            int64_t seq_len, int64_t q_pos, int n_heads, int n_kv_heads,
                            int head_dim, int64_t window, int64_t global_stride,
                            int as_written) {
    (void)n_layers;
    float scale = 1.0f / sqrtf((float)head_dim);
    int n_rep = n_heads / n_kv_heads;
    int64_t cap = window + 130;
    int64_t* pos = (int64_t*)malloc(sizeof(int64_t) * (size_t)cap);
    int64_t k = or_sparse_positions(seq_len, q_pos, window, global_stride, pos, cap);
    if (k > cap) {
        free(pos);
        pos = (int64_t*)malloc(sizeof(int64_t) * (size_t)k);
        or_sparse_positions(seq_len, q_pos, window, global_stride, pos, k);
    }
    int nblk = (head_dim + 31) / 32;
    float* scores = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
    for (int h = 0; h < n_heads; h++) {
        int kv_h = h / n_rep;
        const float* qh = q + (int64_t)h * head_dim;
        float* oh = out + (int64_t)h * head_dim;
        float max_score = -INFINITY;
        for (int64_t idx = 0; idx < k; idx++) {
            int64_t t = pos[idx];
            int64_t pid = or_page_id(t);
            int zone;
            int64_t bs = or_resolve_flat(pid, &zone);
            int64_t slot = or_slot_in_page(t);
            const uint8_t* page = k_q4_pages[pid] + ((int64_t)layer_idx * n_kv_heads + kv_h) * bs * nblk * 20;
            float acc[16] = {0};
            for (int b = 0; b < nblk; b++) {
                const uint8_t* base = page + (slot * nblk + b) * 20;
                float d = or_f16_to_f32((uint16_t)(base[0] | (base[1] << 8)));
                float dmin = or_f16_to_f32((uint16_t)(base[2] | (base[3] << 8)));
                for (int j = 0; j < 16; j++) {
                    uint8_t byte = base[4 + j];
                    float klo = fmaf(d, (float)(byte & 0x0f), dmin);   /* element 2j   */
                    float khi = fmaf(d, (float)(byte >> 4), dmin);     /* element 2j+1 */
                    float qlo, qhi;
                    if (as_written) { qlo = qh[b * 32 + j]; qhi = qh[b * 32 + 16 + j]; }
                    else { qlo = qh[b * 32 + 2 * j]; qhi = qh[b * 32 + 2 * j + 1]; }
                    acc[j] = fmaf(klo, qlo, acc[j]);
                    acc[j] = fmaf(khi, qhi, acc[j]);
                }
            }
            float dot = 0.0f;
            for (int j = 0; j < 16; j++) dot += acc[j];
            float s = dot * scale;
            scores[idx] = s;
            if (s > max_score) max_score = s;
        }
        float sum_exp = 0.0f;
        for (int64_t idx = 0; idx < k; idx++) {
            float e = expf(scores[idx] - max_score);
            scores[idx] = e;
            sum_exp += e;
        }
        float inv_sum = 1.0f / sum_exp;
        for (int64_t idx = 0; idx < k; idx++) scores[idx] *= inv_sum;
        memset(oh, 0, sizeof(float) * (size_t)head_dim);
        for (int64_t idx = 0; idx < k; idx++) {
            float w = scores[idx];
            if (w < 1e-8f) continue;
            int64_t t = pos[idx];
            int64_t pid = or_page_id(t);
            int zone;
            int64_t bs = or_resolve_flat(pid, &zone);
            int64_t slot = or_slot_in_page(t);
            const uint8_t* page = v_q4_pages[pid] + ((int64_t)layer_idx * n_kv_heads + kv_h) * bs * nblk * 20;
            for (int b = 0; b < nblk; b++) {
                const uint8_t* base = page + (slot * nblk + b) * 20;
                float d = or_f16_to_f32((uint16_t)(base[0] | (base[1] << 8)));
                float dmin = or_f16_to_f32((uint16_t)(base[2] | (base[3] << 8)));
                for (int j = 0; j < 16; j++) {
                    uint8_t byte = base[4 + j];
                    float vlo = fmaf(d, (float)(byte & 0x0f), dmin);
                    float vhi = fmaf(d, (float)(byte >> 4), dmin);
                    int olo = as_written ? b * 32 + j : b * 32 + 2 * j;
                    int ohi = as_written ? b * 32 + 16 + j : b * 32 + 2 * j + 1;
                    oh[olo] = fmaf(vlo, w, oh[olo]);
                    oh[ohi] = fmaf(vhi, w, oh[ohi]);
                }
            }
        }
    }
    free(scores);
    free(pos);
}

/* ======================================================================= */
/* RoPE — swamp-engine/src/ops.rs:20-84                                      */
/* ======================================================================= */

/* init_rope_lut (ops.rs:20-38): freq = 1 / theta^((2k) / head_dim) in f32,
 * angle = m * freq, (cos, sin) of the angle; libm powf / cosf / sinf are the
 * functions Rust's f32::powf / cos / sin call. */
void or_rope_lut(float* lut, int head_dim, int64_t max_seq_len) {
    int half = head_dim / 2;
    for (int64_t m = 0; m < max_seq_len; m++) {
        for (int k = 0; k < half; k++) {
            float freq = 1.0f / powf(10000.0f, (float)(2 * k) / (float)head_dim);
            float angle = (float)m * freq;
            lut[(m * half + k) * 2] = cosf(angle);
            lut[(m * half + k) * 2 + 1] = sinf(angle);
        }
    }
}

/* apply_rotation_pair (ops.rs:70-84): x' = x cos - y sin, y' = x sin + y cos */
static void rope_rotate(float* vec, const float* cs, int half) {
    for (int k = 0; k < half; k++) {
        float x = vec[2 * k], y = vec[2 * k + 1];
        float c = cs[2 * k], s = cs[2 * k + 1];
        vec[2 * k] = x * c - y * s;
        vec[2 * k + 1] = x * s + y * c;
    }
}

/* apply_rope_ufc (ops.rs:42-68): position clamped to max_context - 1 */
void or_apply_rope(float* q, float* k, int64_t pos, int n_q_heads, int n_kv_heads, int head_dim,
                   int64_t max_context, const float* lut) {
    int half = head_dim / 2;
    if (pos > max_context - 1) pos = max_context - 1;
    const float* cs = lut + pos * half * 2;
    for (int h = 0; h < n_q_heads; h++) rope_rotate(q + (int64_t)h * head_dim, cs, half);
    for (int h = 0; h < n_kv_heads; h++) rope_rotate(k + (int64_t)h * head_dim, cs, half);
}

/* ======================================================================= */
/* Mojo sparse_attention_q4 — swamp-gpu/kernels/attention.mojo:40-152       */
/* ======================================================================= */

static float mojo_dequant(const float* blk, int i) {        /* attention.mojo:70-78 */
    int byte = (int)blk[2 + i / 2];
    int nib = (byte >> ((i % 2) * 4)) & 0x0F;
    return blk[0] * (float)nib + blk[1];
}

/* flash_attn_head (attention.mojo:40-118) for every head (:122-152) */
void or_mojo_sparse_attention_q4(const float* q, const float* k_q4, const float* v_q4,
                                 const int32_t* positions, float* out, int n_heads, int head_dim,
                                 int n_sparse) {
    const int blocks = (head_dim + 31) / 32, blk_f = blocks * 20;
    const float scale = 1.0f / sqrtf((float)head_dim);
    float scores[64];
    for (int h = 0; h < n_heads; h++) {
        const float* qh = q + (int64_t)h * head_dim;
        float* oh = out + (int64_t)h * head_dim;
        float m = -1e10f, d = 0.0f;
        for (int i = 0; i < head_dim; i++) oh[i] = 0.0f;
        for (int t0 = 0; t0 < n_sparse; t0 += 64) {
            int n_tile = n_sparse - t0 < 64 ? n_sparse - t0 : 64;
            float max_score = -1e10f;
            for (int p = 0; p < n_tile; p++) {
                const float* kr = k_q4 + (int64_t)positions[t0 + p] * blk_f;
                float dot = 0.0f;
                for (int b = 0; b < blocks; b++)
                    for (int i = 0; i < 32 && b * 32 + i < head_dim; i++)
                        dot += mojo_dequant(kr + b * 20, i) * qh[b * 32 + i];
                float sc = dot * scale;
                scores[p] = sc;
                if (sc > max_score) max_score = sc;
            }
            float tile_d = 0.0f;
            for (int p = 0; p < n_tile; p++) tile_d += expf(scores[p] - max_score);
            float new_m = fmaxf(m, max_score);
            d = d * expf(m - new_m) + tile_d * expf(max_score - new_m);
            m = new_m;
            for (int p = 0; p < n_tile; p++) {
                float w = expf(scores[p] - m) / d;
                if (w < 1e-8f) continue;
                const float* vr = v_q4 + (int64_t)positions[t0 + p] * blk_f;
                for (int b = 0; b < blocks; b++)
                    for (int i = 0; i < 32 && b * 32 + i < head_dim; i++)
                        oh[b * 32 + i] += mojo_dequant(vr + b * 20, i) * w;
            }
        }
    }
}

/* ======================================================================= */
/* Q4_K GEMV — swamp-gpu/kernels/fused_attention.cu:858-914                  */
/* ======================================================================= */

void or_gemv_q4k(const uint8_t* w, const float* x, float* out, int n_rows, int n_blocks) {
    for (int row = 0; row < n_rows; row++) {
        float total = 0.0f;
        for (int blk = 0; blk < n_blocks; blk++) {
            const uint8_t* b = w + ((size_t)blk * n_rows + row) * 144;
            float d = or_f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
            float dmin = or_f16_to_f32((uint16_t)(b[2] | (b[3] << 8)));
            float scales[8], mins[8];
            for (int j = 0; j < 4; j++) {
                scales[j] = (float)(b[4 + j] & 63);
                mins[j] = (float)(b[8 + j] & 63);
            }
            for (int j = 4; j < 8; j++) {
                scales[j] = (float)((b[8 + j] & 0xF) | ((b[4 + j - 4] >> 6) << 4));
                mins[j] = (float)((b[8 + j] >> 4) | ((b[4 + j] >> 6) << 4));
            }
            const uint8_t* qs = b + 16;
            float dot = 0.0f;
            for (int sb = 0; sb < 8; sb++) {
                for (int k = 0; k < 32; k++) {
                    int nib = (qs[sb * 16 + k / 2] >> ((k % 2) * 4)) & 0x0F;
                    float xk = x[blk * 256 + sb * 32 + k];
                    dot += (d * (float)(nib - 8) * scales[sb] + dmin * mins[sb]) * xk;
                }
            }
            total += dot;
        }
        out[row] = total;
    }
}

/* ======================================================================= */
/* Q16.16 softmax — swamp-kernels/src/lib.rs:97-223 (AVX-512 path)          */
/* ======================================================================= */

int32_t or_exp_q16_16(int32_t x_fixed) {         /* lib.rs:97-103 */
    if (x_fixed < -655360) return 0;
    if (x_fixed >= 0) return 65536;
    float x_real = (float)x_fixed / 65536.0f;
    float r = roundf(expf(x_real) * 65536.0f);
    r = fmaxf(r, 0.0f);
    return (int32_t)r;
}

void or_exp_q16_16_many(const int32_t* x_fixed, int32_t* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = or_exp_q16_16(x_fixed[i]);
}

static int32_t sat_f32_to_i32(float x) {          /* Rust `as i32` */
    if (x != x) return 0;
    if (x >= 2147483648.0f) return 2147483647;
    if (x <= -2147483648.0f) return (int32_t)0x80000000u;
    return (int32_t)x;
}

/* mojo_softmax_padic (lib.rs:181-223) taking the AVX-512 kernel
 * (lib.rs:108-179): 16-wide blocks normalise with a 32-bit wrapping multiply
 * then a logical shift, the scalar tail with a 64-bit multiply. */
void or_softmax_padic(const float* logits, float* probs, int n, float temperature) {
    if (!logits || !probs || n <= 0) return;
    float inv_tmp = 1.0f / fmaxf(temperature, 1e-6f);
    int32_t* fixed = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
    int32_t* fo = (int32_t*)calloc((size_t)n, sizeof(int32_t));
    for (int i = 0; i < n; i++) {
        float a = logits[i] * inv_tmp;
        fixed[i] = sat_f32_to_i32(a * 65536.0f);
    }
    int32_t max_val = INT32_MIN;
    for (int i = 0; i < n; i++) if (fixed[i] > max_val) max_val = fixed[i];
    int64_t sum = 0;
    for (int i = 0; i < n; i++) {
        int32_t diff = (int32_t)((uint32_t)fixed[i] - (uint32_t)max_val);
        int32_t e = or_exp_q16_16(diff);
        fo[i] = e;
        sum += e;
    }
    if (sum > 0) {
        int32_t inv_sum = (int32_t)(uint32_t)((1ull << 32) / (uint64_t)sum);
        /* 16-wide blocks cover [0, 16*floor(n/16)): _mm512_mullo_epi32 keeps the
         * low 32 bits, _mm512_srli_epi32 shifts them logically. */
        int simd_end = (n / 16) * 16;
        for (int i = 0; i < simd_end; i++) {
            uint32_t mul = (uint32_t)fo[i] * (uint32_t)inv_sum;
            fo[i] = (int32_t)(mul >> 16);
        }
        for (int i = simd_end; i < n; i++)
            fo[i] = (int32_t)(((int64_t)fo[i] * (int64_t)inv_sum) >> 16);
    }
    for (int i = 0; i < n; i++) probs[i] = (float)fo[i] / 65536.0f;
    free(fixed);
    free(fo);
}

/* ======================================================================= */
/* Stokes KV store — swamp-kernels/src/lib.rs:27-85                          */
/* ======================================================================= */

typedef struct {
    int64_t n, cap, hd;
    float* keys;
    float* values;
    float* scores;
} stokes_t;

void* or_stokes_init(int head_dim) {
    stokes_t* s = (stokes_t*)calloc(1, sizeof(stokes_t));
    s->hd = head_dim;
    return s;
}

void or_stokes_append(void* h, int token_id, const float* k, const float* v, float score) {
    (void)token_id;
    stokes_t* s = (stokes_t*)h;
    if (!s || !k || !v) return;
    if (s->n + 1 > s->cap) {
        s->cap = s->cap ? s->cap * 2 : 64;
        s->keys = (float*)realloc(s->keys, sizeof(float) * (size_t)(s->cap * s->hd));
        s->values = (float*)realloc(s->values, sizeof(float) * (size_t)(s->cap * s->hd));
        s->scores = (float*)realloc(s->scores, sizeof(float) * (size_t)s->cap);
    }
    memcpy(s->keys + s->n * s->hd, k, sizeof(float) * (size_t)s->hd);
    memcpy(s->values + s->n * s->hd, v, sizeof(float) * (size_t)s->hd);
    s->scores[s->n] = score;
    s->n++;
    if (s->n > 4096) {
        /* min_by with partial_cmp: first index of the minimum */
        int64_t mi = 0;
        for (int64_t i = 1; i < s->n; i++) if (s->scores[i] < s->scores[mi]) mi = i;
        memmove(s->keys + mi * s->hd, s->keys + (mi + 1) * s->hd,
                sizeof(float) * (size_t)((s->n - mi - 1) * s->hd));
        memmove(s->values + mi * s->hd, s->values + (mi + 1) * s->hd,
                sizeof(float) * (size_t)((s->n - mi - 1) * s->hd));
        memmove(s->scores + mi, s->scores + mi + 1, sizeof(float) * (size_t)(s->n - mi - 1));
        s->n--;
    }
}

void or_stokes_free(void* h) {
    stokes_t* s = (stokes_t*)h;
    if (!s) return;
    free(s->keys);
    free(s->values);
    free(s->scores);
    free(s);
}

int64_t or_stokes_len(void* h) { return h ? ((stokes_t*)h)->n : 0; }
const float* or_stokes_keys(void* h) { return ((stokes_t*)h)->keys; }
const float* or_stokes_values(void* h) { return ((stokes_t*)h)->values; }
const float* or_stokes_scores(void* h) { return ((stokes_t*)h)->scores; }

/* ======================================================================= */
/* new-layout references                                                     */
/* ======================================================================= */

typedef struct {
    int kind;              /* 0 paged f32, 1 q4 window+ring, 2 q4 partial, 3 prefill */
    float* out;
    const float* q;
    const void* pool;
    const int32_t* page_table;
    const int32_t* seq_lens;
    const float* ring;
    int ring_tokens;
    int64_t window;
    int64_t tok_begin, tok_end;
    int batch, max_pages, n_heads, n_kv, hd, pt;
    float scale;
    /* prefill */
    const uint16_t* q16;
    int64_t q_start, n_q;
    /* work split */
    int64_t item_begin, item_end;
} job_t;

static const float* paged_row_f32(const float* pool, const int32_t* table, int max_pages, int b,
                                  int64_t t, int n_kv, int kv_h, int kv, int pt, int hd) {
    int64_t page = table[(int64_t)b * max_pages + t / pt];
    int64_t slot = t % pt;
    return pool + (((page * n_kv + kv_h) * 2 + kv) * pt + slot) * hd;
}

static const uint8_t* paged_row_q4(const uint8_t* pool, const int32_t* table, int max_pages, int b,
                                   int64_t t, int n_kv, int kv_h, int kv, int pt, int nblk) {
    int64_t page = table[(int64_t)b * max_pages + t / pt];
    int64_t slot = t % pt;
    return pool + ((((page * n_kv + kv_h) * 2 + kv) * pt + slot) * nblk) * 20;
}

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static void run_items(job_t* j) {
    int hd = j->hd, n_rep = j->n_heads / j->n_kv, nblk = (hd + 31) / 32;
    for (int64_t it = j->item_begin; it < j->item_end; it++) {
        if (j->kind == 3) {
            int64_t i = it / j->n_heads;
            int h = (int)(it % j->n_heads), kv_h = h / n_rep;
            int64_t pos = j->q_start + i, n = pos + 1;
            const uint16_t* qh = j->q16 + (i * j->n_heads + h) * hd;
            const uint16_t* pool = (const uint16_t*)j->pool;
            double* s = (double*)malloc(sizeof(double) * (size_t)n);
            double mx = -INFINITY;
            for (int64_t t = 0; t < n; t++) {
                int64_t page = j->page_table[t / j->pt], slot = t % j->pt;
                const uint16_t* kr = pool + (((page * j->n_kv + kv_h) * 2 + 0) * j->pt + slot) * hd;
                double acc = 0.0;
                for (int d = 0; d < hd; d++) acc += (double)bf16_to_f32(qh[d]) * (double)bf16_to_f32(kr[d]);
                s[t] = acc * (double)j->scale;
                if (s[t] > mx) mx = s[t];
            }
            double l = 0.0;
            for (int64_t t = 0; t < n; t++) { s[t] = exp(s[t] - mx); l += s[t]; }
            double* o = (double*)calloc((size_t)hd, sizeof(double));
            for (int64_t t = 0; t < n; t++) {
                int64_t page = j->page_table[t / j->pt], slot = t % j->pt;
                const uint16_t* vr = pool + (((page * j->n_kv + kv_h) * 2 + 1) * j->pt + slot) * hd;
                for (int d = 0; d < hd; d++) o[d] += s[t] * (double)bf16_to_f32(vr[d]);
            }
            float* oh = j->out + (i * j->n_heads + h) * hd;
            for (int d = 0; d < hd; d++) oh[d] = (float)(o[d] / l);
            free(o);
            free(s);
            continue;
        }
        int b = (int)(it / j->n_heads), h = (int)(it % j->n_heads), kv_h = h / n_rep;
        const float* qh = j->q + ((int64_t)b * j->n_heads + h) * hd;
        int64_t t0, t1, ring_from = INT64_MAX;
        if (j->kind == 0) {
            t0 = 0;
            t1 = j->seq_lens[b];
        } else if (j->kind == 1) {
            t1 = j->seq_lens[b];
            t0 = t1 - j->window > 0 ? t1 - j->window : 0;
            ring_from = t1 - j->ring_tokens > 0 ? t1 - j->ring_tokens : 0;
        } else {
            t0 = j->tok_begin;
            t1 = j->tok_end;
        }
        int64_t n = t1 > t0 ? t1 - t0 : 0;
        float* out_row = j->kind == 2 ? j->out + ((int64_t)b * j->n_heads + h) * (hd + 2)
                                      : j->out + ((int64_t)b * j->n_heads + h) * hd;
        if (n == 0) {
            memset(out_row, 0, sizeof(float) * (size_t)hd);
            if (j->kind == 2) { out_row[hd] = -INFINITY; out_row[hd + 1] = 0.0f; }
            continue;
        }
        if (j->kind == 2) {
            /* partial over Q4 rows: the same per-head algorithm as attend_head
             * (scores, max, serial exp sum, normalised AXPY), keeping (max,
             * sum); each row is dequantized when it is used, so memory does
             * not grow with the range (the values are the same either way) */
            float* scores = (float*)malloc(sizeof(float) * (size_t)n);
            float row[hd];
            float mx = -INFINITY;
            for (int64_t i = 0; i < n; i++) {
                const uint8_t* pk = paged_row_q4((const uint8_t*)j->pool, j->page_table, j->max_pages, b, t0 + i,
                                                 j->n_kv, kv_h, 0, j->pt, nblk);
                or_q4_dequant_rows(pk, 1, hd, row);
                float sc = or_dot_product_raw(qh, row, hd) * j->scale;
                scores[i] = sc;
                if (sc > mx) mx = sc;
            }
            float l = 0.0f;
            for (int64_t i = 0; i < n; i++) { float e = expf(scores[i] - mx); scores[i] = e; l += e; }
            float inv = 1.0f / l;
            for (int64_t i = 0; i < n; i++) scores[i] *= inv;
            memset(out_row, 0, sizeof(float) * (size_t)hd);
            for (int64_t i = 0; i < n; i++) {
                const uint8_t* pv = paged_row_q4((const uint8_t*)j->pool, j->page_table, j->max_pages, b, t0 + i,
                                                 j->n_kv, kv_h, 1, j->pt, nblk);
                or_q4_dequant_rows(pv, 1, hd, row);
                or_weighted_sum_raw(out_row, row, scores[i], hd);
            }
            out_row[hd] = mx;
            out_row[hd + 1] = l;
            free(scores);
            continue;
        }
        const float** kr = (const float**)malloc(sizeof(float*) * (size_t)n);
        const float** vr = (const float**)malloc(sizeof(float*) * (size_t)n);
        float* deq = NULL;
        if (j->kind != 0) deq = (float*)malloc(sizeof(float) * (size_t)(n * 2 * hd));
        for (int64_t i = 0; i < n; i++) {
            int64_t t = t0 + i;
            if (j->kind == 0) {
                kr[i] = paged_row_f32((const float*)j->pool, j->page_table, j->max_pages, b, t, j->n_kv, kv_h, 0, j->pt, hd);
                vr[i] = paged_row_f32((const float*)j->pool, j->page_table, j->max_pages, b, t, j->n_kv, kv_h, 1, j->pt, hd);
            } else if (t >= ring_from) {
                int64_t slot = t % j->ring_tokens;
                kr[i] = j->ring + ((((int64_t)b * j->n_kv + kv_h) * 2 + 0) * j->ring_tokens + slot) * hd;
                vr[i] = j->ring + ((((int64_t)b * j->n_kv + kv_h) * 2 + 1) * j->ring_tokens + slot) * hd;
            } else {
                const uint8_t* pk = paged_row_q4((const uint8_t*)j->pool, j->page_table, j->max_pages, b, t, j->n_kv, kv_h, 0, j->pt, nblk);
                const uint8_t* pv = paged_row_q4((const uint8_t*)j->pool, j->page_table, j->max_pages, b, t, j->n_kv, kv_h, 1, j->pt, nblk);
                or_q4_dequant_rows(pk, 1, hd, deq + (2 * i) * hd);
                or_q4_dequant_rows(pv, 1, hd, deq + (2 * i + 1) * hd);
                kr[i] = deq + (2 * i) * hd;
                vr[i] = deq + (2 * i + 1) * hd;
            }
        }
        float* scores = (float*)malloc(sizeof(float) * (size_t)n);
        attend_head(out_row, qh, kr, vr, n, hd, j->scale, scores, NULL, NULL);
        free(scores);
        free(deq);
        free(kr);
        free(vr);
    }
}

static void* run_items_thread(void* p) {
    run_items((job_t*)p);
    return NULL;
}

static void run_parallel(job_t* base, int64_t n_items, int n_threads) {
    if (n_threads <= 1 || n_items <= 1) {
        base->item_begin = 0;
        base->item_end = n_items;
        run_items(base);
        return;
    }
    if (n_threads > n_items) n_threads = (int)n_items;
    job_t* jobs = (job_t*)malloc(sizeof(job_t) * (size_t)n_threads);
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)n_threads);
    for (int i = 0; i < n_threads; i++) {
        jobs[i] = *base;
        jobs[i].item_begin = n_items * i / n_threads;
        jobs[i].item_end = n_items * (i + 1) / n_threads;
        pthread_create(&th[i], NULL, run_items_thread, &jobs[i]);
    }
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
}

void or_decode_paged_f32(float* out, const float* q, const float* pool, const int32_t* page_table,
                         const int32_t* seq_lens, int batch, int max_pages, int n_heads,
                         int n_kv_heads, int head_dim, int page_tokens, float scale,
                         int n_threads) {
    job_t j;
    memset(&j, 0, sizeof(j));
    j.kind = 0; j.out = out; j.q = q; j.pool = pool; j.page_table = page_table;
    j.seq_lens = seq_lens; j.batch = batch; j.max_pages = max_pages; j.n_heads = n_heads;
    j.n_kv = n_kv_heads; j.hd = head_dim; j.pt = page_tokens; j.scale = scale;
    run_parallel(&j, (int64_t)batch * n_heads, n_threads);
}

void or_decode_q4_window_ring(float* out, const float* q, const uint8_t* pool,
                              const int32_t* page_table, const int32_t* seq_lens,
                              const float* ring, int ring_tokens, int64_t window, int batch,
                              int max_pages, int n_heads, int n_kv_heads, int head_dim,
                              int page_tokens, float scale, int n_threads) {
    job_t j;
    memset(&j, 0, sizeof(j));
    j.kind = 1; j.out = out; j.q = q; j.pool = pool; j.page_table = page_table;
    j.seq_lens = seq_lens; j.ring = ring; j.ring_tokens = ring_tokens; j.window = window;
    j.batch = batch; j.max_pages = max_pages; j.n_heads = n_heads; j.n_kv = n_kv_heads;
    j.hd = head_dim; j.pt = page_tokens; j.scale = scale;
    run_parallel(&j, (int64_t)batch * n_heads, n_threads);
}

void or_decode_q4_partial(float* part, const float* q, const uint8_t* pool,
                          const int32_t* page_table, int64_t tok_begin, int64_t tok_end,
                          int batch, int max_pages, int n_heads, int n_kv_heads, int head_dim,
                          int page_tokens, float scale, int n_threads) {
    job_t j;
    memset(&j, 0, sizeof(j));
    j.kind = 2; j.out = part; j.q = q; j.pool = pool; j.page_table = page_table;
    j.tok_begin = tok_begin; j.tok_end = tok_end; j.batch = batch; j.max_pages = max_pages;
    j.n_heads = n_heads; j.n_kv = n_kv_heads; j.hd = head_dim; j.pt = page_tokens;
    j.scale = scale;
    run_parallel(&j, (int64_t)batch * n_heads, n_threads);
}

void or_lse_combine(float* out, const float* parts, int G, int64_t rows, int head_dim) {
    int w = head_dim + 2;
    for (int64_t r = 0; r < rows; r++) {
        double M = -INFINITY;
        for (int g = 0; g < G; g++) {
            const float* p = parts + ((int64_t)g * rows + r) * w;
            if (p[head_dim + 1] > 0.0f && p[head_dim] > M) M = p[head_dim];
        }
        double den = 0.0;
        double acc[1024];
        for (int d = 0; d < head_dim; d++) acc[d] = 0.0;
        if (M != -INFINITY) {
            for (int g = 0; g < G; g++) {
                const float* p = parts + ((int64_t)g * rows + r) * w;
                if (!(p[head_dim + 1] > 0.0f)) continue;
                double wt = (double)p[head_dim + 1] * exp((double)p[head_dim] - M);
                den += wt;
                for (int d = 0; d < head_dim; d++) acc[d] += wt * (double)p[d];
            }
        }
        for (int d = 0; d < head_dim; d++) out[r * head_dim + d] = den > 0.0 ? (float)(acc[d] / den) : 0.0f;
    }
}

void or_prefill_paged_bf16(float* out, const uint16_t* q, const uint16_t* pool,
                           const int32_t* page_table, int max_pages, int64_t q_start, int64_t n_q,
                           int n_heads, int n_kv_heads, int head_dim, int page_tokens, float scale,
                           int n_threads) {
    job_t j;
    memset(&j, 0, sizeof(j));
    j.kind = 3; j.out = out; j.q16 = q; j.pool = pool; j.page_table = page_table;
    j.max_pages = max_pages; j.q_start = q_start; j.n_q = n_q; j.n_heads = n_heads;
    j.n_kv = n_kv_heads; j.hd = head_dim; j.pt = page_tokens; j.scale = scale;
    run_parallel(&j, n_q * n_heads, n_threads);
}
