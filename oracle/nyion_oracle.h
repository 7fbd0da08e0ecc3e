/*
 * nyion_oracle.h — CPU restatement of the reference attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * kernels in nyion.rs_b200/csrc and the timed CPU baseline of bench.py.  The
 * product path never links, loads or calls it; only tests/, the smoke() check
 * in __graft_entry__.py and bench.py's cpu_baseline / --impl reference legs do.
 *
 * Every function restates one piece of the reference (bmcc-DEV/Nyion.rs) and
 * cites the file:line it follows.  The reference's Rust cannot be compiled in
 * this environment (no cargo/rustc, crates not vendored), so it is restated in
 * C with the same operation order:
 *   - swamp-kernels/src/simd.rs        dot/AXPY (16-lane FMA + quarter reduce)
 *   - swamp-engine/src/cache.rs        zone geometry, Q4 quantizer, dequant
 *   - swamp-engine/src/ops.rs          attention, attention_tracked,
 *                                      attention_sparse_q4
 *   - swamp-kernels/src/lib.rs         Q16.16 softmax, Stokes KV store
 * plus the new-layout references (16-token page table, Q4 window + fp32 ring,
 * bf16 causal prefill, split-KV log-sum-exp merge) built from the same
 * per-head algorithm.
 */
#ifndef NYION_ORACLE_H
#define NYION_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- half precision (half 2.7.1 f16::from_f32 / to_f32 semantics) ---- */
uint16_t or_f16_from_f32(float x);        /* IEEE binary16, round-to-nearest-even */
float    or_f16_to_f32(uint16_t h);       /* exact */
int      or_f16c_available(void);         /* 1 if the host CPU has F16C */
uint16_t or_f16_from_f32_f16c(float x);   /* hardware conversion, for cross-checks */

/* ---- zone geometry (cache.rs:17-21, 185-237, 593-611) ---- */
int64_t or_zone_index(int64_t pos);
int64_t or_block_size_for(int64_t pos);
int64_t or_page_id(int64_t pos);
int64_t or_slot_in_page(int64_t pos);
int64_t or_page_start_for(int64_t pos);
int64_t or_zone_page_count(int zone, int64_t max_seq_len);
int64_t or_total_pages(int64_t max_seq_len);
/* flat page id -> (zone, block size); returns block size, writes zone */
int64_t or_resolve_flat(int64_t flat_id, int* zone);

/* ---- Q4 block: [f16 d][f16 dmin][16 B nibbles] per 32 values ---- */
/* Quantizes `len` (<=32) values into `blk` (20 bytes), OR-ing nibbles into the
 * existing bytes exactly like cache.rs:637-663.  Pass a zeroed block for a
 * first write. */
void or_q4_quantize_block(const float* src, int len, uint8_t* blk);
/* Dequantizes one block (cache.rs:375-394): d*q + dmin, separate mul and add */
void or_q4_dequant_block(const uint8_t* blk, int len, float* dst);
/* Whole rows: src [n_rows][head_dim] -> dst [n_rows][blocks*20] (zeroed first) */
void or_q4_quantize_rows(const float* src, int64_t n_rows, int head_dim, uint8_t* dst);
void or_q4_dequant_rows(const uint8_t* src, int64_t n_rows, int head_dim, float* dst);

/* ---- SIMD inner loops (simd.rs:37-68, 108-121, 145-180) ---- */
float or_dot_product_raw(const float* a, const float* b, int n);
void  or_weighted_sum_raw(float* out, const float* v, float score, int n);
int   or_avx512_available(void);

/* ---- reference-layout page store (cache.rs PagedKVCache) ----
 * k_pages[flat_id] / v_pages[flat_id] point at f32 pages laid out
 * [layer][kv_head][slot][head_dim] with slot count = the zone's block size. */
void or_attention(float* out, const float* q,
                  const float* const* k_pages, const float* const* v_pages,
                  int n_layers, int layer_idx, int64_t seq_len, int64_t q_pos,
                  int n_heads, int n_kv_heads, int head_dim);
void or_attention_tracked(float* out, const float* q,
                          const float* const* k_pages, const float* const* v_pages,
                          int n_layers, int layer_idx, int64_t seq_len, int64_t q_pos,
                          int n_heads, int n_kv_heads, int head_dim, double* importance);
/* attention_sparse_q4 (ops.rs:597-723).  q4 pages are [layer][kv][slot][blk*20].
 * as_written=1 reproduces the reference's nibble/lane pairing; 0 pairs element
 * i with q[i] (the writer-consistent order of cache.rs). */
void or_attention_sparse_q4(float* out, const float* q,
                            const uint8_t* const* k_q4_pages, const uint8_t* const* v_q4_pages,
                            int n_layers, int layer_idx, int64_t seq_len, int64_t q_pos,
                            int n_heads, int n_kv_heads, int head_dim,
                            int64_t window, int64_t global_stride, int as_written);
/* the position set of attention_sparse / attention_sparse_q4 (ops.rs:101-113) */
int64_t or_sparse_positions(int64_t seq_len, int64_t q_pos, int64_t window,
                            int64_t global_stride, int64_t* positions, int64_t cap);

/* ---- RoPE of the CPU engine (swamp-engine/src/ops.rs:20-84) ---- */
/* lut [max_seq_len][head_dim/2][2] = (cos, sin) of pos * 10000^(-2k/head_dim) */
void or_rope_lut(float* lut, int head_dim, int64_t max_seq_len);
/* rotates q [n_q_heads][head_dim] and k [n_kv_heads][head_dim] in place at
 * min(pos, max_context - 1) */
void or_apply_rope(float* q, float* k, int64_t pos, int n_q_heads, int n_kv_heads, int head_dim,
                   int64_t max_context, const float* lut);

/* ---- Mojo sparse_attention_q4 (swamp-gpu/kernels/attention.mojo:40-152) ----
 * rows of ceil(hd/32) blocks x 20 floats [d, dmin, 16 byte values, 2 unused];
 * tiles of 64 positions; earlier tiles are not rescaled (as written). */
void or_mojo_sparse_attention_q4(const float* q, const float* k_q4, const float* v_q4,
                                 const int32_t* positions, float* out, int n_heads, int head_dim,
                                 int n_sparse);

/* ---- Q4_K GEMV of the layer graph (swamp-gpu/kernels/fused_attention.cu:858-914) ----
 * w column-major super-blocks (block b of row r at (b * n_rows + r) * 144),
 * x [n_blocks * 256], out [n_rows]; the kernel's formula as written. */
void or_gemv_q4k(const uint8_t* w, const float* x, float* out, int n_rows, int n_blocks);

/* ---- Q16.16 softmax (swamp-kernels/src/lib.rs:97-223) ---- */
int32_t or_exp_q16_16(int32_t x_fixed);
void    or_exp_q16_16_many(const int32_t* x_fixed, int32_t* out, int64_t n);
void    or_softmax_padic(const float* logits, float* probs, int n, float temperature);

/* ---- Stokes KV store (swamp-kernels/src/lib.rs:27-85) ---- */
void* or_stokes_init(int head_dim);
void  or_stokes_append(void* h, int token_id, const float* k, const float* v, float score);
void  or_stokes_free(void* h);
int64_t or_stokes_len(void* h);
const float* or_stokes_keys(void* h);
const float* or_stokes_values(void* h);
const float* or_stokes_scores(void* h);

/* ---- new-layout references (per-head algorithm of ops.rs:170-278) ---- */
/* 16-token (page_tokens) fp32 pages: page = [n_kv][2 (K,V)][page_tokens][head_dim].
 * Sequence b attends tokens [0, seq_lens[b]).  q/out [batch][n_heads][head_dim].
 * n_threads > 1 splits (batch x head) across pthreads. */
void or_decode_paged_f32(float* out, const float* q, const float* pool,
                         const int32_t* page_table, const int32_t* seq_lens,
                         int batch, int max_pages, int n_heads, int n_kv_heads,
                         int head_dim, int page_tokens, float scale, int n_threads);
/* Q4 pages: page = [n_kv][2][page_tokens][blocks*20].  Attends tokens
 * [max(0,L-window), L) with tokens >= L-ring_tokens read from the fp32 ring
 * ring [batch][n_kv][2][ring_tokens][head_dim] at slot pos % ring_tokens and the
 * rest dequantized (cache.rs:375-394) from the Q4 pages. */
void or_decode_q4_window_ring(float* out, const float* q, const uint8_t* pool,
                              const int32_t* page_table, const int32_t* seq_lens,
                              const float* ring, int ring_tokens, int64_t window,
                              int batch, int max_pages, int n_heads, int n_kv_heads,
                              int head_dim, int page_tokens, float scale, int n_threads);
/* Partial (m, l, o) over tokens [tok_begin, tok_end) of Q4 pages, in the
 * log-sum-exp form the split-KV merge consumes: part [batch][n_heads][head_dim+2]
 * = (o (normalised by l), m, l) with scores pre-scaled by `scale`. */
void or_decode_q4_partial(float* part, const float* q, const uint8_t* pool,
                          const int32_t* page_table, int64_t tok_begin, int64_t tok_end,
                          int batch, int max_pages, int n_heads, int n_kv_heads,
                          int head_dim, int page_tokens, float scale, int n_threads);
/* Merge G partials [G][rows][head_dim+2] into out [rows][head_dim] (double). */
void or_lse_combine(float* out, const float* parts, int G, int64_t rows, int head_dim);
/* Causal chunked prefill over bf16 pages: page = [n_kv][2][page_tokens][head_dim]
 * bf16 (raw uint16).  Queries q [n_q][n_heads][head_dim] bf16 at positions
 * q_start + i attend tokens [0, q_start + i]; out fp32 [n_q][n_heads][head_dim].
 * Accumulates in double. */
void or_prefill_paged_bf16(float* out, const uint16_t* q, const uint16_t* pool,
                           const int32_t* page_table, int max_pages, int64_t q_start,
                           int64_t n_q, int n_heads, int n_kv_heads, int head_dim,
                           int page_tokens, float scale, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
