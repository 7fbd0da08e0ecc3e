/*
 * nyion_attn.h — C ABI of libnyion_attn.so, the B200 (sm_100a) attention hot
 * path of bmcc-DEV/Nyion.rs.
 *
 * Plain pointers and sizes only.  Device pointers are caller-owned unless a
 * comment says otherwise; `stream` is a cudaStream_t passed as void* (NULL =
 * the legacy default stream).  Every nyion_attn_* function returns an
 * int32_t status: 0 = NYION_OK, negative = error, with a readable message from
 * nyion_attn_last_error() (per calling thread).  There is no CPU fallback
 * behind any entry point: a missing device or an unsupported shape is an
 * error.
 *
 * Each entry point names the reference interface it replaces (paths are
 * relative to the reference repository root).
 */
#ifndef NYION_ATTN_H
#define NYION_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NYION_ATTN_VERSION 100

enum {
  NYION_OK = 0,
  NYION_ERR_INVALID = -1,      /* bad argument (null pointer, size, alignment) */
  NYION_ERR_CUDA = -2,         /* CUDA runtime error; message has the CUDA text */
  NYION_ERR_UNSUPPORTED = -3,  /* shape this build has no kernel for (e.g. head_dim != 64) */
  NYION_ERR_DEVICE = -4,       /* device error word set: page id out of range, wait timeout */
  NYION_ERR_WORKSPACE = -5     /* workspace missing or too small */
};

/* Device error word bits (nyion_attn_device_error). */
#define NYION_DEVERR_PAGE_RANGE 1
#define NYION_DEVERR_WAIT_TIMEOUT 2
#define NYION_DEVERR_SHAPE 4

/* ------------------------------------------------------------------ status */
int32_t nyion_attn_version(void);
const char* nyion_attn_last_error(void);
/* Synchronises `stream`, returns the current device's error word in *bits and
 * clears it (the bits of every entry point that has run on the device,
 * nyion_attn_decode_paged_f32_noalloc's own word included; no allocation).
 * Returns NYION_ERR_DEVICE when any bit was set.  Replaces the
 * reference's per-call stderr + `return -1` (fused_attention.cu:218-240),
 * which cannot see asynchronous device faults. */
int32_t nyion_attn_device_error(void* stream, int32_t* bits);

/* --------------------------------------------------------------- workspace */
/* Bytes of device workspace the decode entry points need for `batch`
 * sequences of `n_kv_heads` KV heads (split-KV partials + per-(seq, kv head)
 * counters).  The counters must start at zero: allocate, then call
 * nyion_attn_workspace_reset once; the kernels leave them at zero again.
 * The counters sit in a block of fixed size for a given n_kv_heads, so one
 * workspace serves every batch size up to the one it was sized for.
 * Calls that share one workspace must not overlap on the GPU. */
size_t nyion_attn_decode_workspace_size(int32_t batch, int32_t n_kv_heads, int32_t n_heads,
                                        int32_t head_dim);
int32_t nyion_attn_workspace_reset(void* workspace, size_t bytes, void* stream);

/* Host staging for callers with host buffers (the reference copies the query
 * in and the output out with cudaMemcpy around its CUDA attention call,
 * swamp-gpu/kernels/fused_attention.cu:313-330).
 * nyion_attn_host_map: the device address of page-locked host memory
 * (cudaHostAlloc / cudaHostRegister), NYION_ERR_CUDA for pageable memory.
 * nyion_attn_copy_async: copies `bytes` from src to dst on `stream` with an SM
 * kernel; either side may be a mapped host address from nyion_attn_host_map
 * or device memory.  Ranges must not overlap.  In a CUDA graph the copy is a
 * kernel node. */
int32_t nyion_attn_host_map(const void* host, void** device_ptr);
int32_t nyion_attn_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* ------------------------------------------------------ HBM arena ---------
 * The device side of HeterogeneousMemoryAllocator: the five operations of the
 * reference's DeviceAllocator trait (swamp-tensors/src/hma.rs:215-221;
 * implemented for Vulkan in swamp-gpu/src/lib.rs:101-150), from which the KV
 * page pools, page tables and per-step buffers are carved.
 * nyion_attn_arena_create reserves `capacity` bytes of HBM on the current
 * device with one cudaMalloc; allocate_device carves 256-byte-aligned blocks
 * from it (best fit; freed blocks coalesce), so allocating and freeing pages
 * calls neither cudaMalloc nor cudaFree.  allocate_unified returns managed
 * memory (host- and device-addressable; the reference's UnifiedMapped).
 * Allocations are named by a handle; *dev_ptr / *ptr is the device address
 * the attention entry points take.  upload / download copy min(bytes, size)
 * bytes between host memory and the allocation's start (synchronous for a
 * NULL stream, else on `stream`), as the reference's upload / download copy
 * min(src, dst) bytes.  No free range large enough: NYION_ERR_WORKSPACE (the
 * reference's None).  Unknown handle: NYION_ERR_INVALID.  Thread-safe.
 * nyion_attn_arena_info reports the reservation, the bytes in live device
 * blocks and the largest free range. */
int32_t nyion_attn_arena_create(size_t capacity, void** arena);
int32_t nyion_attn_arena_destroy(void* arena);
int32_t nyion_attn_arena_allocate_device(void* arena, size_t size, uint64_t* handle, void** dev_ptr);
int32_t nyion_attn_arena_allocate_unified(void* arena, size_t size, uint64_t* handle, void** ptr);
int32_t nyion_attn_arena_free(void* arena, uint64_t handle);
int32_t nyion_attn_arena_upload(void* arena, uint64_t handle, const void* src, size_t bytes, void* stream);
int32_t nyion_attn_arena_download(void* arena, uint64_t handle, void* dst, size_t bytes, void* stream);
int32_t nyion_attn_arena_info(void* arena, size_t* capacity, size_t* used, size_t* largest_free);

/* ---------------------------------------------------- paged fp32 decode ----
 * GQA decode attention with online softmax over an fp32 paged KV pool, one
 * query token per sequence.  Replaces the per-head score/softmax/AXPY loops
 * of ops::attention (swamp-engine/src/ops.rs:170-278) for a batch of
 * sequences, and the Attention node of the ComputeGraph
 * (swamp-gpu/src/compute_graph.rs:14-25, swamp-engine/src/scheduler.rs:120-171).
 *
 *   q          [batch][n_heads][head_dim] f32
 *   kv_pool    [n_pool_pages][n_kv_heads][2 (K,V)][page_tokens][head_dim] f32
 *   page_table [batch][max_pages] int32 page ids into kv_pool
 *   seq_lens   [batch] int32: sequence b attends tokens [0, seq_lens[b]) (device)
 *   out        [batch][n_heads][head_dim] f32 (zeros where seq_lens[b] == 0)
 * Query head h reads KV head h / (n_heads / n_kv_heads) (ops.rs:191).
 * scale <= 0 selects 1/sqrt(head_dim) (ops.rs:181).
 * This build: head_dim 64, n_heads / n_kv_heads == 8, page_tokens 16,
 * batch <= 512 per call (larger batches are split into several launches).
 * workspace: nyion_attn_decode_workspace_size(batch, ...) bytes, reset once;
 * NULL selects a library-owned workspace (first use allocates: not under
 * stream capture). */
int32_t nyion_attn_decode_paged_f32(const float* q, const float* kv_pool, int64_t n_pool_pages,
                                    const int32_t* page_table, int32_t max_pages,
                                    const int32_t* seq_lens, float* out, int32_t batch,
                                    int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                    int32_t page_tokens, float scale, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* ------------------------------------- paged fp32 decode, no allocation ----
 * No counterpart in the reference.  Same arguments and result as
 * nyion_attn_decode_paged_f32 without the workspace, for callers that must
 * not allocate device memory while decoding (a serving loop that cannot
 * afford cudaFree's device-wide synchronisation, a host whose HBM is fully
 * owned by its own arena, a plugin host that forbids library allocations).  The
 * split-KV scratch is a fixed 8 MiB device array inside the library, reserved
 * on every GPU that loads it; the call allocates nothing.  Limit: batch <= 512;
 * with 4 KV heads (the whole-page kernel of the main entry) every such batch
 * fits; otherwise (148 + batch * n_kv_heads) * 6 partial slots of 2112 bytes
 * must fit the 8 MiB (about batch * n_kv_heads <= 500 on B200); larger calls
 * return NYION_ERR_WORKSPACE.  The first call on a device resolves the
 * array's address (cudaGetSymbolAddress): make it before any stream capture.
 * Calls share the array: calls that overlap on the GPU race, so serialise
 * them.  Page-id range errors of this variant set its own device error word,
 * which nyion_attn_device_error reads and clears with the shared one (it
 * allocates nothing when only this entry point has run on the device).  The
 * resolved addresses belong to the current CUDA context: do not use the
 * library again after cudaDeviceReset. */
int32_t nyion_attn_decode_paged_f32_noalloc(const float* q, const float* kv_pool,
                                            int64_t n_pool_pages, const int32_t* page_table,
                                            int32_t max_pages, const int32_t* seq_lens,
                                            float* out, int32_t batch, int32_t n_heads,
                                            int32_t n_kv_heads, int32_t head_dim,
                                            int32_t page_tokens, float scale, void* stream);

/* ------------------------------------------------------------ 4-bit KV -----
 * Block format of swamp-engine/src/cache.rs:637-663: 32 values -> 20 bytes
 * [f16 d][f16 dmin][16 bytes nibbles], element i in byte i/2, low nibble for
 * even i.  Rows are head_dim values: ceil(head_dim/32) blocks per row. */

/* Quantizer of PagedKVCache::save / save_at (cache.rs:637-663, 768-807), one
 * fresh row at a time (nibbles written into zeroed bytes): bit-exact.
 * src [n_rows][head_dim] f32 -> dst [n_rows][ceil(head_dim/32)][20] bytes. */
int32_t nyion_attn_quantize_q4(const float* src, uint8_t* dst, int64_t n_rows, int32_t head_dim,
                               void* stream);
/* Dequant of ensure_f32_page_in_zone (cache.rs:375-394), bit-exact:
 * f32(d) * q + f32(dmin) with separate multiply and add. */
int32_t nyion_attn_dequant_q4(const uint8_t* src, float* dst, int64_t n_rows, int32_t head_dim,
                              void* stream);

/* Q4 paged decode over a token range per sequence, producing log-sum-exp
 * partials: the per-GPU step of the split-KV path and the 4-bit part of
 * attention_sparse_q4's window (swamp-engine/src/ops.rs:597-723, with the
 * writer-consistent nibble order of cache.rs).
 *   kv_pool    [n_pool_pages][4 KV heads][K|V][16 slots][2 blocks x 20 B]
 *   page_table [batch][max_pages] (16-token pages, absolute positions)
 *   sequence b attends tokens [tok_begin[b], tok_end[b]) (device arrays), or
 *   [u_begin, u_end) for every sequence when the arrays are NULL
 *   part       [batch][n_heads][head_dim + 2]: o normalised by l, then m (max
 *              scaled score, natural log units), l = sum exp(s - m); an empty
 *              range gives (0, -inf, 0).
 * This build: 32 query heads, 4 KV heads, head_dim 64, page_tokens 16.
 * One launch per 512 sequences: the CTAs that share a sequence merge their
 * partials in the same launch (the last to finish merges).
 * workspace: nyion_attn_q4_workspace_size(batch) bytes whose leading merge
 * counters are zero before the first call (nyion_attn_workspace_reset once;
 * every call leaves them at zero), or NULL for the library-owned one.  Calls
 * that share a workspace must not overlap on the GPU. */
size_t nyion_attn_q4_workspace_size(int32_t batch);
int32_t nyion_attn_decode_q4_partial(const float* q, const uint8_t* kv_pool, int64_t n_pool_pages,
                                     const int32_t* page_table, int32_t max_pages,
                                     const int32_t* tok_begin, const int32_t* tok_end,
                                     int32_t u_begin, int32_t u_end, float* part, int32_t batch,
                                     int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                     int32_t page_tokens, float scale, void* workspace,
                                     size_t workspace_bytes, void* stream);
/* Merges n_parts partial arrays [n_parts][rows][head_dim + 2] (the format
 * above) into out [rows][head_dim]: m = max m_g, w_g = l_g exp(m_g - m),
 * out = sum w_g o_g / sum w_g.  Rows whose partials are all empty give 0. */
int32_t nyion_attn_lse_combine(const float* parts, int32_t n_parts, int64_t rows, int32_t head_dim,
                               float* out, void* stream);
/* 4-bit windowed decode with an fp32 ring: sequence b of
 * length L = seq_lens[b] attends [max(0, L - window), L); the newest
 * min(ring_tokens, window) tokens come from the fp32 ring
 * ring [batch][4][K|V][ring_tokens][head_dim] at slot pos % ring_tokens
 * (ring_tokens <= 128), the
 * older ones from the Q4 pages.  out [batch][n_heads][head_dim].
 * workspace: nyion_attn_q4_workspace_size(batch) + 2 * batch * n_heads *
 * (head_dim + 2) * 4 + 8 * batch bytes (reset once, as above), or NULL. */
int32_t nyion_attn_decode_q4_window_ring(const float* q, const uint8_t* kv_pool,
                                         int64_t n_pool_pages, const int32_t* page_table,
                                         int32_t max_pages, const int32_t* seq_lens,
                                         const float* ring, int32_t ring_tokens, int32_t window,
                                         float* out, int32_t batch, int32_t n_heads,
                                         int32_t n_kv_heads, int32_t head_dim, int32_t page_tokens,
                                         float scale, void* workspace, size_t workspace_bytes,
                                         void* stream);

/* ------------------------------------------------ position-list decode -----
 * Attention over an explicit list of token positions per sequence, the
 * position-set form of ops::attention_sparse (swamp-engine/src/ops.rs:85-168)
 * and ops::attention_fugu (ops.rs:445-541; window, sentinel and DSPark
 * positions concatenated): scores of q against K[pos] for every listed
 * position (duplicates count twice, as in the reference's loops), softmax over
 * the set, weighted sum of V[pos].
 *   kv_format 0: kv_pool f32 [n_pool_pages][n_kv][K|V][16][head_dim]
 *   kv_format 1: kv_pool Q4  [n_pool_pages][n_kv][K|V][16][2 blocks x 20 B]
 *   positions [batch][max_positions], n_positions [batch] (device arrays):
 *   sequence b uses positions[b][0 .. n_positions[b]); an empty set gives 0.
 *   out [batch][n_heads][head_dim].
 * A position whose page entry is outside [0, n_pool_pages) is skipped and
 * raises the page-range bit of the device error word.
 * workspace: nyion_attn_positions_workspace_size(batch, n_heads,
 * max_positions) bytes (per-(sequence, KV head) merge counters first: reset
 * once with nyion_attn_workspace_reset, every call leaves them at zero), or
 * NULL.  One launch: the last CTA of each (sequence, KV head) merges the
 * splits.  This build: head_dim 64, GQA group 8. */
size_t nyion_attn_positions_workspace_size(int32_t batch, int32_t n_heads, int32_t max_positions);
int32_t nyion_attn_decode_positions(const float* q, const void* kv_pool, int32_t kv_format,
                                    int64_t n_pool_pages, const int32_t* page_table,
                                    int32_t max_pages, const int32_t* positions,
                                    const int32_t* n_positions, int32_t max_positions, float* out,
                                    int32_t batch, int32_t n_heads, int32_t n_kv_heads,
                                    int32_t head_dim, int32_t page_tokens, float scale,
                                    void* workspace, size_t workspace_bytes, void* stream);
/* ops::attention_sparse_q4 (swamp-engine/src/ops.rs:597-723) on 4-bit pages:
 * with valid_end = seq_lens[b] - 1 (the reference's min(q_pos, seq_len - 1)),
 * window_start = valid_end - window + 1 when valid_end > window, else 0, the
 * position set is { global_stride * gi : gi < min(window_start /
 * global_stride, 128) } followed by [window_start, valid_end].  The window
 * runs on the Q4 page kernel (nyion_attn_decode_q4_partial), the global
 * positions on the position kernel, which folds the window's log-sum-exp
 * partial into its own and writes `out` (two launches, plus one that turns
 * seq_lens into window ranges).  Nibbles in the writer's order (cache.rs:637-663).
 * workspace: nyion_attn_sparse_q4_workspace_size(batch, n_heads) bytes (the
 * Q4 decode's merge counters first: reset once, left at zero), or NULL. */
size_t nyion_attn_sparse_q4_workspace_size(int32_t batch, int32_t n_heads);
int32_t nyion_attn_sparse_q4(const float* q, const uint8_t* kv_pool, int64_t n_pool_pages,
                             const int32_t* page_table, int32_t max_pages, const int32_t* seq_lens,
                             int32_t window, int32_t global_stride, float* out, int32_t batch,
                             int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                             int32_t page_tokens, float scale, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ------------------------------------------- reference-layout fp32 decode ----
 * ops::attention (swamp-engine/src/ops.rs:170-278) with the same argument
 * meaning: one sequence, query head h reads KV head h / (n_heads/n_kv_heads),
 * tokens [0, min(q_pos, seq_len - 1)] attended, scale 1/sqrt(head_dim).
 * The KV cache is the reference's PagedKVCache f32 page geometry
 * (swamp-engine/src/cache.rs:17-21, 185-237, 681-747) placed in two HBM
 * arenas (K and V): flat pages 0..127 of 32 slots, 128..1119 of 128 slots,
 * then 1024-slot pages, consecutive, each [n_layers][n_kv_heads][slots][head_dim]
 * f32.  n_arena_pages = pages present in each arena.  Uses the
 * library-owned workspace (first use allocates: not under stream capture). */
int32_t nyion_attn_decode_zoned_f32(float* out, const float* q, const float* k_arena,
                                    const float* v_arena, int64_t n_arena_pages, int32_t n_layers,
                                    int32_t layer_idx, int64_t seq_len, int64_t q_pos,
                                    int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                    void* stream);
/* ops::attention_tracked (ops.rs:283-401): the same decode plus, for every
 * position t in [0, min(q_pos, seq_len - 1)], importance[t] += sum over the
 * query heads of the softmax weight p_h(t) (double, device array of seq_len;
 * masked positions are left unchanged, as adding 0 leaves them).  The weights
 * are recomputed from the scores in two small launches after the decode
 * (the path the executor takes for short sequences). */
int32_t nyion_attn_decode_zoned_f32_tracked(float* out, const float* q, const float* k_arena,
                                            const float* v_arena, int64_t n_arena_pages,
                                            int32_t n_layers, int32_t layer_idx, int64_t seq_len,
                                            int64_t q_pos, int32_t n_heads, int32_t n_kv_heads,
                                            int32_t head_dim, double* importance, void* stream);

/* ------------------------------------------- split-KV across GPUs, peer exchange ----
 * No reference counterpart (the reference has no multi-GPU attention); the
 * merge is the log-sum-exp identity of attention.mojo:89-96.  One process
 * per GPU; rank r holds the 4-bit pages of its token range [u_begin, u_end).
 * Every rank owns a mailbox (nyion_attn_splitkv_mailbox_bytes, allocated and
 * zeroed by nyion_attn_mailbox_alloc) and opens every other rank's through
 * CUDA IPC (nyion_attn_ipc_handle gives 64 bytes to send, nyion_attn_ipc_open
 * maps a received one).  nyion_attn_decode_q4_splitkv then runs the rank's
 * decode, whose CTAs that merge a sequence's partials write each (sequence,
 * head) row's partial into every rank's mailbox over peer memory as 64-bit
 * words tagged with the step's epoch; a second kernel on the same stream waits
 * (at most timeout_ms; 0 = 2000) until all ranks' words of the row carry it
 * and writes the combined attention to `out` [batch][n_heads][head_dim] on
 * every rank (two launches per call).  With world 1 the merged rows are
 * written directly by the decode (one launch, no mailbox traffic).
 * workspace: nyion_attn_q4_workspace_size(batch) bytes (reset once) or NULL.
 * `mailboxes` is a host array of `world` device pointers ([rank] = own).
 * All ranks must call it the same number of times with the same batch;
 * steps alternate two mailbox halves, so it is graph-replayable.  A wait that
 * runs out sets NYION_DEVERR_WAIT_TIMEOUT (read with nyion_attn_device_error)
 * and leaves `out` undefined.  batch <= 512, world <= 8. */
size_t nyion_attn_splitkv_mailbox_bytes(int32_t batch, int32_t n_heads);
int32_t nyion_attn_mailbox_alloc(size_t bytes, void** ptr);
int32_t nyion_attn_mailbox_free(void* ptr);
int32_t nyion_attn_ipc_handle(void* dev_ptr, void* handle_out /* 64 bytes */);
int32_t nyion_attn_ipc_open(const void* handle /* 64 bytes */, void** dev_ptr);
int32_t nyion_attn_ipc_close(void* dev_ptr);
int32_t nyion_attn_decode_q4_splitkv(const float* q, const uint8_t* kv_pool, int64_t n_pool_pages,
                                     const int32_t* page_table, int32_t max_pages, int32_t u_begin,
                                     int32_t u_end, float* out, int32_t batch, int32_t n_heads,
                                     int32_t n_kv_heads, int32_t head_dim, int32_t page_tokens,
                                     float scale, void* const* mailboxes, int32_t world, int32_t rank,
                                     int32_t timeout_ms, void* workspace, size_t workspace_bytes,
                                     void* stream);

/* ------------------------------------------------ chunked causal prefill ----
 * The attention step of prefill_slice (swamp-engine/src/executor.rs:106-138):
 * for every prompt token t of a chunk the reference calls ops::attention with
 * seq_len = pos_offset + t + 1 (ops.rs:170-278), after storing the chunk's
 * K/V at positions pos_offset.. (executor.rs:106-111); chunks are
 * PREFILL_CHUNK_SIZE = 4096 tokens (executor.rs:185).  This entry computes a
 * whole chunk at once on the tensor cores from a bf16 paged cache:
 *   q          [n_q][n_heads][head_dim] bf16, query positions q_start + i;
 *   kv_pool    [n_pool_pages][n_kv_heads][2 (K,V)][page_tokens][head_dim] bf16,
 *              already holding positions [0, q_start + n_q);
 *   page_table [max_pages] int32 page ids of the sequence;
 *   out        [n_q][n_heads][head_dim] f32.
 * Query i attends tokens [0, q_start + i]; head h reads KV head
 * h / (n_heads / n_kv_heads); scale <= 0 means 1/sqrt(head_dim).  This build
 * takes head_dim 64, GQA group 8, page_tokens 16.  Scores, probabilities and
 * products run in bf16 x bf16 -> f32 (the reference computes in f32). */
int32_t nyion_attn_prefill_paged_bf16(const void* q, const void* kv_pool, int64_t n_pool_pages,
                                      const int32_t* page_table, int32_t max_pages,
                                      int64_t q_start, int64_t n_q, float* out, int32_t n_heads,
                                      int32_t n_kv_heads, int32_t head_dim, int32_t page_tokens,
                                      float scale, void* stream);

/* ------------------------------------------------------- f16 KV caches ----
 * Decode over f16 caches [n_kv_heads][stride][head_dim] (query head h reads
 * KV head h / (n_heads / n_kv_heads); scale <= 0 means 1/sqrt(head_dim)).
 * Split-KV partials and per-KV-head merge counters go to `workspace`
 * (nyion_attn_f16_workspace_size bytes, reset once with
 * nyion_attn_workspace_reset and left with its counters at zero; null =
 * library-owned, allocated on first use: not under stream capture).
 *
 * nyion_attn_decode_contig_f16: tokens [0, seq_len) of a contiguous half
 * cache — gpu_attention_streamed_half (fused_attention.cu:534-582) with a
 * caller workspace.
 *
 * nyion_attn_decode_ring_f16: the layer-graph attention node over the f16
 * ring of `window` slots (kernel_scores_dptr / kernel_softmax_v_dptr,
 * fused_attention.cu:1505-1556): the length is read from device memory at
 * run time (*d_seq_len, clamped to [0, window] as scheduler.rs:103-171 does
 * on the host), so a captured graph replays correctly as it grows. */
size_t nyion_attn_f16_workspace_size(int32_t n_heads, int32_t max_tokens);
int32_t nyion_attn_decode_contig_f16(const float* q, const void* k_cache, const void* v_cache,
                                     float* out, int32_t n_heads, int32_t n_kv_heads,
                                     int32_t seq_len, int32_t head_dim, int32_t kv_stride,
                                     float scale, void* workspace, size_t workspace_bytes,
                                     void* stream);
int32_t nyion_attn_decode_ring_f16(const float* q, const void* k_ring, const void* v_ring,
                                   const int32_t* d_seq_len, float* out, int32_t n_heads,
                                   int32_t n_kv_heads, int32_t head_dim, int32_t window,
                                   float scale, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* ------------------------------------------------ swamp-kernels C ABIs ----
 * Q16.16 softmax (swamp-kernels/src/lib.rs:97-223), bit-exact with the
 * reference's AVX-512 path: logits -> Q16.16 at temperature T, exp in fixed
 * point, sum, normalisation (16-wide blocks with the 32-bit wrapping multiply,
 * tail with the 64-bit one).  Silent on null pointers or n <= 0, like the
 * reference.  nyion_attn_softmax_padic takes device pointers and a stream;
 * mojo_softmax_padic has the reference's name and host pointers
 * (synchronous). */
int32_t nyion_attn_softmax_padic(const float* logits, float* probs, int32_t n, float temperature,
                                 void* stream);
void mojo_softmax_padic(const float* logits, float* probs, int n, float temperature);
/* exp_q16_16 (swamp-kernels/src/lib.rs:97-103) of the softmax above, over a
 * device array: out[i] = 0 for x < -655360, 65536 for x >= 0, else
 * round(exp(x / 65536) * 65536).  Device pointers, asynchronous on `stream`. */
int32_t nyion_attn_exp_q16_16(const int32_t* x_fixed, int32_t* out, int64_t n, void* stream);

/* Stokes KV store (lib.rs:27-85), same names and arguments: keys / values of
 * head_dim floats per appended token (host pointers), a score per token;
 * above 4096 tokens the first minimum-score token is removed and the order of
 * the rest kept.  The rows live in HBM (nyion_attn_stokes_view returns device
 * pointers [n][head_dim] for the decode entry points); a NaN score, where the
 * reference panics, skips the eviction and records an error.  Not
 * thread-safe, like the reference. */
void* mojo_stokes_init(int head_dim);
void mojo_stokes_append(void* cache, int token_id, const float* key, const float* value, float score);
void mojo_stokes_free(void* cache);
int32_t nyion_attn_stokes_view(void* cache, const float** keys, const float** values, int32_t* n,
                               int32_t* head_dim);

/* ------------------------------------------------------- KV write path ----
 * The step before attention: RoPE on the new token's q and k, then K and V
 * saved into the caches, in one launch.
 * RoPE follows the CPU engine (swamp-engine/src/ops.rs:20-84): table
 * [max_context][head_dim/2] of (cos, sin), freq = 1 / 10000^(2k/head_dim),
 * angle = pos * freq; pair (2k, 2k+1) -> (x cos - y sin, x sin + y cos);
 * position clamped to max_context - 1.  nyion_attn_rope_table builds the
 * table on the host with the C library's powf / cosf / sinf (what Rust's f32
 * methods call) and uploads it to `table` (nyion_attn_rope_table_bytes),
 * synchronously; rotated vectors are then bit-identical to apply_rope_ufc's. */
size_t nyion_attn_rope_table_bytes(int32_t head_dim, int32_t max_context);
int32_t nyion_attn_rope_table(float* table, int32_t head_dim, int32_t max_context, void* stream);
/* Rows = new tokens (a decode batch, or the tokens of a prefill chunk).
 *   q  [rows][n_heads][head_dim] f32, rotated in place (NULL: no q);
 *   k  [rows][n_kv_heads][head_dim] f32, rotated in place; v likewise, read;
 *   positions [rows] absolute positions; row_seq [rows] the sequence (page
 *   table row, ring row) of each row, NULL = row i is sequence i;
 *   rope_table NULL = no rotation (a plain save).
 * Destinations, each optional (NULL skips it), all at position pos of the
 * row's sequence, page = page_table[seq][pos / 16], slot = pos % 16:
 *   pool_q4   [n_pool_pages][n_kv][K|V][16][2 x 20 B]: PagedKVCache::save's
 *             4-bit blocks of a fresh slot (cache.rs:637-663), bit-exact;
 *   pool_f32  [n_pool_pages][n_kv][K|V][16][head_dim] f32 (save's f32 copy,
 *             cache.rs:671-677);
 *   pool_bf16 same layout in bf16 (RNE), the chunked prefill's cache;
 *   q_bf16    [rows][n_heads][head_dim] bf16 copy of the rotated q;
 *   ring_f32  [n_seq][n_kv][K|V][ring_tokens][head_dim] at pos % ring_tokens
 *             (the windowed 4-bit decode's fp32 ring).
 * A row whose page is missing (pos outside the table, id outside the pool)
 * writes no page and raises the page-range device error bit.  This build:
 * head_dim 64, n_kv_heads <= 16. */
int32_t nyion_attn_kv_write_paged(float* q, float* k, const float* v, const int32_t* positions,
                                  const int32_t* row_seq, int32_t rows, int32_t n_heads,
                                  int32_t n_kv_heads, int32_t head_dim, const float* rope_table,
                                  int32_t max_context, const int32_t* page_table,
                                  int32_t max_pages, int64_t n_pool_pages, uint8_t* pool_q4,
                                  float* pool_f32, void* pool_bf16, void* q_bf16,
                                  float* ring_f32, int32_t ring_tokens, void* stream);
/* Layer-graph steps RoPE + KV save (swamp-gpu/kernels/fused_attention.cu:
 * 1438-1472, 1619-1625) for one sequence, graph-capturable: pos =
 * *d_seq_len - 1 read on the device, slot = *d_wpos (or pos % window when
 * d_wpos is NULL); k_ring / v_ring [n_kv][window][head_dim] f16 (RNE).  RoPE
 * as above (the CPU engine's table; the reference's CUDA kernel evaluates
 * powf / cosf / sinf under --use_fast_math instead). */
int32_t nyion_attn_kv_write_ring_f16(float* q, float* k, const float* v, const int32_t* d_seq_len,
                                     const int32_t* d_wpos, void* k_ring, void* v_ring,
                                     int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                     int32_t window, const float* rope_table, int32_t max_context,
                                     void* stream);

/* ------------------------------------------------------- cold-tier pages ----
 * The reference's NVMe cold slot (swamp-engine/src/cache.rs:251-276, 440-483,
 * 485-529): [K q4 page][V q4 page], a q4 page = [n_layers][n_kv][block_slots]
 * [ceil(head_dim/32) x 20 B] (cache.rs:681-747), block_slots 32 / 128 / 1024
 * for zones 0 / 1 / 2; the reference reads and writes slot s of a zone at
 * file offset s * 2 * q4_page_bytes(zone) (nyion_attn_cold_slot_offset).
 * nyion_attn_cold_to_pool scatters one slot into per-layer 4-bit page pools
 * [n_pool_pages][n_kv][K|V][16][40] (the format the Q4 kernels read):
 * layer_pools = host array of n_layers device pool pointers (8-byte aligned,
 * n_layers <= 128), page_ids = device [n_layers][block_slots / 16]
 * destination page of each 16-slot run.  `slot` may be HBM or pinned host
 * memory mapped into the device address space (read over the bus); every
 * pointer is checked with cudaPointerGetAttributes before the launch.
 * nyion_attn_pool_to_cold gathers the same pages back into a slot image
 * (eviction).  Page ids outside [0, n_pool_pages) raise the page-range bit
 * and move nothing for those rows.  This build: head_dim 64. */
size_t nyion_attn_cold_q4_page_bytes(int32_t block_slots, int32_t n_layers, int32_t n_kv_heads,
                                     int32_t head_dim);
int64_t nyion_attn_cold_slot_offset(int64_t slot, int32_t block_slots, int32_t n_layers,
                                    int32_t n_kv_heads, int32_t head_dim);
int32_t nyion_attn_cold_to_pool(const uint8_t* slot, int32_t block_slots, int32_t n_layers,
                                int32_t n_kv_heads, int32_t head_dim, uint8_t* const* layer_pools,
                                const int32_t* page_ids, int64_t n_pool_pages, void* stream);
int32_t nyion_attn_pool_to_cold(uint8_t* const* layer_pools, const int32_t* page_ids,
                                int32_t block_slots, int32_t n_layers, int32_t n_kv_heads,
                                int32_t head_dim, int64_t n_pool_pages, uint8_t* slot,
                                void* stream);

/* ------------------------------------------------- O-projection Q4_K GEMV ----
 * The layer graph's GEMV (swamp-gpu/kernels/fused_attention.cu:858-925) so
 * the attention output stays on the device: w = Q4_K super-blocks of 256
 * columns (144 B: f16 d, f16 dmin, 12 B of 6-bit scales/mins, 128 B of
 * nibbles), column-major at super-block level (block b of row r at
 * (b * n_rows + r) * 144, as gpu_upload_weights_transposed stores them),
 * weight = d (nib - 8) scale_sb + dmin min_sb as the reference kernel
 * computes it.  x [batch][n_blocks * 256] f32, out [batch][n_rows] f32;
 * w 16-byte aligned. */
int32_t nyion_attn_gemv_q4k(const uint8_t* w, const float* x, float* out, int32_t n_rows,
                            int32_t n_blocks, int32_t batch, void* stream);
/* fused_attention.cu:916-925, same name and arguments (batch 1). */
void gpu_gemv_q4k(const uint8_t* d_w, const float* d_x, float* d_out, int n_rows, int n_blocks,
                  void* stream);

/* ----------------------------------------------------------- Mojo FFI -----
 * swamp-gpu/kernels/attention.mojo:122-152 `sparse_attention_q4`, with the
 * argument list its Rust binding declares (swamp-gpu/src/mojo.rs:5, 65-97):
 * raw host pointers q [n_heads][head_dim] f32, k_q4 / v_q4 rows of
 * ceil(head_dim/32) blocks x 20 f32 [d, dmin, 16 byte values, 2 unused]
 * indexed by position, positions [n_sparse] int32, out [n_heads][head_dim];
 * window and global_stride unused (as in the Mojo kernel).  Tiles of 64
 * positions with the kernel's running (m, d) per tile and no rescaling of
 * earlier tiles, weights < 1e-8 skipped — as written.  Only the listed rows
 * are copied to the GPU; synchronous.  head_dim <= 256. */
void sparse_attention_q4(uint64_t q, uint64_t k_q4, uint64_t v_q4, uint64_t positions, uint64_t out,
                         int32_t n_heads, int32_t head_dim, int32_t n_sparse, int32_t window,
                         int32_t global_stride);

/* ---------------------------------------------- reference CUDA C ABI -------
 * Same names, arguments and 0 / -1 results as swamp-gpu/kernels/fused_attention.cu,
 * so the reference's Rust declarations (swamp-gpu/src/lib.rs:586-677) link
 * against this library unchanged.  K/V are contiguous
 * [n_kv_heads][kv_stride][head_dim]; the decode attends tokens [0, seq_len).
 * On failure the message is in nyion_attn_last_error() (the reference prints
 * to stderr). */

/* fused_attention.cu:194-243 (device pointers, default stream) */
int gpu_attention_device(const float* d_q, const float* d_k_cache, const float* d_v_cache,
                         float* d_output, int n_heads, int n_kv_heads, int seq_len, int head_dim,
                         int kv_stride);
/* fused_attention.cu:483-531 */
int gpu_attention_streamed(const float* d_q, const float* d_k_cache, const float* d_v_cache,
                           float* d_output, int n_heads, int n_kv_heads, int seq_len,
                           int head_dim, int kv_stride, void* stream);
/* fused_attention.cu:335-405 (host pointers; copies in and out, synchronous) */
int gpu_attention_forward(const float* q, const float* k_cache, const float* v_cache,
                          float* output, int n_heads, int n_kv_heads, int seq_len, int head_dim);
/* fused_attention.cu:597-664: a replayable CUDA graph of one decode at fixed
 * shapes.  d_scores is accepted for ABI compatibility and not used (scores
 * never leave on-chip memory).  Returns NULL on failure. */
void* gpu_graph_create_attention(const float* d_q, const float* d_k_cache,
                                 const float* d_v_cache, float* d_scores, float* d_output,
                                 int n_heads, int n_kv_heads, int seq_len, int head_dim,
                                 int kv_stride);
/* fused_attention.cu:669-679 (either kind of graph handle) */
int gpu_graph_replay_attention(void* graph_handle, void* stream);
/* fused_attention.cu:682-686 (either kind of graph handle) */
void gpu_graph_destroy(void* graph_handle);
/* fused_attention.cu:534-582: f16 K/V cache ([n_kv][kv_stride][head_dim] half;
 * `void*` here so C callers need no half type) */
int gpu_attention_streamed_half(const float* d_q, const void* d_k_cache, const void* d_v_cache,
                                float* d_output, int n_heads, int n_kv_heads, int seq_len,
                                int head_dim, int kv_stride, void* stream);
/* fused_attention.cu:244-258 / 744-762: cudaMalloc of [n_kv][max_seq_len][head_dim]
 * f32 / f16; NULL on failure. */
void* gpu_alloc_kv_buffer(int n_kv_heads, int max_seq_len, int head_dim, size_t* out_bytes);
void* gpu_alloc_kv_buffer_half(int n_kv_heads, int max_seq_len, int head_dim, size_t* out_bytes);
/* fused_attention.cu:260-285: one (kv_head, pos) row, host -> device, synchronous */
int gpu_copy_kv_to_buffer(float* d_buf, const float* h_src, int kv_head, int pos, int n_kv_heads,
                          int max_seq_len, int head_dim);
/* fused_attention.cu:287-312, 456-481: all KV heads of position pos
 * (h_src [n_kv][head_dim]) in one strided copy; synchronous / on `stream` */
int gpu_copy_kv_layer(float* d_buf, const float* h_src, int pos, int n_kv_heads, int max_seq_len,
                      int head_dim);
int gpu_copy_kv_layer_async(float* d_buf, const float* h_src, int pos, int n_kv_heads,
                            int max_seq_len, int head_dim, void* stream);
/* fused_attention.cu:764-812: host f32 [n_kv][head_dim] -> f16 (RNE) rows of
 * d_buf [n_kv][max_seq_len][head_dim] at pos, through a library-owned device
 * staging buffer, on `stream` */
int gpu_copy_kv_layer_async_half(void* d_buf, const float* h_src, int pos, int n_kv_heads,
                                 int max_seq_len, int head_dim, void* stream);
/* fused_attention.cu:687-717 */
void* gpu_graph_create_attention_half(const float* d_q, const void* d_k_cache,
                                      const void* d_v_cache, float* d_scores, float* d_output,
                                      int n_heads, int n_kv_heads, int seq_len, int head_dim,
                                      int kv_stride);

#ifdef __cplusplus
}
#endif

#endif /* NYION_ATTN_H */
