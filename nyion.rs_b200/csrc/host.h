// host.h — internal host-side helpers shared by the entry points.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "nyion_attn.h"

namespace nyion {

// Records a message for nyion_attn_last_error() and returns `status`.
int32_t fail(int32_t status, const char* fmt, ...);
// Maps a CUDA runtime error to NYION_ERR_CUDA with its text; 0 on success.
int32_t check_cuda(cudaError_t e, const char* what);

struct DeviceInfo {
  int device;
  int num_sms;
  int32_t* err_word;  // device error word (lazily allocated, zeroed)
};
// Info for the current device; allocates the error word on first use.
int32_t device_info(DeviceInfo** out);
// The current device's error word if device_info has already set it up on
// this device, else null (never allocates).
int32_t* device_error_word_if_ready();
// The allocation-free decode's own error word on the current device once that
// entry point has run there, else null (decode_f32.cu; never allocates).
int32_t* noalloc_error_word_if_ready();

// Sets `func`'s dynamic shared-memory limit to `smem` bytes on the current
// device (once per kernel and device) and returns in *occ (when non-null) how
// many blocks of `threads` threads are resident per SM.  Thread-safe: the
// per-(kernel, device) results are kept under a mutex.
int32_t kernel_setup(const void* func, size_t smem, int threads, int* occ);

// 2-D row-major tensor map over `rows` rows of `row_elems` elements of
// `dtype`, box = (box_x elements, box_y rows), 128-byte swizzle.
int32_t encode_rows_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                         const void* base, uint64_t row_elems, uint64_t rows, uint32_t box_x,
                         uint32_t box_y, CUtensorMapSwizzle swizzle);

// General tiled tensor map: `rank` dims (innermost first), byte strides of
// dims 1..rank-1, box extents; element strides 1, zero fill out of range.
int32_t encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                    const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                    CUtensorMapSwizzle swizzle);

// Internal workspace for entry points called without one (and those whose
// reference signature carries none: gpu_attention_device and friends).  One
// buffer per device and kind: kWsCounters for the kernels that keep merge
// counters at the start of their workspace (they must read zero there; the
// kernels leave them at zero), kWsScratch for the others, whose partials
// would otherwise land on those counters.  `zero_prefix` = the counter bytes
// of this call: when more than the previous call's on that buffer, they are
// cleared on `stream` first.  Grown with cudaMalloc and zeroed with cudaMemset,
// so the first call at a given size must not be under capture.
enum WsKind { kWsScratch = 0, kWsCounters = 1, kWsKinds = 2 };
int32_t internal_workspace(size_t bytes, void** ptr, WsKind kind = kWsScratch, size_t zero_prefix = 0,
                           cudaStream_t stream = nullptr);

// Launch with programmatic dependent launch allowed: the grid may be scheduled
// while the previous grid in the stream runs; the kernel itself calls
// griddepcontrol.wait (pdl_wait) before it touches global memory that grid
// may write.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// Zoned decode of short contexts (decode_f32.cu): one launch for up to
// zoned_small_max() tokens, optionally adding the importance weights of
// ops::attention_tracked.  Arguments as nyion_attn_decode_zoned_f32, with the
// attended token count instead of seq_len / q_pos.
int64_t zoned_small_max();
int32_t zoned_small(float* out, const float* q, const float* k_arena, const float* v_arena, int64_t n_arena_pages,
                    int32_t n_layers, int32_t layer_idx, int64_t n_tokens, int32_t n_kv_heads, int32_t head_dim,
                    double* importance, void* stream);

// Whole-page fp32 paged decode for 4 KV heads (decode_pages.cu): workspace
// bytes for `batch` sequences, and the launch (workspace zeroed once, left
// with its counters at zero).
size_t pages_workspace_bytes(int batch);
int32_t launch_pages(const float* q, const float* kv_pool, int64_t n_pool_pages, const int32_t* page_table,
                     int32_t max_pages, const int32_t* seq_lens, float* out, int32_t batch, float qscale,
                     void* ws, cudaStream_t stream, int32_t* err_word = nullptr, int num_sms = 0);
// Leading bytes of the page kernel's workspace that hold its merge counters.
size_t pages_counter_bytes();

// Single-sequence decode over row caches (decode_contig.cu), head_dim 64 and
// GQA group 8: contiguous f32 / f16 caches [n_kv][stride][64] (f16 optionally
// with a device length clamped to `window`) and the zone-page arena.  `sl2` is
// scale * log2(e).  Workspace: contig_workspace_bytes(n_kv, max tokens), its
// leading counters zeroed once (null = the library's, zeroed on allocation).
size_t contig_workspace_bytes(int n_kv, int max_tokens);
int32_t contig_rows_f32(const float* q, const float* k, const float* v, float* out, int n_kv, int64_t stride, int n,
                        float sl2, void* ws, size_t ws_bytes, cudaStream_t stream);
int32_t contig_rows_f16(const float* q, const void* k, const void* v, float* out, int n_kv, int64_t stride, int n,
                        const int32_t* d_len, int window, float sl2, void* ws, size_t ws_bytes, cudaStream_t stream);
int32_t contig_zoned_f32(const float* q, const float* k_arena, const float* v_arena, float* out, int n_kv,
                         int n_layers, int layer, int64_t n_pages, int n, float sl2, void* ws, size_t ws_bytes,
                         cudaStream_t stream);

// Leading bytes of the 4-bit decode's workspace that hold its merge counters
// (decode_q4.cu): zero before the first call, left at zero by every call.
size_t q4_counter_bytes();

// Decode for the shapes the specialised kernels do not take (decode_generic.cu):
// head_dim 64 or 128, 1 to 8 query heads per KV head, any number of KV heads.
enum GenFormat : int32_t { kGenF32 = 0, kGenF16 = 1, kGenBF16 = 2, kGenQ4 = 3 };
enum GenLayout : int32_t { kGenPaged = 0, kGenRows = 1, kGenZoned = 2 };
struct GenericCall {
  const char* who = "decode";
  const void* q = nullptr;          // [rows][n_heads][head_dim] f32 (bf16 when q_bf16)
  int32_t q_bf16 = 0;
  const void* k = nullptr;          // paged: the pool; rows / zoned: K
  const void* v = nullptr;          // rows / zoned: V
  const int32_t* table = nullptr;   // paged: [rows][max_pages], or one row shared by all rows
  int32_t table_shared = 0, max_pages = 0;
  int64_t n_pool_pages = 0;
  int32_t n_heads = 0, n_kv = 0, head_dim = 0, rows = 0;
  // attended tokens of row b: [0, lens[b]); [tok_begin[b], tok_end[b]) or [u_begin, u_end);
  // causal_base >= 0: [0, causal_base + b + 1); d_len: [0, min(*d_len, window))
  const int32_t* lens = nullptr;
  const int32_t* tok_begin = nullptr;
  const int32_t* tok_end = nullptr;
  int32_t u_begin = 0, u_end = 0;
  int64_t causal_base = -1;
  const int32_t* d_len = nullptr;
  int32_t window = 0;
  int64_t stride = 0;               // rows layout: tokens per KV head
  int32_t n_layers = 0, layer = 0;  // zoned layout
  int64_t n_pages = 0;              // zoned: arena pages
  float scale = 0.f;                // <= 0: 1 / sqrt(head_dim)
  int32_t part_mode = 0;            // 0: out [rows][H][hd]; 1: [rows][H][hd + 2] (o / l, m natural, l)
  float* out = nullptr;
  int64_t max_tokens = 0;           // bound on any row's attended tokens (sizes the splits)
  int32_t fmt = kGenF32, layout = kGenPaged;
};
bool generic_shape_ok(int n_heads, int n_kv_heads, int head_dim);
// Uses the library-owned workspace (allocated on first use: not under stream capture).
int32_t generic_decode(const GenericCall& c, cudaStream_t stream);

// Handle behind gpu_graph_create_attention[_half]: the instantiated graph
// and the workspace it owns (freed by gpu_graph_destroy).
struct AttnGraph {
  cudaGraphExec_t exec;
  void* ws;
};

}  // namespace nyion
