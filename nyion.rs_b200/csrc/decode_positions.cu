// decode_positions.cu — decode attention over an explicit list of token
// positions of the 16-token paged pools (fp32 or 4-bit), and the reference's
// window + global sparse attention built on it.
//
//   * ops::attention_sparse / attention_fugu (swamp-engine/src/ops.rs:85-168,
//     445-541): fp32 attention over a position set (window, every stride-th
//     older token, DSPark picks) — nyion_attn_decode_positions, kv format 0;
//   * ops::attention_sparse_q4 (ops.rs:597-723): the same over 4-bit pages,
//     positions = stride * gi for gi < min(window_start / stride, 128), then
//     the window [window_start, valid_end] — nyion_attn_sparse_q4: the window
//     is a token range of the Q4 page kernel (decode_q4.cu), the global
//     positions go through this kernel, and the two log-sum-exp partials are
//     merged.  Nibbles are read in the writer's order (element i in byte i/2,
//     low nibble for even i, cache.rs:637-663).
//
// Scattered positions cannot use page-granular copies, so this kernel reads
// rows directly: CTA = (sequence, KV head, 256-position split), warp = one
// query head of the GQA group; a lane takes one position of a 32-position
// chunk for the score (its K row from global memory, fp32 dot with the
// pre-scaled query in registers), then the warp walks the chunk for P.V
// (lane = two output dims, p broadcast by shuffle); online softmax in the
// log2 domain; one (o/l, m, l) partial per split, merged by
// nyion_attn_lse_combine.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "host.h"

extern "C" int32_t nyion_attn_lse_combine(const float* parts, int32_t n_parts, int64_t rows,
                                          int32_t head_dim, float* out, void* stream);
extern "C" int32_t nyion_attn_decode_q4_partial(const float* q, const uint8_t* kv_pool, int64_t n_pool_pages,
                                                const int32_t* page_table, int32_t max_pages,
                                                const int32_t* tok_begin, const int32_t* tok_end,
                                                int32_t u_begin, int32_t u_end, float* part, int32_t batch,
                                                int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                                int32_t page_tokens, float scale, void* workspace,
                                                size_t workspace_bytes, void* stream);
extern "C" size_t nyion_attn_q4_workspace_size(int32_t batch);

namespace nyion {
namespace posd {

constexpr int HD = 64;
constexpr int GROUP = 8;
constexpr int PAGE = 16;
constexpr int SPLIT = 256;
constexpr int THREADS = 32 * GROUP;
constexpr int PART = HD + 2;
constexpr int MAX_GLOBAL = 128;        // attention_sparse*: at most 128 global tokens

struct Params {
  const float* q;                // [batch][H][64]
  const void* pool;              // f32 [pages][n_kv][2][16][64] or q4 [pages][n_kv][2][16][40]
  const int32_t* table;          // [batch][max_pages]
  const int32_t* positions;      // [batch][max_positions] (explicit mode)
  const int32_t* n_positions;    // [batch] (explicit mode)
  const int32_t* seq_lens;       // [batch] (rule mode)
  int32_t max_positions;
  int32_t window, stride;        // rule mode: stride * gi, gi < min(window_start / stride, 128)
  int32_t batch, n_kv, max_pages;
  int64_t n_pool_pages;
  float sl2;                     // scale * log2(e)
  float* part;                   // [n_split][batch * H][66]
  int32_t* err;
};

// number of positions of sequence b and position j
template <bool RULE>
__device__ __forceinline__ int count_of(const Params& p, int b) {
  if (!RULE) return max(0, min(p.n_positions[b], p.max_positions));
  const int len = p.seq_lens[b];
  if (len <= 0) return 0;
  const int valid_end = len - 1;
  const int ws = valid_end > p.window ? valid_end - p.window + 1 : 0;
  return min(ws / p.stride, MAX_GLOBAL);
}
template <bool RULE>
__device__ __forceinline__ int position_of(const Params& p, int b, int j) {
  return RULE ? p.stride * j : p.positions[(int64_t)b * p.max_positions + j];
}

template <bool Q4>
__device__ __forceinline__ void load_row(const Params& p, int64_t page, int kvh, int kv, int slot, float (&x)[HD]) {
  if (!Q4) {
    const float4* r = reinterpret_cast<const float4*>(static_cast<const float*>(p.pool) +
                                                      (((page * p.n_kv + kvh) * 2 + kv) * PAGE + slot) * HD);
#pragma unroll
    for (int c = 0; c < HD / 4; ++c) {
      const float4 v = __ldg(r + c);
      x[4 * c] = v.x; x[4 * c + 1] = v.y; x[4 * c + 2] = v.z; x[4 * c + 3] = v.w;
    }
  } else {
    const uint2* r = reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(p.pool) +
                                                    (((page * p.n_kv + kvh) * 2 + kv) * PAGE + slot) * 40);
    uint32_t w[10];
#pragma unroll
    for (int c = 0; c < 5; ++c) {
      const uint2 v = __ldg(r + c);
      w[2 * c] = v.x;
      w[2 * c + 1] = v.y;
    }
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      // block blk occupies bytes [20 blk, 20 blk + 20): words 5 blk .. 5 blk + 4
      const uint32_t hdr = w[5 * blk];
      const float d = __half2float(__ushort_as_half((unsigned short)(hdr & 0xFFFF)));
      const float dm = __half2float(__ushort_as_half((unsigned short)(hdr >> 16)));
#pragma unroll
      for (int wq = 0; wq < 4; ++wq) {
        const uint32_t nib = w[5 * blk + 1 + wq];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int i = 8 * wq + e;                         // element: byte i/2, low nibble for even i
          const uint32_t n = (nib >> (8 * (e >> 1) + 4 * (e & 1))) & 0xF;
          x[32 * blk + i] = __fadd_rn(__fmul_rn(d, (float)n), dm);
        }
      }
    }
  }
}

template <bool Q4>
__device__ __forceinline__ float2 load_pair(const Params& p, int64_t page, int kvh, int slot, int lane) {
  if (!Q4) {
    return __ldg(reinterpret_cast<const float2*>(static_cast<const float*>(p.pool) +
                                                 (((page * p.n_kv + kvh) * 2 + 1) * PAGE + slot) * HD) + lane);
  }
  const uint8_t* r = static_cast<const uint8_t*>(p.pool) + (((page * p.n_kv + kvh) * 2 + 1) * PAGE + slot) * 40;
  const int blk = lane >> 4, byte = lane & 15;              // dims 2 lane, 2 lane + 1
  const uint32_t hdr = __ldg(reinterpret_cast<const uint32_t*>(r + 20 * blk));
  const float d = __half2float(__ushort_as_half((unsigned short)(hdr & 0xFFFF)));
  const float dm = __half2float(__ushort_as_half((unsigned short)(hdr >> 16)));
  const uint32_t b = __ldg(r + 20 * blk + 4 + byte);
  return make_float2(__fadd_rn(__fmul_rn(d, (float)(b & 0xF)), dm), __fadd_rn(__fmul_rn(d, (float)(b >> 4)), dm));
}

template <bool Q4, bool RULE>
__global__ void __launch_bounds__(THREADS) positions_kernel(const Params p) {
  const int b = blockIdx.x / p.n_kv, kvh = blockIdx.x % p.n_kv, split = blockIdx.y;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.n_kv * GROUP, h = kvh * GROUP + w;
  const int n = count_of<RULE>(p, b);
  const int j0 = split * SPLIT, j1 = min(j0 + SPLIT, n);
  float* dst = p.part + ((int64_t)split * p.batch * H + (int64_t)b * H + h) * PART;
  if (j0 >= j1) {
    dst[2 * lane] = 0.f;
    dst[2 * lane + 1] = 0.f;
    if (lane == 0) {
      dst[HD] = -INFINITY;
      dst[HD + 1] = 0.f;
    }
    return;
  }
  float qr[HD];
#pragma unroll
  for (int d = 0; d < HD; d += 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p.q + ((int64_t)b * H + h) * HD + d));
    qr[d] = v.x * p.sl2; qr[d + 1] = v.y * p.sl2; qr[d + 2] = v.z * p.sl2; qr[d + 3] = v.w * p.sl2;
  }
  float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
  for (int c0 = j0; c0 < j1; c0 += 32) {
    const int j = c0 + lane;
    int64_t page = -1;
    int slot = 0;
    if (j < j1) {
      const int pos = position_of<RULE>(p, b, j);
      const int pidx = pos / PAGE;
      if (pos >= 0 && pidx < p.max_pages) page = p.table[(int64_t)b * p.max_pages + pidx];
      if (page < 0 || page >= p.n_pool_pages) {
        record_error(p.err, kErrPageRange);
        page = -1;
      }
      slot = pos % PAGE;
    }
    float s = -INFINITY;
    if (page >= 0) {
      float kr[HD];
      load_row<Q4>(p, page, kvh, 0, slot, kr);
      float a = 0.f;
#pragma unroll
      for (int d = 0; d < HD; ++d) a = fmaf(qr[d], kr[d], a);
      s = a;
    }
    const float cmx = warp_max(s);
    if (cmx == -INFINITY) continue;                  // no valid position in this chunk
    const float mn = fmaxf(m, cmx);
    const float alpha = exp2f(m - mn);
    const float pt = page >= 0 ? exp2f(s - mn) : 0.f;
    l = fmaf(l, alpha, warp_sum(pt));
    o0 *= alpha;
    o1 *= alpha;
    const int cnt = min(32, j1 - c0);
    for (int jj = 0; jj < cnt; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, pt, jj);
      const int64_t pg = __shfl_sync(0xffffffffu, page, jj);
      const int sl = __shfl_sync(0xffffffffu, slot, jj);
      if (pg < 0) continue;                          // warp-uniform
      const float2 v = load_pair<Q4>(p, pg, kvh, sl, lane);
      o0 = fmaf(pj, v.x, o0);
      o1 = fmaf(pj, v.y, o1);
    }
    m = mn;
  }
  const float inv = l > 0.f ? 1.0f / l : 0.f;
  dst[2 * lane] = o0 * inv;
  dst[2 * lane + 1] = o1 * inv;
  if (lane == 0) {
    dst[HD] = l > 0.f ? m * 0.69314718055994531f : -INFINITY;
    dst[HD + 1] = l;
  }
}

__global__ void window_ranges_kernel(const int32_t* __restrict__ seq_lens, int batch, int window,
                                     int32_t* __restrict__ tb, int32_t* __restrict__ te) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int len = seq_lens[b];
  if (len <= 0) {
    tb[b] = 0;
    te[b] = 0;
    return;
  }
  const int valid_end = len - 1;
  tb[b] = valid_end > window ? valid_end - window + 1 : 0;
  te[b] = valid_end + 1;
}

size_t part_bytes(int n_sets, int batch, int H) { return (size_t)n_sets * batch * H * PART * sizeof(float); }

int32_t check(const void* q, const void* pool, const int32_t* table, const float* out, int32_t batch,
              int32_t n_heads, int32_t n_kv, int32_t hd, int32_t page_tokens, const char* who) {
  if (!q || !pool || !table || !out) return fail(NYION_ERR_INVALID, "%s: null pointer argument", who);
  if (hd != HD || n_kv <= 0 || n_heads != n_kv * GROUP)
    return fail(NYION_ERR_UNSUPPORTED, "%s: this build takes head_dim 64 and GQA group 8", who);
  if (page_tokens != PAGE) return fail(NYION_ERR_UNSUPPORTED, "%s: page_tokens must be 16", who);
  if (batch <= 0) return fail(NYION_ERR_INVALID, "%s: batch must be > 0", who);
  if ((reinterpret_cast<uintptr_t>(pool) | reinterpret_cast<uintptr_t>(q)) & 15)
    return fail(NYION_ERR_INVALID, "%s: q and the pool must be 16-byte aligned", who);
  return NYION_OK;
}

}  // namespace posd
}  // namespace nyion

using namespace nyion;
using namespace nyion::posd;

extern "C" size_t nyion_attn_positions_workspace_size(int32_t batch, int32_t n_heads, int32_t max_positions) {
  const int ns = max_positions <= 0 ? 1 : (max_positions + SPLIT - 1) / SPLIT;
  return part_bytes(ns, batch, n_heads);
}

extern "C" int32_t nyion_attn_decode_positions(const float* q, const void* kv_pool, int32_t kv_format,
                                               int64_t n_pool_pages, const int32_t* page_table, int32_t max_pages,
                                               const int32_t* positions, const int32_t* n_positions,
                                               int32_t max_positions, float* out, int32_t batch, int32_t n_heads,
                                               int32_t n_kv_heads, int32_t head_dim, int32_t page_tokens,
                                               float scale, void* workspace, size_t workspace_bytes,
                                               void* stream) {
  int32_t st = check(q, kv_pool, page_table, out, batch, n_heads, n_kv_heads, head_dim, page_tokens,
                     "decode_positions");
  if (st) return st;
  if (!positions || !n_positions || max_positions <= 0)
    return fail(NYION_ERR_INVALID, "decode_positions: positions, n_positions and max_positions > 0 required");
  if (kv_format != 0 && kv_format != 1) return fail(NYION_ERR_INVALID, "decode_positions: kv_format 0 (f32) or 1 (q4)");
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st) return st;
  const int ns = (max_positions + SPLIT - 1) / SPLIT;
  const size_t need = part_bytes(ns, batch, n_heads);
  if (!workspace) {
    st = internal_workspace(need, &workspace);
    if (st) return st;
  } else if (workspace_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "decode_positions: workspace %zu < %zu", workspace_bytes, need);
  }
  Params p{};
  p.q = q;
  p.pool = kv_pool;
  p.table = page_table;
  p.positions = positions;
  p.n_positions = n_positions;
  p.max_positions = max_positions;
  p.batch = batch;
  p.n_kv = n_kv_heads;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.sl2 = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  p.part = static_cast<float*>(workspace);
  p.err = dev->err_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(batch * n_kv_heads), (unsigned)ns);
  if (kv_format == 0) positions_kernel<false, false><<<grid, THREADS, 0, s>>>(p);
  else positions_kernel<true, false><<<grid, THREADS, 0, s>>>(p);
  st = check_cuda(cudaGetLastError(), "decode_positions launch");
  if (st) return st;
  return nyion_attn_lse_combine(p.part, ns, (int64_t)batch * n_heads, HD, out, stream);
}

extern "C" size_t nyion_attn_sparse_q4_workspace_size(int32_t batch, int32_t n_heads) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  return al(nyion_attn_q4_workspace_size(batch)) + al(part_bytes(2, batch, n_heads)) +
         (size_t)2 * batch * sizeof(int32_t);
}

extern "C" int32_t nyion_attn_sparse_q4(const float* q, const uint8_t* kv_pool, int64_t n_pool_pages,
                                        const int32_t* page_table, int32_t max_pages, const int32_t* seq_lens,
                                        int32_t window, int32_t global_stride, float* out, int32_t batch,
                                        int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t page_tokens,
                                        float scale, void* workspace, size_t workspace_bytes, void* stream) {
  int32_t st = check(q, kv_pool, page_table, out, batch, n_heads, n_kv_heads, head_dim, page_tokens, "sparse_q4");
  if (st) return st;
  if (!seq_lens || window <= 0 || global_stride <= 0)
    return fail(NYION_ERR_INVALID, "sparse_q4: seq_lens, window > 0 and global_stride > 0 required");
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st) return st;
  const size_t need = nyion_attn_sparse_q4_workspace_size(batch, n_heads);
  if (!workspace) {
    st = internal_workspace(need, &workspace);
    if (st) return st;
  } else if (workspace_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "sparse_q4: workspace %zu < %zu", workspace_bytes, need);
  }
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  // [Q4 kernel workspace (its counters first, as every entry that shares the
  // library-owned buffer keeps them)][2 partial arrays: window, global][ranges]
  uint8_t* w = static_cast<uint8_t*>(workspace);
  void* q4ws = w;
  float* parts = reinterpret_cast<float*>(w + al(nyion_attn_q4_workspace_size(batch)));
  int32_t* tb = reinterpret_cast<int32_t*>(w + al(nyion_attn_q4_workspace_size(batch)) +
                                           al(part_bytes(2, batch, n_heads)));
  int32_t* te = tb + batch;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  window_ranges_kernel<<<(batch + 127) / 128, 128, 0, s>>>(seq_lens, batch, window, tb, te);
  st = check_cuda(cudaGetLastError(), "sparse_q4 ranges");
  if (st) return st;
  // window [window_start, valid_end] on the Q4 page kernel
  st = nyion_attn_decode_q4_partial(q, kv_pool, n_pool_pages, page_table, max_pages, tb, te, 0, 0, parts, batch,
                                    n_heads, n_kv_heads, head_dim, page_tokens, scale, q4ws,
                                    nyion_attn_q4_workspace_size(batch), stream);
  if (st) return st;
  // global tokens stride * gi
  Params p{};
  p.q = q;
  p.pool = kv_pool;
  p.table = page_table;
  p.seq_lens = seq_lens;
  p.window = window;
  p.stride = global_stride;
  p.batch = batch;
  p.n_kv = n_kv_heads;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.sl2 = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  p.part = parts + (size_t)batch * n_heads * PART;
  p.err = dev->err_word;
  positions_kernel<true, true><<<dim3((unsigned)(batch * n_kv_heads), 1), THREADS, 0, s>>>(p);
  st = check_cuda(cudaGetLastError(), "sparse_q4 global launch");
  if (st) return st;
  return nyion_attn_lse_combine(parts, 2, (int64_t)batch * n_heads, HD, out, stream);
}
