// kv_write.cu — the KV write path: RoPE on the new token's q and k, then the
// rotated K and V saved into every cache format the attention kernels read,
// in one launch.
//
//   * RoPE of the CPU engine (swamp-engine/src/ops.rs:20-84): a table
//     [max_context][head_dim/2] of (cos, sin) with freq = 1 / 10000^(2k/hd),
//     angle = pos * freq (init_rope_lut), pairs (2k, 2k+1) rotated as
//     x' = x cos - y sin, y' = x sin + y cos with separate multiplies and
//     adds (apply_rotation_pair), position clamped to max_context - 1
//     (apply_rope_ufc).  The table is built on the host with the C library's
//     powf / cosf / sinf (the functions Rust's f32 methods call) and uploaded,
//     so a rotated vector is bit-identical to the CPU engine's;
//   * 4-bit save of PagedKVCache::save / save_at (cache.rs:613-679, 749-811):
//     per 32-value block d = max|x| / 7, dmin = min x, stored as f16 (RNE),
//     q = clamp(round((x - dmin) / d), 0, 15) with the unrounded d and dmin,
//     nibbles of a fresh slot (element i in byte i/2, low nibble for even i):
//     bit-exact;
//   * the fp32 copy save() keeps when the f32 page exists (cache.rs:671-677),
//     the bf16 pages of the chunked prefill kernel, the fp32 ring of the
//     windowed 4-bit decode, and the layer graph's f16 ring
//     (kernel_rope + kernel_kv_save, swamp-gpu/kernels/fused_attention.cu:
//     1438-1472, wpos = pos % window as gpu_graph_replay_layer sets it).
//
// One CTA per row (a decode token of one sequence, or one token of a prefill
// chunk).  Phase 1 rotates q (written back in place, plus an optional bf16
// copy) and k (in place, and into shared memory with v).  Phase 2: one warp
// per 32-value block quantizes (lane = element: max / min by shuffles,
// nibbles OR-ed across 8-lane groups, five 4-byte stores per block), and the
// CTA's threads write the f32 / bf16 / ring copies with coalesced stores.
// A row whose position has no page (outside the table, or an id outside the
// pool) raises the page-range bit of the device error word and writes no page.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>
#include <string.h>

#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace kvw {

constexpr int HD = 64;
constexpr int HALF = HD / 2;
constexpr int PAGE = 16;
constexpr int THREADS = 256;
constexpr int MAX_KV = 16;
constexpr int Q4ROW = 40;            // 2 blocks x 20 bytes

struct Params {
  float* q;                          // [rows][n_heads][64], rotated in place (nullable)
  float* k;                          // [rows][n_kv][64], rotated in place
  const float* v;                    // [rows][n_kv][64]
  const int32_t* positions;          // [rows] absolute positions
  const int32_t* row_seq;            // [rows] sequence of each row (nullable: row i -> sequence i)
  int32_t rows, n_heads, n_kv;
  const float2* rope;                // [max_context][32] (cos, sin) or null: no rotation
  int32_t max_context;
  const int32_t* table;              // [n_seq][max_pages]
  int32_t max_pages;
  int64_t n_pool_pages;
  uint8_t* pool_q4;                  // [pages][n_kv][2][16][40]
  float* pool_f32;                   // [pages][n_kv][2][16][64]
  __nv_bfloat16* pool_bf16;          // [pages][n_kv][2][16][64]
  __nv_bfloat16* q_bf16;             // [rows][n_heads][64]
  float* ring_f32;                   // [n_seq][n_kv][2][ring_tokens][64]
  int32_t ring_tokens;
  __half* ring16_k;                  // [n_kv][ring16][64] (single sequence)
  __half* ring16_v;
  int32_t ring16;
  const int32_t* d_seq_len;          // f16-ring mode: pos = *d_seq_len - 1
  const int32_t* d_wpos;             //               slot = *d_wpos, or pos % ring16
  int32_t* err;
};

__device__ __forceinline__ float2 rotate(float2 xy, float2 cs) {
  return make_float2(__fsub_rn(__fmul_rn(xy.x, cs.x), __fmul_rn(xy.y, cs.y)),
                     __fadd_rn(__fmul_rn(xy.x, cs.y), __fmul_rn(xy.y, cs.x)));
}

// One 32-value block by one warp (lane = element): 20 bytes at dst.
__device__ __forceinline__ void quantize_block_warp(float x, uint8_t* dst, int lane) {
  float mx = fabsf(x), mn = x;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
  }
  mx = fmaxf(mx, 0.0f);                          // the reference starts max|x| at 0
  const float d = mx > 1e-10f ? __fdiv_rn(mx, 7.0f) : 0.0f;
  uint32_t q = 0;
  if (d > 1e-10f) {
    const float r = fminf(fmaxf(roundf(__fdiv_rn(__fsub_rn(x, mn), d)), 0.0f), 15.0f);
    q = (uint32_t)r;
  }
  uint32_t w = q << ((lane & 7) * 4);
  w |= __shfl_xor_sync(0xffffffffu, w, 1);
  w |= __shfl_xor_sync(0xffffffffu, w, 2);
  w |= __shfl_xor_sync(0xffffffffu, w, 4);
  uint32_t* out = reinterpret_cast<uint32_t*>(dst);
  if (lane == 0) {
    out[0] = (uint32_t)__half_as_ushort(__float2half_rn(d)) |
             ((uint32_t)__half_as_ushort(__float2half_rn(mn)) << 16);
  }
  if ((lane & 7) == 0) out[1 + (lane >> 3)] = w;
}

template <bool RING16>
__global__ void __launch_bounds__(THREADS) kv_write_kernel(const Params p) {
  __shared__ float kv_s[2][MAX_KV][HD];
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int pos;
  if (RING16) pos = *p.d_seq_len - 1;
  else pos = p.positions[row];
  const int seq = p.row_seq ? p.row_seq[row] : row;
  const float2* cs = nullptr;
  if (p.rope) cs = p.rope + (int64_t)min(max(pos, 0), p.max_context - 1) * HALF;

  // phase 1: rotate q (in place, bf16 copy) and k; k and v to shared memory
  if (p.q) {
    float2* qr = reinterpret_cast<float2*>(p.q + (int64_t)row * p.n_heads * HD);
    for (int i = tid; i < p.n_heads * HALF; i += THREADS) {
      float2 xy = qr[i];
      if (cs) {
        xy = rotate(xy, __ldg(cs + (i & (HALF - 1))));
        qr[i] = xy;
      }
      if (p.q_bf16)
        reinterpret_cast<__nv_bfloat162*>(p.q_bf16 + (int64_t)row * p.n_heads * HD)[i] = __floats2bfloat162_rn(xy.x, xy.y);
    }
  }
  {
    float2* kr = reinterpret_cast<float2*>(p.k + (int64_t)row * p.n_kv * HD);
    const float2* vr = reinterpret_cast<const float2*>(p.v + (int64_t)row * p.n_kv * HD);
    for (int i = tid; i < p.n_kv * HALF; i += THREADS) {
      float2 xy = kr[i];
      if (cs) {
        xy = rotate(xy, __ldg(cs + (i & (HALF - 1))));
        kr[i] = xy;
      }
      reinterpret_cast<float2*>(&kv_s[0][0][0])[i] = xy;
      reinterpret_cast<float2*>(&kv_s[1][0][0])[i] = vr[i];
    }
  }
  __syncthreads();

  if (RING16) {
    // layer-graph f16 ring of one sequence: [n_kv][ring16][64] for K and V
    const int slot = p.d_wpos ? *p.d_wpos : (pos >= 0 ? pos % p.ring16 : -1);
    if (slot < 0 || slot >= p.ring16) {
      if (tid == 0) record_error(p.err, kErrPageRange);
      return;
    }
    for (int i = tid; i < p.n_kv * HD; i += THREADS) {
      const int h = i / HD, d = i % HD;
      const int64_t o = ((int64_t)h * p.ring16 + slot) * HD + d;
      p.ring16_k[o] = __float2half_rn(kv_s[0][h][d]);
      p.ring16_v[o] = __float2half_rn(kv_s[1][h][d]);
    }
    return;
  }

  if (p.ring_f32 && pos >= 0) {
    const int slot = pos % p.ring_tokens;
    for (int i = tid; i < 2 * p.n_kv * HD; i += THREADS) {
      const int kv = i / (p.n_kv * HD), h = (i / HD) % p.n_kv, d = i % HD;
      p.ring_f32[((((int64_t)seq * p.n_kv + h) * 2 + kv) * p.ring_tokens + slot) * HD + d] = kv_s[kv][h][d];
    }
  }
  if (!p.pool_q4 && !p.pool_f32 && !p.pool_bf16) return;
  int64_t page = -1;
  if (pos >= 0 && pos / PAGE < p.max_pages) page = p.table[(int64_t)seq * p.max_pages + pos / PAGE];
  if (page < 0 || page >= p.n_pool_pages) {
    if (tid == 0) record_error(p.err, kErrPageRange);
    return;
  }
  const int slot = pos % PAGE;
  if (p.pool_q4) {
    for (int b = warp; b < p.n_kv * 4; b += THREADS / 32) {     // (kv, head, block)
      const int kv = b / (p.n_kv * 2), h = (b / 2) % p.n_kv, blk = b & 1;
      uint8_t* dst = p.pool_q4 + (((page * p.n_kv + h) * 2 + kv) * PAGE + slot) * Q4ROW + blk * 20;
      quantize_block_warp(kv_s[kv][h][blk * 32 + lane], dst, lane);
    }
  }
  if (p.pool_f32 || p.pool_bf16) {
    for (int i = tid; i < 2 * p.n_kv * HD; i += THREADS) {
      const int kv = i / (p.n_kv * HD), h = (i / HD) % p.n_kv, d = i % HD;
      const int64_t o = (((page * p.n_kv + h) * 2 + kv) * PAGE + slot) * HD + d;
      if (p.pool_f32) p.pool_f32[o] = kv_s[kv][h][d];
      if (p.pool_bf16) p.pool_bf16[o] = __float2bfloat16_rn(kv_s[kv][h][d]);
    }
  }
}

// float -> half into [n_kv][max_seq_len][head_dim] at `pos` (the f16 cache of
// gpu_copy_kv_layer_async_half)
__global__ void to_half_strided_kernel(const float* __restrict__ src, __half* __restrict__ dst, int pos,
                                       int n_kv, int max_seq_len, int head_dim) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_kv * head_dim) return;
  const int h = i / head_dim, d = i % head_dim;
  dst[((int64_t)h * max_seq_len + pos) * head_dim + d] = __float2half_rn(src[i]);
}

int32_t check_common(const float* k, const float* v, int32_t n_heads, int32_t n_kv, int32_t head_dim,
                     const float* rope, int32_t max_context, const char* who) {
  if (!k || !v) return fail(NYION_ERR_INVALID, "%s: k and v are required", who);
  if (head_dim != HD) return fail(NYION_ERR_UNSUPPORTED, "%s: this build takes head_dim 64", who);
  if (n_kv <= 0 || n_kv > MAX_KV) return fail(NYION_ERR_UNSUPPORTED, "%s: n_kv_heads must be in [1, 16]", who);
  if (n_heads < 0) return fail(NYION_ERR_INVALID, "%s: n_heads < 0", who);
  if (rope && max_context <= 0) return fail(NYION_ERR_INVALID, "%s: max_context must be > 0", who);
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 7)
    return fail(NYION_ERR_INVALID, "%s: k and v must be 8-byte aligned", who);
  return NYION_OK;
}

// the f32 staging buffer of gpu_copy_kv_layer_async_half, per device
struct Staging {
  float* ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_stage_mu;
std::vector<Staging> g_stage;

}  // namespace kvw
}  // namespace nyion

using namespace nyion;
using namespace nyion::kvw;

extern "C" size_t nyion_attn_rope_table_bytes(int32_t head_dim, int32_t max_context) {
  if (head_dim <= 0 || max_context <= 0) return 0;
  return (size_t)max_context * (size_t)(head_dim / 2) * 2 * sizeof(float);
}

extern "C" int32_t nyion_attn_rope_table(float* table, int32_t head_dim, int32_t max_context, void* stream) {
  if (!table) return fail(NYION_ERR_INVALID, "rope_table: null table");
  if (head_dim <= 0 || (head_dim & 1) || max_context <= 0)
    return fail(NYION_ERR_INVALID, "rope_table: head_dim must be even and > 0, max_context > 0");
  const int half = head_dim / 2;
  std::vector<float> freq(half);
  for (int k = 0; k < half; ++k) freq[k] = 1.0f / powf(10000.0f, (float)(2 * k) / (float)head_dim);
  std::vector<float> host((size_t)max_context * half * 2);
  unsigned nt = std::thread::hardware_concurrency();
  nt = nt == 0 ? 1 : (nt > 16 ? 16 : nt);
  if ((size_t)max_context < 4096) nt = 1;
  std::vector<std::thread> pool;
  for (unsigned t = 0; t < nt; ++t) {
    pool.emplace_back([&, t]() {
      const int64_t m0 = (int64_t)max_context * t / nt, m1 = (int64_t)max_context * (t + 1) / nt;
      for (int64_t m = m0; m < m1; ++m) {
        for (int k = 0; k < half; ++k) {
          const float angle = (float)m * freq[k];
          host[((size_t)m * half + k) * 2] = cosf(angle);
          host[((size_t)m * half + k) * 2 + 1] = sinf(angle);
        }
      }
    });
  }
  for (auto& th : pool) th.join();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t st = check_cuda(cudaMemcpyAsync(table, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice, s),
                          "rope_table upload");
  if (st) return st;
  return check_cuda(cudaStreamSynchronize(s), "rope_table upload");
}

extern "C" int32_t nyion_attn_kv_write_paged(float* q, float* k, const float* v, const int32_t* positions,
                                             const int32_t* row_seq, int32_t rows, int32_t n_heads,
                                             int32_t n_kv_heads, int32_t head_dim, const float* rope_table,
                                             int32_t max_context, const int32_t* page_table, int32_t max_pages,
                                             int64_t n_pool_pages, uint8_t* pool_q4, float* pool_f32,
                                             void* pool_bf16, void* q_bf16, float* ring_f32, int32_t ring_tokens,
                                             void* stream) {
  if (rows <= 0) return rows == 0 ? NYION_OK : fail(NYION_ERR_INVALID, "kv_write_paged: rows < 0");
  int32_t st = check_common(k, v, n_heads, n_kv_heads, head_dim, rope_table, max_context, "kv_write_paged");
  if (st) return st;
  if (!positions) return fail(NYION_ERR_INVALID, "kv_write_paged: positions required");
  if ((pool_q4 || pool_f32 || pool_bf16) && (!page_table || max_pages <= 0 || n_pool_pages <= 0))
    return fail(NYION_ERR_INVALID, "kv_write_paged: a page pool needs page_table, max_pages, n_pool_pages");
  if (ring_f32 && ring_tokens <= 0) return fail(NYION_ERR_INVALID, "kv_write_paged: ring_tokens must be > 0");
  if (q_bf16 && !q) return fail(NYION_ERR_INVALID, "kv_write_paged: q_bf16 needs q");
  if (q && (reinterpret_cast<uintptr_t>(q) & 7)) return fail(NYION_ERR_INVALID, "kv_write_paged: q must be 8-byte aligned");
  if ((reinterpret_cast<uintptr_t>(pool_q4) & 3) || (reinterpret_cast<uintptr_t>(q_bf16) & 3))
    return fail(NYION_ERR_INVALID, "kv_write_paged: pool_q4 and q_bf16 must be 4-byte aligned");
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st) return st;
  Params p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.positions = positions;
  p.row_seq = row_seq;
  p.rows = rows;
  p.n_heads = q ? n_heads : 0;
  p.n_kv = n_kv_heads;
  p.rope = reinterpret_cast<const float2*>(rope_table);
  p.max_context = max_context;
  p.table = page_table;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.pool_q4 = pool_q4;
  p.pool_f32 = pool_f32;
  p.pool_bf16 = static_cast<__nv_bfloat16*>(pool_bf16);
  p.q_bf16 = static_cast<__nv_bfloat16*>(q_bf16);
  p.ring_f32 = ring_f32;
  p.ring_tokens = ring_tokens;
  p.err = dev->err_word;
  kv_write_kernel<false><<<rows, THREADS, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError(), "kv_write_paged launch");
}

extern "C" int32_t nyion_attn_kv_write_ring_f16(float* q, float* k, const float* v, const int32_t* d_seq_len,
                                                const int32_t* d_wpos, void* k_ring, void* v_ring,
                                                int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                                int32_t window, const float* rope_table, int32_t max_context,
                                                void* stream) {
  int32_t st = check_common(k, v, n_heads, n_kv_heads, head_dim, rope_table, max_context, "kv_write_ring_f16");
  if (st) return st;
  if (!d_seq_len || !k_ring || !v_ring || window <= 0)
    return fail(NYION_ERR_INVALID, "kv_write_ring_f16: d_seq_len, k_ring, v_ring and window > 0 required");
  if (q && (reinterpret_cast<uintptr_t>(q) & 7)) return fail(NYION_ERR_INVALID, "kv_write_ring_f16: q must be 8-byte aligned");
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st) return st;
  Params p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.rows = 1;
  p.n_heads = q ? n_heads : 0;
  p.n_kv = n_kv_heads;
  p.rope = reinterpret_cast<const float2*>(rope_table);
  p.max_context = max_context;
  p.ring16_k = static_cast<__half*>(k_ring);
  p.ring16_v = static_cast<__half*>(v_ring);
  p.ring16 = window;
  p.d_seq_len = d_seq_len;
  p.d_wpos = d_wpos;
  p.err = dev->err_word;
  kv_write_kernel<true><<<1, THREADS, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_cuda(cudaGetLastError(), "kv_write_ring_f16 launch");
}

// ---- reference C ABI: contiguous KV buffers (fused_attention.cu:244-312,
// 456-481, 744-812), same names, arguments and 0 / -1 results ---------------

extern "C" void* gpu_alloc_kv_buffer(int n_kv_heads, int max_seq_len, int head_dim, size_t* out_bytes) {
  const size_t bytes = (size_t)n_kv_heads * max_seq_len * head_dim * sizeof(float);
  void* ptr = nullptr;
  if (n_kv_heads <= 0 || max_seq_len <= 0 || head_dim <= 0 ||
      check_cuda(cudaMalloc(&ptr, bytes), "gpu_alloc_kv_buffer")) {
    if (out_bytes) *out_bytes = 0;
    return nullptr;
  }
  if (out_bytes) *out_bytes = bytes;
  return ptr;
}

extern "C" void* gpu_alloc_kv_buffer_half(int n_kv_heads, int max_seq_len, int head_dim, size_t* out_bytes) {
  const size_t bytes = (size_t)n_kv_heads * max_seq_len * head_dim * sizeof(__half);
  void* ptr = nullptr;
  if (n_kv_heads <= 0 || max_seq_len <= 0 || head_dim <= 0 ||
      check_cuda(cudaMalloc(&ptr, bytes), "gpu_alloc_kv_buffer_half")) {
    if (out_bytes) *out_bytes = 0;
    return nullptr;
  }
  if (out_bytes) *out_bytes = bytes;
  return ptr;
}

extern "C" int gpu_copy_kv_to_buffer(float* d_buf, const float* h_src, int kv_head, int pos, int n_kv_heads,
                                     int max_seq_len, int head_dim) {
  if (!d_buf || !h_src || kv_head < 0 || kv_head >= n_kv_heads || pos < 0 || pos >= max_seq_len) {
    fail(NYION_ERR_INVALID, "gpu_copy_kv_to_buffer: bad argument");
    return -1;
  }
  const size_t off = ((size_t)kv_head * max_seq_len + pos) * head_dim;
  return check_cuda(cudaMemcpy(d_buf + off, h_src, (size_t)head_dim * sizeof(float), cudaMemcpyHostToDevice),
                    "gpu_copy_kv_to_buffer")
             ? -1
             : 0;
}

// All KV heads of one position in one strided copy (the reference issues one
// copy per head).
static int copy_layer(float* d_buf, const float* h_src, int pos, int n_kv_heads, int max_seq_len, int head_dim,
                      cudaStream_t stream, bool async, const char* who) {
  if (!d_buf || !h_src || n_kv_heads <= 0 || head_dim <= 0 || pos < 0 || pos >= max_seq_len) {
    fail(NYION_ERR_INVALID, "%s: bad argument", who);
    return -1;
  }
  const size_t row = (size_t)head_dim * sizeof(float);
  cudaError_t e = cudaMemcpy2DAsync(d_buf + (size_t)pos * head_dim, (size_t)max_seq_len * row, h_src, row, row,
                                    (size_t)n_kv_heads, cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess && !async) e = cudaStreamSynchronize(stream);
  return check_cuda(e, who) ? -1 : 0;
}

extern "C" int gpu_copy_kv_layer(float* d_buf, const float* h_src, int pos, int n_kv_heads, int max_seq_len,
                                 int head_dim) {
  return copy_layer(d_buf, h_src, pos, n_kv_heads, max_seq_len, head_dim, nullptr, false, "gpu_copy_kv_layer");
}

extern "C" int gpu_copy_kv_layer_async(float* d_buf, const float* h_src, int pos, int n_kv_heads, int max_seq_len,
                                       int head_dim, void* stream) {
  return copy_layer(d_buf, h_src, pos, n_kv_heads, max_seq_len, head_dim, static_cast<cudaStream_t>(stream), true,
                    "gpu_copy_kv_layer_async");
}

extern "C" int gpu_copy_kv_layer_async_half(void* d_buf, const float* h_src, int pos, int n_kv_heads,
                                            int max_seq_len, int head_dim, void* stream) {
  if (!d_buf || !h_src || n_kv_heads <= 0 || head_dim <= 0 || pos < 0 || pos >= max_seq_len) {
    fail(NYION_ERR_INVALID, "gpu_copy_kv_layer_async_half: bad argument");
    return -1;
  }
  int dev = -1;
  if (check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return -1;
  const size_t bytes = (size_t)n_kv_heads * head_dim * sizeof(float);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* stage = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_stage_mu);
    if ((int)g_stage.size() <= dev) g_stage.resize(dev + 1);
    Staging& sg = g_stage[dev];
    if (sg.bytes < bytes) {
      if (sg.ptr) {
        cudaDeviceSynchronize();
        cudaFree(sg.ptr);
        sg.ptr = nullptr;
        sg.bytes = 0;
      }
      if (check_cuda(cudaMalloc(&sg.ptr, bytes), "gpu_copy_kv_layer_async_half staging")) return -1;
      sg.bytes = bytes;
    }
    stage = sg.ptr;
  }
  if (check_cuda(cudaMemcpyAsync(stage, h_src, bytes, cudaMemcpyHostToDevice, s), "gpu_copy_kv_layer_async_half"))
    return -1;
  const int n = n_kv_heads * head_dim;
  to_half_strided_kernel<<<(n + 255) / 256, 256, 0, s>>>(stage, static_cast<__half*>(d_buf), pos, n_kv_heads,
                                                         max_seq_len, head_dim);
  return check_cuda(cudaGetLastError(), "gpu_copy_kv_layer_async_half launch") ? -1 : 0;
}
