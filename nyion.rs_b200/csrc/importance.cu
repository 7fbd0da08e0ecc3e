// importance.cu — the importance output of ops::attention_tracked
// (swamp-engine/src/ops.rs:283-401): for every position t of the sequence,
// importance[t] += sum over query heads h of p_h(t), p = softmax of the scaled
// scores over [0, valid_end] (0 at masked positions), accumulated in double
// on top of the caller's values, as the reference does under its Mutex.
// The attention output itself comes from the zoned decode kernel
// (decode_f32.cu); this file adds the per-position weights.
//
// The executor takes this path for short sequences (the Full strategy, up to
// 512 tokens): there the short-context zoned kernel (decode_f32.cu) computes
// output and weights in one launch.  Longer contexts take two small launches
// after the zoned decode:
//   scores_kernel     grid (KV head, 256-position chunk), warp = query head of
//                     the group, lane = position: s = q.K_t * scale * log2(e)
//                     (fp32), stored [H][T], plus the chunk's (max, sum 2^(s-max))
//                     per head;
//   importance_kernel grid over 256-position chunks: each CTA merges the chunk
//                     partials of every head into (M_h, L_h) in shared memory,
//                     then thread = position: importance[t] += sum_h
//                     2^(s_h,t - M_h) / L_h.
// K rows are read from the reference zone-page arena (cache.rs:185-237,
// 681-747): zone z of pages with 32 / 128 / 1024 slots, each page
// [layer][kv head][slot][head_dim], pages consecutive.
#include <math.h>

#include "common.cuh"
#include "host.h"

extern "C" int32_t nyion_attn_decode_zoned_f32(float* out, const float* q, const float* k_arena,
                                               const float* v_arena, int64_t n_arena_pages,
                                               int32_t n_layers, int32_t layer_idx,
                                               int64_t seq_len, int64_t q_pos, int32_t n_heads,
                                               int32_t n_kv_heads, int32_t head_dim, void* stream);

namespace nyion {
namespace imp {

constexpr int HD = 64;
constexpr int GROUP = 8;
constexpr int CHUNK = 256;
constexpr int THREADS = 256;
constexpr int MAX_HEADS = 128;

struct Params {
  const float* q;          // [H][64]
  const float* k_arena;
  int64_t n_arena_pages;
  int32_t n_layers, layer, n_kv;
  int32_t n_valid;         // valid_end + 1 positions attended
  int32_t n_chunks;
  float sl2;               // scale * log2(e)
  float* scores;           // [H][n_valid] log2-domain scaled scores
  float2* part;            // [H][n_chunks] (max, sum 2^(s - max))
  double* importance;      // [seq_len]
  int32_t* err;
};

// row of position t, KV head kvh in the zone arena, or -1 when its page is absent
__device__ __forceinline__ int64_t zoned_row(const Params& p, int64_t t, int kvh) {
  const int zone = t < 4096 ? 0 : (t < 131072 ? 1 : 2);
  const int64_t bs = zone == 0 ? 32 : (zone == 1 ? 128 : 1024);
  const int64_t zs = zone == 0 ? 0 : (zone == 1 ? 4096 : 131072);
  const int64_t zpage = zone == 0 ? 0 : (zone == 1 ? 128 : 1120);
  const int64_t lp = (int64_t)p.n_layers * p.n_kv;
  const int64_t zrow = zone == 0 ? 0 : (zone == 1 ? 128 * lp * 32 : 128 * lp * 32 + 992 * lp * 128);
  const int64_t local = (t - zs) / bs, slot = (t - zs) % bs;
  if (zpage + local >= p.n_arena_pages) return -1;
  return zrow + local * lp * bs + ((int64_t)p.layer * p.n_kv + kvh) * bs + slot;
}

__global__ void __launch_bounds__(THREADS) scores_kernel(const Params p) {
  const int kvh = blockIdx.x, chunk = blockIdx.y;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = kvh * GROUP + w;
  float qr[HD];
#pragma unroll
  for (int d = 0; d < HD; d += 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p.q + (int64_t)h * HD + d));
    qr[d] = v.x * p.sl2; qr[d + 1] = v.y * p.sl2; qr[d + 2] = v.z * p.sl2; qr[d + 3] = v.w * p.sl2;
  }
  float m = -INFINITY, l = 0.f;
  for (int j = 0; j < CHUNK / 32; ++j) {
    const int t = chunk * CHUNK + j * 32 + lane;
    if (t >= p.n_valid) break;
    float s = -INFINITY;
    const int64_t row = zoned_row(p, t, kvh);
    if (row >= 0) {
      const float4* kr = reinterpret_cast<const float4*>(p.k_arena + row * HD);
      float a = 0.f;
#pragma unroll
      for (int c = 0; c < HD / 4; ++c) {
        const float4 k = __ldg(kr + c);
        a = fmaf(qr[4 * c], k.x, a);
        a = fmaf(qr[4 * c + 1], k.y, a);
        a = fmaf(qr[4 * c + 2], k.z, a);
        a = fmaf(qr[4 * c + 3], k.w, a);
      }
      s = a;
    } else {
      record_error(p.err, kErrPageRange);
    }
    p.scores[(int64_t)h * p.n_valid + t] = s;
    if (s > -INFINITY) {
      const float mn = fmaxf(m, s);
      l = l * exp2f(m - mn) + exp2f(s - mn);
      m = mn;
    }
  }
  // warp merge of the lanes' (m, l)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float mo = __shfl_xor_sync(0xffffffffu, m, o);
    const float lo = __shfl_xor_sync(0xffffffffu, l, o);
    const float mn = fmaxf(m, mo);
    if (mn > -INFINITY) {
      l = (m > -INFINITY ? l * exp2f(m - mn) : 0.f) + (mo > -INFINITY ? lo * exp2f(mo - mn) : 0.f);
      m = mn;
    }
  }
  if (lane == 0) p.part[(int64_t)h * p.n_chunks + chunk] = make_float2(m, l);
}

__global__ void __launch_bounds__(THREADS) importance_kernel(const Params p, int32_t n_heads) {
  __shared__ float sm[MAX_HEADS], sinv[MAX_HEADS];
  // merge every head's chunk partials (one warp per head, round-robin)
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int h = w; h < n_heads; h += THREADS / 32) {
    float m = -INFINITY, l = 0.f;
    for (int c = lane; c < p.n_chunks; c += 32) {
      const float2 pr = p.part[(int64_t)h * p.n_chunks + c];
      const float mn = fmaxf(m, pr.x);
      if (mn > -INFINITY) {
        l = (m > -INFINITY ? l * exp2f(m - mn) : 0.f) + (pr.x > -INFINITY ? pr.y * exp2f(pr.x - mn) : 0.f);
        m = mn;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m, o);
      const float lo = __shfl_xor_sync(0xffffffffu, l, o);
      const float mn = fmaxf(m, mo);
      if (mn > -INFINITY) {
        l = (m > -INFINITY ? l * exp2f(m - mn) : 0.f) + (mo > -INFINITY ? lo * exp2f(mo - mn) : 0.f);
        m = mn;
      }
    }
    if (lane == 0) {
      sm[h] = m;
      sinv[h] = l > 0.f ? 1.0f / l : 0.f;
    }
  }
  __syncthreads();
  const int t = blockIdx.x * THREADS + threadIdx.x;
  if (t >= p.n_valid) return;
  double acc = 0.0;
  for (int h = 0; h < n_heads; ++h) {
    const float s = p.scores[(int64_t)h * p.n_valid + t];
    const float pr = s > -INFINITY ? exp2f(s - sm[h]) * sinv[h] : 0.f;
    acc += (double)pr;
  }
  p.importance[t] += acc;
}

}  // namespace imp
}  // namespace nyion

using namespace nyion;
using namespace nyion::imp;

extern "C" int32_t nyion_attn_decode_zoned_f32_tracked(float* out, const float* q, const float* k_arena,
                                                       const float* v_arena, int64_t n_arena_pages,
                                                       int32_t n_layers, int32_t layer_idx, int64_t seq_len,
                                                       int64_t q_pos, int32_t n_heads, int32_t n_kv_heads,
                                                       int32_t head_dim, double* importance, void* stream) {
  if (!importance) return fail(NYION_ERR_INVALID, "decode_zoned_f32_tracked: importance is required");
  if (n_heads > MAX_HEADS)
    return fail(NYION_ERR_UNSUPPORTED, "decode_zoned_f32_tracked: at most %d query heads", MAX_HEADS);
  if (seq_len > 0 && q_pos >= 0) {
    const int64_t ve = q_pos < seq_len - 1 ? q_pos : seq_len - 1;
    if (ve + 1 <= zoned_small_max() && head_dim == HD && n_kv_heads > 0 && n_heads == n_kv_heads * GROUP &&
        n_layers > 0 && layer_idx >= 0 && layer_idx < n_layers && out && q && k_arena && v_arena)
      return zoned_small(out, q, k_arena, v_arena, n_arena_pages, n_layers, layer_idx, ve + 1, n_kv_heads, head_dim,
                         importance, stream);   // one launch: output and weights
  }
  int32_t st = nyion_attn_decode_zoned_f32(out, q, k_arena, v_arena, n_arena_pages, n_layers, layer_idx, seq_len,
                                           q_pos, n_heads, n_kv_heads, head_dim, stream);
  if (st) return st;
  // the zoned decode has checked the shapes and arguments
  const int64_t valid_end = q_pos < seq_len - 1 ? q_pos : seq_len - 1;
  const int n_valid = (int)(valid_end + 1);
  const int n_chunks = (n_valid + CHUNK - 1) / CHUNK;
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st) return st;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t sc_bytes = al((size_t)n_heads * n_valid * sizeof(float));
  const size_t need = sc_bytes + (size_t)n_heads * n_chunks * sizeof(float2);
  void* ws = nullptr;
  st = internal_workspace(need, &ws);
  if (st) return st;
  Params p{};
  p.q = q;
  p.k_arena = k_arena;
  p.n_arena_pages = n_arena_pages;
  p.n_layers = n_layers;
  p.layer = layer_idx;
  p.n_kv = n_kv_heads;
  p.n_valid = n_valid;
  p.n_chunks = n_chunks;
  p.sl2 = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  p.scores = static_cast<float*>(ws);
  p.part = reinterpret_cast<float2*>(static_cast<uint8_t*>(ws) + sc_bytes);
  p.importance = importance;
  p.err = dev->err_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  scores_kernel<<<dim3((unsigned)n_kv_heads, (unsigned)n_chunks), THREADS, 0, s>>>(p);
  st = check_cuda(cudaGetLastError(), "decode_zoned_f32_tracked scores");
  if (st) return st;
  importance_kernel<<<(unsigned)((n_valid + THREADS - 1) / THREADS), THREADS, 0, s>>>(p, n_heads);
  return check_cuda(cudaGetLastError(), "decode_zoned_f32_tracked importance");
}
