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
// Scattered positions cannot use page-granular copies, so the CTA gathers rows:
// CTA = (sequence, KV head, 128-position split).  Thread t < 128 resolves
// position t of the split to its page row; then every thread brings one K or
// V row (256 B, all sixteen 16-byte loads in flight; 4-bit rows are
// dequantized on the way with the reference's separate multiply and add) into
// shared memory, so each row crosses from memory once for all 8 query heads.
// The split is then computed in 32-position tiles: scores with thread =
// (position, 1/8 of the dims) holding the pre-scaled query of the 8 heads for
// its dims and a reduce-scatter over its 8 lanes; softmax with warp = head
// (online, log2 domain); P.V with warp = 4 positions, lane = (4 dims, 4
// heads).  The 8 warps' P.V sums are folded in shared memory into one
// (o/l, m, l) partial per head and split, merged by nyion_attn_lse_combine.
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
constexpr int SPLIT = 128;            // positions per CTA
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

// 4-bit row `row` (40 bytes: two 20-byte blocks [f16 d][f16 dmin][16 nibble
// bytes]) dequantized into x[64]; element i of a block in byte i/2, low nibble
// for even i (the writer's order, cache.rs:637-663)
__device__ __forceinline__ void load_row_q4(const Params& p, int64_t row, float (&x)[HD]) {
  const uint2* r = reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(p.pool) + row * 40);
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
        const int i = 8 * wq + e;
        const uint32_t n = (nib >> (8 * (e >> 1) + 4 * (e & 1))) & 0xF;
        x[32 * blk + i] = __fadd_rn(__fmul_rn(d, (float)n), dm);
      }
    }
  }
}

struct GatherSmem {
  float k[SPLIT][HD];
  float v[SPLIT][HD];
  float qs[GROUP][HD];
  int64_t row[SPLIT];               // K row index in the pool (V: + PAGE), -1: none
  float sp[2][32][9];               // scores, then probabilities: [position][head], padded
  float alpha[2][GROUP];
};

// one K or V row of the pool into x[64]: f32 as is, 4-bit dequantized
// (cache.rs:375-394: d * q + dmin with a separate multiply and add)
template <bool Q4>
__device__ __forceinline__ void gather_row(const Params& p, int64_t row, float* dst) {
  if (!Q4) {
    const float4* r = reinterpret_cast<const float4*>(static_cast<const float*>(p.pool) + row * HD);
    float4 v[HD / 4];
#pragma unroll
    for (int c = 0; c < HD / 4; ++c) v[c] = __ldg(r + c);
#pragma unroll
    for (int c = 0; c < HD / 4; ++c) reinterpret_cast<float4*>(dst)[c] = v[c];
  } else {
    float x[HD];
    load_row_q4(p, row, x);
#pragma unroll
    for (int c = 0; c < HD / 4; ++c)
      reinterpret_cast<float4*>(dst)[c] = make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
  }
}

template <bool Q4, bool RULE>
__global__ void __launch_bounds__(THREADS) positions_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  GatherSmem& sm = *reinterpret_cast<GatherSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 15) & ~uintptr_t(15));
  const int b = blockIdx.x / p.n_kv, kvh = blockIdx.x % p.n_kv, split = blockIdx.y;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int H = p.n_kv * GROUP;
  const int n = count_of<RULE>(p, b);
  const int j0 = split * SPLIT, j1 = min(j0 + SPLIT, n);
  if (j0 >= j1) {   // nothing to attend in this split: empty partials
    for (int i = tid; i < GROUP * PART; i += THREADS) {
      const int h = i / PART, e = i % PART;
      p.part[((int64_t)split * p.batch * H + (int64_t)b * H + kvh * GROUP + h) * PART + e] =
          e == HD ? -INFINITY : 0.f;
    }
    return;
  }
  const int cnt = j1 - j0;
  // ---- positions -> pool rows; q ----
  const float q0 = p.q[((int64_t)b * H + kvh * GROUP) * HD + tid];
  const float q1 = p.q[((int64_t)b * H + kvh * GROUP) * HD + tid + 256];
  if (tid < SPLIT) {
    int64_t r = -1;
    if (tid < cnt) {
      const int pos = position_of<RULE>(p, b, j0 + tid);
      const int pidx = pos / PAGE;
      int64_t page = -1;
      if (pos >= 0 && pidx < p.max_pages) page = p.table[(int64_t)b * p.max_pages + pidx];
      if (page < 0 || page >= p.n_pool_pages) record_error(p.err, kErrPageRange);
      else r = ((page * p.n_kv + kvh) * 2) * PAGE + pos % PAGE;
    }
    sm.row[tid] = r;
  }
  sm.qs[tid / HD][tid % HD] = q0 * p.sl2;
  sm.qs[(tid + 256) / HD][(tid + 256) % HD] = q1 * p.sl2;
  __syncthreads();
  // ---- gather: thread -> (row tid / 2, K or V) ----
  {
    const int r = tid >> 1, kv = tid & 1;
    float* dst = kv ? sm.v[r] : sm.k[r];
    const int64_t row = r < cnt ? sm.row[r] : -1;
    if (row >= 0) {
      gather_row<Q4>(p, row + kv * PAGE, dst);
    } else {
#pragma unroll
      for (int c = 0; c < HD / 4; ++c) reinterpret_cast<float4*>(dst)[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  // query slice: thread (position j, slice c) holds q[h][dims 4c..4c+3, 32+4c..32+4c+3]
  const int j = tid >> 3, c = tid & 7;
  __syncthreads();
  float qr[GROUP][8];
#pragma unroll
  for (int h = 0; h < GROUP; ++h)
#pragma unroll
    for (int e = 0; e < 8; ++e) qr[h][e] = sm.qs[h][e < 4 ? 4 * c + e : 32 + 4 * c + (e - 4)];
  const int dq = lane & 15, hh = lane >> 4;
  float o[4][4];
#pragma unroll
  for (int e = 0; e < 4; ++e) o[e][0] = o[e][1] = o[e][2] = o[e][3] = 0.f;
  float M = -INFINITY, l = 0.f;   // softmax state of head w
  const int n_tiles = (cnt + 31) / 32;
  for (int i = 0; i < n_tiles; ++i) {
    const int buf = i & 1, t0 = 32 * i;
    // ---- scores: 8 head partials over this thread's 8 dims, reduce-scatter over 8 lanes ----
    float part[GROUP];
    {
      const float4 a = *reinterpret_cast<const float4*>(&sm.k[t0 + j][4 * c]);
      const float4 bb = *reinterpret_cast<const float4*>(&sm.k[t0 + j][32 + 4 * c]);
      const float x[8] = {a.x, a.y, a.z, a.w, bb.x, bb.y, bb.z, bb.w};
#pragma unroll
      for (int h = 0; h < GROUP; ++h) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(qr[h][e], x[e], acc);
        part[h] = acc;
      }
    }
    float r4[4], r2[2];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float send = (c & 4) ? part[e] : part[e + 4];
      const float keep = (c & 4) ? part[e + 4] : part[e];
      r4[e] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float send = (c & 2) ? r4[e] : r4[e + 2];
      const float keep = (c & 2) ? r4[e + 2] : r4[e];
      r2[e] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    {
      const float send = (c & 1) ? r2[0] : r2[1];
      const float keep = (c & 1) ? r2[1] : r2[0];
      const float sc = keep + __shfl_xor_sync(0xffffffffu, send, 1);
      const bool valid = t0 + j < cnt && sm.row[t0 + j] >= 0;
      sm.sp[buf][j][c] = valid ? sc : -INFINITY;
    }
    __syncthreads();
    // ---- softmax: warp = head, lane = position ----
    {
      const float sc = sm.sp[buf][lane][w];
      const float mn = fmaxf(M, warp_max(sc));
      float alpha = 1.f, pr = 0.f;
      if (mn > -INFINITY) {
        alpha = exp2f(M - mn);
        pr = exp2f(sc - mn);
      }
      l = fmaf(l, alpha, warp_sum(pr));
      M = mn;
      sm.sp[buf][lane][w] = pr;
      if (lane == 0) sm.alpha[buf][w] = alpha;
    }
    __syncthreads();
    // ---- P.V: warp = positions 4w..4w+3 of the tile, lane = (dims 4dq.., heads 4hh..) ----
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = sm.alpha[buf][4 * hh + e];
      o[e][0] *= a; o[e][1] *= a; o[e][2] *= a; o[e][3] *= a;
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int tok = 4 * w + jj;
      const float4 v = *reinterpret_cast<const float4*>(&sm.v[t0 + tok][4 * dq]);   // zeros past the end
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = sm.sp[buf][tok][4 * hh + e];
        o[e][0] = fmaf(pe, v.x, o[e][0]);
        o[e][1] = fmaf(pe, v.y, o[e][1]);
        o[e][2] = fmaf(pe, v.z, o[e][2]);
        o[e][3] = fmaf(pe, v.w, o[e][3]);
      }
    }
  }
  __syncthreads();   // K rows are no longer read: fold the 8 warps' sums there
  float* red = &sm.k[0][0];   // [warp][head][64]
#pragma unroll
  for (int e = 0; e < 4; ++e)
    *reinterpret_cast<float4*>(red + (w * GROUP + 4 * hh + e) * HD + 4 * dq) =
        make_float4(o[e][0], o[e][1], o[e][2], o[e][3]);
  __syncthreads();
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int ww = 0; ww < 8; ++ww) {
    const float2 x = *reinterpret_cast<const float2*>(red + (ww * GROUP + w) * HD + 2 * lane);
    acc.x += x.x;
    acc.y += x.y;
  }
  const int h = kvh * GROUP + w;   // warp w holds head w's (M, l)
  float* dst = p.part + ((int64_t)split * p.batch * H + (int64_t)b * H + h) * PART;
  const float inv = l > 0.f ? 1.0f / l : 0.f;
  dst[2 * lane] = acc.x * inv;
  dst[2 * lane + 1] = acc.y * inv;
  if (lane == 0) {
    dst[HD] = l > 0.f ? M * 0.69314718055994531f : -INFINITY;
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

constexpr size_t kSmem = sizeof(GatherSmem) + 16;

template <bool Q4, bool RULE>
int32_t launch_positions(dim3 grid, const Params& p, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  const int di = dev < 64 ? dev : 0;
  if (!attr_set[di]) {
    const int32_t st = check_cuda(cudaFuncSetAttribute(positions_kernel<Q4, RULE>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem),
                                  "cudaFuncSetAttribute(positions)");
    if (st) return st;
    attr_set[di] = true;
  }
  positions_kernel<Q4, RULE><<<grid, THREADS, kSmem, stream>>>(p);
  return check_cuda(cudaGetLastError(), "positions launch");
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
  st = kv_format == 0 ? launch_positions<false, false>(grid, p, s) : launch_positions<true, false>(grid, p, s);
  if (st) return st;
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
  st = launch_positions<true, true>(dim3((unsigned)(batch * n_kv_heads), 1), p, s);   // <= 128 globals: one split
  if (st) return st;
  return nyion_attn_lse_combine(parts, 2, (int64_t)batch * n_heads, HD, out, stream);
}
