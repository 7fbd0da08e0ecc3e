// decode_contig.cu — single-sequence decode over row caches: the layouts
// where one KV head's tokens are consecutive 64-wide rows.
//
//   * contiguous f32 / f16 caches [n_kv][stride][64] behind the reference's
//     CUDA C ABI (gpu_attention_device / _streamed / _streamed_half and the
//     gpu_graph_* pair, swamp-gpu/kernels/fused_attention.cu:194-243,
//     :483-582, :597-717; the two-pass kernel_scores +
//     kernel_softmax_weighted_sum at :20-124);
//   * the f16 ring of the layer-graph attention node, its length read from
//     device memory at run time (kernel_scores_dptr / kernel_softmax_v_dptr,
//     fused_attention.cu:1505-1556; the scheduler clamps the length to the
//     ring window, scheduler.rs:103-171);
//   * the zone-page arena of ops::attention (swamp-engine/src/ops.rs:170-278
//     over cache.rs:185-237, 681-747) above the short-context kernel's 512
//     tokens: zone pages of 32 / 128 / 1024 slots hold each KV head's slots
//     as consecutive rows, so every 32-token tile is one run of rows there too.
//
// One call is a few MB to a few tens of MB read once, so the design is about
// keeping HBM busy from the first cycle and keeping the merge short:
//
//   * grid = (KV head, split): each CTA owns a contiguous range of 32-token
//     tiles; splits are sized so ~2 CTAs run per SM (TARGET_CTAS);
//   * thread 0 streams the tiles with 1-D bulk copies (K rows, V rows) into a
//     96 KB ring of stages, all stages in flight from the start; a stage is
//     refilled one barrier after its last reader is done;
//   * scores: thread = (token, 1/8 of the dims) holds the pre-scaled query of
//     all 8 heads of the GQA group for its dims (64 registers), reads its K
//     slice from shared memory once (conflict-free 16-byte loads) and folds
//     the 8 head partials across its 8 lanes by a reduce-scatter (7 shuffles)
//     — every K byte is read from shared memory once for all 8 heads;
//   * softmax: warp = head, lane = token; online log2-domain max and sum;
//   * P.V: warp = 4 tokens of the tile, lane = (4 dims, 4 heads), 16 fp32
//     accumulators; the 8 warps' accumulators are summed once at the end;
//   * every CTA leaves one (m, l, o[8][64]) partial per KV head; a counter per
//     KV head tells the last CTA to merge them: warp = head, the weights
//     computed once per split, then every lane sums its two dims over the
//     splits with 8 loads in flight.  A single split writes the output
//     directly.  All arithmetic is fp32 FMA (no operand rounding).
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace contig {

constexpr int HD = 64;
constexpr int GROUP = 8;
constexpr int TILE = 32;               // tokens per stage
constexpr int THREADS = 256;
constexpr int KV_BYTES = 96 * 1024;    // stage ring
constexpr int TARGET_CTAS = 296;       // 2 CTAs per SM on 148 SMs
constexpr int MAX_SPLITS = TARGET_CTAS;

enum Layout { kRows = 0, kZoned = 1 };

struct Params {
  const float* q;            // [n_kv * 8][64]
  const void* k;             // rows of 64 elements
  const void* v;
  float* out;                // [n_kv * 8][64]
  int64_t stride;            // kRows: rows per KV head
  int32_t n_kv;
  int32_t n;                 // tokens attended (host length), when d_len is null
  const int32_t* d_len;      // device length, clamped to [0, window]
  int32_t window;
  int32_t n_layers, layer;   // kZoned
  int64_t n_pages;           // kZoned: pages in the arena
  int32_t tiles_per_split;
  int32_t n_splits;
  float sl2;                 // scale * log2(e)
  int32_t* cnt;              // [n_kv] merge counters (start at 0, left at 0)
  float2* part_ml;           // [n_kv][n_splits][8] (m, l)
  float* part_o;             // [n_kv][n_splits][8][64] o relative to m
  int32_t* err;
};

template <typename T>
struct Geo {
  static constexpr int RB = HD * (int)sizeof(T);            // row bytes
  static constexpr int TILE_BYTES = TILE * RB;              // one of K, V
  static constexpr int STAGES = KV_BYTES / (2 * TILE_BYTES);
};

struct Tail {                       // after the stage ring
  uint64_t full[16];
  int32_t rows[16];                 // valid rows copied into the stage (0: none)
  float sp[2][TILE][9];             // scores, then probabilities: [token][head], padded
  float alpha[2][GROUP];
  int32_t last;
};

size_t smem_bytes() { return KV_BYTES + sizeof(Tail) + 128; }

// first row of the 32-token tile starting at t0 for KV head kvh, or -1 when
// its zone page is not in the arena
template <int LAYOUT>
__device__ __forceinline__ int64_t tile_row(const Params& p, int kvh, int t0) {
  if (LAYOUT == kRows) return (int64_t)kvh * p.stride + t0;
  // cache.rs:185-237, 681-747: zone z holds pages of bs_z slots laid out
  // [layer][kv head][slot][64]; pages are consecutive in the arena.
  const int zone = t0 < 4096 ? 0 : (t0 < 131072 ? 1 : 2);
  const int64_t bs = zone == 0 ? 32 : (zone == 1 ? 128 : 1024);
  const int64_t zs = zone == 0 ? 0 : (zone == 1 ? 4096 : 131072);
  const int64_t zpage = zone == 0 ? 0 : (zone == 1 ? 128 : 1120);
  const int64_t lp = (int64_t)p.n_layers * p.n_kv;
  const int64_t zrow = zone == 0 ? 0 : (zone == 1 ? 128 * lp * 32 : 128 * lp * 32 + 992 * lp * 128);
  const int64_t local = (t0 - zs) / bs, slot = (t0 - zs) % bs;
  if (zpage + local >= p.n_pages) return -1;
  return zrow + local * lp * bs + ((int64_t)p.layer * p.n_kv + kvh) * bs + slot;
}

template <typename T, int LAYOUT>
__device__ __forceinline__ void issue_tile(const Params& p, uint8_t* kv, Tail& t, int kvh, int tile, int n,
                                           int stage) {
  using G = Geo<T>;
  const int t0 = tile * TILE;
  int rows = min(TILE, n - t0);
  const int64_t r0 = tile_row<LAYOUT>(p, kvh, t0);
  if (r0 < 0) {
    record_error(p.err, kErrPageRange);
    rows = 0;
  }
  t.rows[stage] = rows;
  if (rows > 0) {
    uint8_t* dst = kv + stage * 2 * G::TILE_BYTES;
    const uint32_t bytes = (uint32_t)rows * G::RB;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&t.full[stage], 2 * bytes);
    bulk_load(dst, static_cast<const uint8_t*>(p.k) + r0 * G::RB, bytes, &t.full[stage]);
    bulk_load(dst + G::TILE_BYTES, static_cast<const uint8_t*>(p.v) + r0 * G::RB, bytes, &t.full[stage]);
  } else {
    mbar_arrive(&t.full[stage]);
  }
}

// the 8 dims of row slice c: f32 rows take float4 chunks c and c + 8,
// f16 rows take the 16-byte chunk c
template <typename T>
__device__ __forceinline__ void load_slice(uint32_t row_addr, int c, float (&x)[8]) {
  if (sizeof(T) == 4) {
    const float4 a = lds128(row_addr + 16 * c), b = lds128(row_addr + 128 + 16 * c);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
    uint32_t u0, u1, u2, u3;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(u0), "=r"(u1), "=r"(u2), "=r"(u3)
                 : "r"(row_addr + 16 * c));
    const uint32_t u[4] = {u0, u1, u2, u3};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[e]));
      x[2 * e] = f.x;
      x[2 * e + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ int slice_dim(int c, int e) {
  return sizeof(T) == 4 ? (e < 4 ? 4 * c + e : 32 + 4 * c + (e - 4)) : 8 * c + e;
}

// 4 consecutive dims of a V row, starting at dim 4 * dq
template <typename T>
__device__ __forceinline__ float4 load_v4(uint32_t row_addr, int dq) {
  if (sizeof(T) == 4) return lds128(row_addr + 16 * dq);
  uint32_t u0, u1;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(u0), "=r"(u1) : "r"(row_addr + 8 * dq));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u0));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u1));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <typename T, int LAYOUT>
__global__ void __launch_bounds__(THREADS, 2) contig_kernel(const Params p) {
  using G = Geo<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* kv = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  Tail& t = *reinterpret_cast<Tail*>(kv + KV_BYTES);
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;

  int n = p.n;
  if (p.d_len) {
    n = __ldg(p.d_len);
    n = n < 0 ? 0 : (n > p.window ? p.window : n);
  }
  const int n_tiles = (n + TILE - 1) / TILE;
  const int tb = split * p.tiles_per_split;
  const int my_tiles = max(0, min(n_tiles, tb + p.tiles_per_split) - tb);

  if (tid == 0) {
    for (int s = 0; s < G::STAGES; ++s) mbar_init(&t.full[s], 1);
    fence_barrier_init();
    for (int k = 0; k < my_tiles && k < G::STAGES; ++k) issue_tile<T, LAYOUT>(p, kv, t, kvh, tb + k, n, k);
  }

  // query slice: thread (token j, slice c) holds q[h][dims of c] * scale * log2(e)
  const int j = tid >> 3, c = tid & 7;
  float qr[GROUP][8];
  {
    const float* qb = p.q + (int64_t)kvh * GROUP * HD;
#pragma unroll
    for (int h = 0; h < GROUP; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[h][e] = __ldg(qb + h * HD + slice_dim<T>(c, e)) * p.sl2;
  }
  __syncthreads();   // barriers initialised

  const int dq = lane & 15, hh = lane >> 4;
  float o[4][4];
#pragma unroll
  for (int e = 0; e < 4; ++e) o[e][0] = o[e][1] = o[e][2] = o[e][3] = 0.f;
  float M = -INFINITY, l = 0.f;   // softmax state of head w (warp-uniform)
  int issued = my_tiles < G::STAGES ? my_tiles : G::STAGES;
  int i = 0;
  bool aborted = false;
  for (; i < my_tiles; ++i) {
    const int st = i % G::STAGES, buf = i & 1;
    const uint32_t ph = (uint32_t)(i / G::STAGES) & 1u;
    const bool ok = mbar_wait_bounded(&t.full[st], ph);
    const int rows = t.rows[st];
    const uint32_t kbase = smem_u32(kv + st * 2 * G::TILE_BYTES);
    const uint32_t vbase = kbase + G::TILE_BYTES;
    // ---- scores: 8 head partials over this thread's 8 dims ----
    float part[GROUP];
    {
      float x[8];
      load_slice<T>(kbase + j * G::RB, c, x);
#pragma unroll
      for (int h = 0; h < GROUP; ++h) {
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) a = fmaf(qr[h][e], x[e], a);
        part[h] = a;
      }
    }
    // reduce-scatter over the 8 lanes of the token: lane c ends with head c
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
      const float s = keep + __shfl_xor_sync(0xffffffffu, send, 1);
      t.sp[buf][j][c] = j < rows ? s : -INFINITY;
    }
    if (__syncthreads_or(!ok)) {   // every reader of stage (i-1) is done here
      aborted = true;
      break;
    }
    if (tid == 0 && i >= 1 && i - 1 + G::STAGES < my_tiles) {
      issue_tile<T, LAYOUT>(p, kv, t, kvh, tb + i - 1 + G::STAGES, n, (i - 1) % G::STAGES);
      ++issued;
    }
    // ---- softmax: warp = head, lane = token ----
    {
      const float s = t.sp[buf][lane][w];
      const float mn = fmaxf(M, warp_max(s));
      float alpha = 1.f, pr = 0.f;
      if (mn > -INFINITY) {
        alpha = exp2f(M - mn);
        pr = exp2f(s - mn);
      }
      l = fmaf(l, alpha, warp_sum(pr));
      M = mn;
      t.sp[buf][lane][w] = pr;
      if (lane == 0) t.alpha[buf][w] = alpha;
    }
    __syncthreads();
    // ---- P.V: warp = tokens 4w..4w+3, lane = (dims 4dq.., heads 4hh..) ----
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = t.alpha[buf][4 * hh + e];
      o[e][0] *= a; o[e][1] *= a; o[e][2] *= a; o[e][3] *= a;
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int tok = 4 * w + jj;
      if (tok >= rows) break;
      const float4 v = load_v4<T>(vbase + tok * G::RB, dq);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = t.sp[buf][tok][4 * hh + e];
        o[e][0] = fmaf(pe, v.x, o[e][0]);
        o[e][1] = fmaf(pe, v.y, o[e][1]);
        o[e][2] = fmaf(pe, v.z, o[e][2]);
        o[e][3] = fmaf(pe, v.w, o[e][3]);
      }
    }
  }
  if (aborted) {
    // a copy never landed: wait (bounded) for the copies this CTA issued, then
    // publish an empty partial so the merge counters stay consistent
    record_error(p.err, kErrWaitTimeout);
    if (tid == 0)
      for (int k = i; k < issued; ++k) mbar_wait_bounded(&t.full[k % G::STAGES], (uint32_t)(k / G::STAGES) & 1u);
    M = -INFINITY;
    l = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e][0] = o[e][1] = o[e][2] = o[e][3] = 0.f;
  }
  __syncthreads();   // the stage ring is free: sum the 8 warps' accumulators there
  float* red = reinterpret_cast<float*>(kv);   // [warp][head][64]
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
  // thread (head w, dims 2*lane, 2*lane+1); (M, l) of head w are this warp's
  const int h = w;
  float* dst = p.out + ((int64_t)kvh * GROUP + h) * HD + 2 * lane;
  if (p.n_splits == 1) {
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    *reinterpret_cast<float2*>(dst) = make_float2(acc.x * inv, acc.y * inv);
    return;
  }
  const int64_t slot = (int64_t)kvh * p.n_splits + split;
  __stcg(reinterpret_cast<float2*>(p.part_o + (slot * GROUP + h) * HD + 2 * lane), acc);
  if (lane == 0) __stcg(&p.part_ml[slot * GROUP + h], make_float2(M, l));
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(&p.cnt[kvh], 1);
    const int last = old == p.n_splits - 1;
    if (last) atomicExch(&p.cnt[kvh], 0);
    t.last = last;
  }
  __syncthreads();
  if (!t.last) return;
  __threadfence();
  // ---- merge the splits of this KV head: warp = head ----
  float* wgt = reinterpret_cast<float*>(kv + GROUP * GROUP * HD * sizeof(float)) + h * MAX_SPLITS;
  const int S = p.n_splits;
  const float2* ml = p.part_ml + (int64_t)kvh * S * GROUP + h;
  float mx = -INFINITY;
  for (int s = lane; s < S; s += 32) mx = fmaxf(mx, __ldcg(ml + (int64_t)s * GROUP).x);
  mx = warp_max(mx);
  float den = 0.f;
  for (int s = lane; s < S; s += 32) {
    const float2 v = __ldcg(ml + (int64_t)s * GROUP);
    const float wv = (mx > -INFINITY && v.x > -INFINITY) ? exp2f(v.x - mx) : 0.f;
    wgt[s] = wv;
    den = fmaf(wv, v.y, den);
  }
  den = warp_sum(den);
  __syncwarp();
  const float* po = p.part_o + ((int64_t)kvh * S * GROUP + h) * HD + 2 * lane;
  float2 r = make_float2(0.f, 0.f);
  int s = 0;
  for (; s + 8 <= S; s += 8) {
    float2 x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] = __ldcg(reinterpret_cast<const float2*>(po + (int64_t)(s + u) * GROUP * HD));
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float wv = wgt[s + u];
      r.x = fmaf(wv, x[u].x, r.x);
      r.y = fmaf(wv, x[u].y, r.y);
    }
  }
  for (; s < S; ++s) {
    const float2 x = __ldcg(reinterpret_cast<const float2*>(po + (int64_t)s * GROUP * HD));
    const float wv = wgt[s];
    r.x = fmaf(wv, x.x, r.x);
    r.y = fmaf(wv, x.y, r.y);
  }
  const float inv = den > 0.f ? 1.0f / den : 0.f;
  *reinterpret_cast<float2*>(dst) = make_float2(r.x * inv, r.y * inv);
}

struct Plan {
  int n_splits, tiles_per_split;
};

Plan plan(int n_kv, int max_tokens) {
  const int tiles = max_tokens > 0 ? (max_tokens + TILE - 1) / TILE : 1;
  int per_head = TARGET_CTAS / n_kv;
  if (per_head < 1) per_head = 1;
  int s = tiles < per_head ? tiles : per_head;
  const int tps = (tiles + s - 1) / s;
  s = (tiles + tps - 1) / tps;   // no trailing split without tiles
  return {s, tps};
}

size_t al(size_t x) { return (x + 255) & ~size_t(255); }

size_t counters_bytes(int n_kv) { return al((size_t)n_kv * sizeof(int32_t)); }

size_t workspace_bytes(int n_kv, int max_tokens) {
  const Plan pl = plan(n_kv, max_tokens);
  const size_t slots = (size_t)n_kv * pl.n_splits * GROUP;
  return counters_bytes(n_kv) + al(slots * sizeof(float2)) + al(slots * HD * sizeof(float));
}

template <typename T, int LAYOUT>
int32_t launch(Params p, int max_tokens, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (p.n_kv <= 0 || p.n_kv > 65535) return fail(NYION_ERR_INVALID, "row decode: bad n_kv_heads %d", p.n_kv);
  if ((reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v)) & 15)
    return fail(NYION_ERR_INVALID, "row decode: K/V must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(p.out) & 7) return fail(NYION_ERR_INVALID, "row decode: out must be 8-byte aligned");
  DeviceInfo* dev = nullptr;
  int32_t st = device_info(&dev);
  if (st) return st;
  const Plan pl = plan(p.n_kv, max_tokens);
  const size_t need = workspace_bytes(p.n_kv, max_tokens);
  if (!ws) {
    st = internal_workspace(need, &ws, kWsCounters, counters_bytes(p.n_kv), stream);
    if (st) return st;
  } else if (ws_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "row decode: workspace %zu B < %zu B", ws_bytes, need);
  }
  static bool attr_set[64] = {false};
  const int di = dev->device < 64 ? dev->device : 0;
  if (!attr_set[di]) {
    st = check_cuda(cudaFuncSetAttribute(contig_kernel<T, LAYOUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_bytes()),
                    "cudaFuncSetAttribute(row decode)");
    if (st) return st;
    attr_set[di] = true;
  }
  p.n_splits = pl.n_splits;
  p.tiles_per_split = pl.tiles_per_split;
  uint8_t* base = static_cast<uint8_t*>(ws);
  const size_t slots = (size_t)p.n_kv * pl.n_splits * GROUP;
  p.cnt = reinterpret_cast<int32_t*>(base);
  p.part_ml = reinterpret_cast<float2*>(base + counters_bytes(p.n_kv));
  p.part_o = reinterpret_cast<float*>(base + counters_bytes(p.n_kv) + al(slots * sizeof(float2)));
  p.err = dev->err_word;
  contig_kernel<T, LAYOUT><<<dim3((unsigned)p.n_kv, (unsigned)pl.n_splits), THREADS, smem_bytes(), stream>>>(p);
  return check_cuda(cudaGetLastError(), "row decode launch");
}

}  // namespace contig

size_t contig_workspace_bytes(int n_kv, int max_tokens) { return contig::workspace_bytes(n_kv, max_tokens); }

int32_t contig_rows_f32(const float* q, const float* k, const float* v, float* out, int n_kv, int64_t stride, int n,
                        float sl2, void* ws, size_t ws_bytes, cudaStream_t stream) {
  contig::Params p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.stride = stride;
  p.n_kv = n_kv;
  p.n = n;
  p.sl2 = sl2;
  return contig::launch<float, contig::kRows>(p, n, ws, ws_bytes, stream);
}

int32_t contig_rows_f16(const float* q, const void* k, const void* v, float* out, int n_kv, int64_t stride, int n,
                        const int32_t* d_len, int window, float sl2, void* ws, size_t ws_bytes,
                        cudaStream_t stream) {
  contig::Params p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.stride = stride;
  p.n_kv = n_kv;
  p.n = n;
  p.d_len = d_len;
  p.window = window;
  p.sl2 = sl2;
  return contig::launch<__half, contig::kRows>(p, d_len ? window : n, ws, ws_bytes, stream);
}

int32_t contig_zoned_f32(const float* q, const float* k_arena, const float* v_arena, float* out, int n_kv,
                         int n_layers, int layer, int64_t n_pages, int n, float sl2, void* ws, size_t ws_bytes,
                         cudaStream_t stream) {
  contig::Params p{};
  p.q = q;
  p.k = k_arena;
  p.v = v_arena;
  p.out = out;
  p.n_kv = n_kv;
  p.n = n;
  p.n_layers = n_layers;
  p.layer = layer;
  p.n_pages = n_pages;
  p.sl2 = sl2;
  return contig::launch<float, contig::kZoned>(p, n, ws, ws_bytes, stream);
}

}  // namespace nyion
