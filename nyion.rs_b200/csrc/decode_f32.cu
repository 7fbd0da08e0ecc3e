// decode_f32.cu — fp32 GQA decode attention over paged or contiguous KV.
//
// Restates the maths of ops::attention (swamp-engine/src/ops.rs:170-278):
// s_t = scale * <q_h, K_t>, p = softmax(s), o_h = sum_t p_t V_t, query head h
// reading KV head h / (n_heads / n_kv_heads) — as a single-pass online
// softmax on B200:
//
//   * work = (sequence, KV head, 32-token chunk) triples, flattened and cut
//     into equal contiguous ranges, one per persistent CTA (stream-K style),
//     so every SM gets the same number of KV bytes whatever the batch and
//     context mix;
//   * each chunk (2 pages of 16 tokens; K and V, 16 KB) arrives by four
//     128B-swizzled TMA tensor copies per page into a 4-stage mbarrier ring;
//   * the 8 query heads of a GQA group share every K/V byte read: warp w
//     scores heads 2w, 2w+1 for the chunk's 32 tokens (one token per lane, q
//     in registers), the PV product splits heads x dims x token-quarters;
//   * a (sequence, KV head) pair split across CTAs leaves log-sum-exp
//     partials (m, l, o) in the workspace; the last CTA to finish the pair
//     (per-pair counter) merges them and resets the counter to zero.
#include <math.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace f32dec {

constexpr int HD = 64;
constexpr int GROUP = 8;      // query heads per KV head
constexpr int CHUNK = 32;     // tokens per pipeline stage
constexpr int PAGE = 16;      // tokens per page (TMA box height)
constexpr int STAGES = 4;
constexpr int THREADS = 128;
constexpr int SUB = CHUNK * 128;     // one 32-row x 128-byte swizzled subtile
constexpr int STAGE_BYTES = 4 * SUB; // K dims 0-31, K dims 32-63, V 0-31, V 32-63
constexpr int MAX_SEQS = 512;        // sequences per launch
constexpr int MAX_GRID = 1024;
constexpr int RING = 32;             // chunks per page-row prefetch batch

enum Mode { kPool = 0, kContig = 1, kZoned = 2 };

struct Params {
  const float* q;           // [batch][n_kv*GROUP][HD]
  float* out;               // [batch][n_kv*GROUP][HD]
  const int32_t* table;     // pool: [batch][max_pages]
  const int32_t* seq_lens;  // [batch] or null (use uniform_len)
  int32_t uniform_len;
  int32_t batch, n_kv, max_pages;
  int64_t n_pool_pages;
  int32_t kv_stride;        // contiguous: rows per KV head
  int32_t n_layers, layer;  // zoned: layers per page, layer read
  float qscale;             // scale * log2(e)
  int32_t* cnt;             // [batch*n_kv] merge counters (start at 0, left at 0)
  float2* ml;               // [MAX_GRID + pairs][GROUP] (m, l) partials
  float* po;                // [MAX_GRID + pairs][GROUP][HD] unnormalised o partials
  int32_t* err;
};

struct Smem {
  uint8_t kv[STAGES][STAGE_BYTES];   // first member: 1024-byte aligned
  float p[CHUNK][GROUP];
  float alpha[GROUP];
  float lsum[GROUP];
  float mmax[GROUP];
  float red[2][16][16];
  uint64_t full[STAGES];
  int32_t prefix[MAX_SEQS + 1];      // flat chunk index where sequence b starts
  int32_t lens[MAX_SEQS];
  int32_t rows[2][RING][3];          // per chunk: K row of page 0, page 1, page count
  int32_t flag;
  int32_t warp_tot[THREADS / 32];
};

struct Cursor {
  int b, kvh, chunk, nchunks, len;
};

__device__ __forceinline__ int chunks_of(int len) { return (len + CHUNK - 1) / CHUNK; }

__device__ __forceinline__ void seek(Cursor& c, const Smem& s, int batch, int n_kv, int i) {
  int lo = 0, hi = batch;   // invariant: prefix[lo] <= i < prefix[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (s.prefix[mid] <= i) lo = mid; else hi = mid;
  }
  c.b = lo;
  c.len = s.lens[lo];
  c.nchunks = chunks_of(c.len);
  int off = i - s.prefix[lo];
  c.kvh = off / c.nchunks;
  c.chunk = off - c.kvh * c.nchunks;
  (void)n_kv;
}

__device__ __forceinline__ void advance(Cursor& c, const Smem& s, int batch, int n_kv) {
  if (++c.chunk < c.nchunks) return;
  c.chunk = 0;
  if (++c.kvh < n_kv) return;
  c.kvh = 0;
  do { ++c.b; } while (c.b < batch && s.lens[c.b] <= 0);
  if (c.b < batch) {
    c.len = s.lens[c.b];
    c.nchunks = chunks_of(c.len);
  }
}

// Warp 0 fills ring slot `slot` with the page rows of flat chunks
// [first, first + RING) ∩ [first, end): one chunk per lane.
template <int MODE>
__device__ void fill_rows(Smem& s, const Params& p, int slot, int first, int end, int lane) {
  int i = first + lane;
  if (i >= end) return;
  Cursor c;
  seek(c, s, p.batch, p.n_kv, i);
  int tok0 = c.chunk * CHUNK;
  int npg = (c.len - tok0 > PAGE) ? 2 : 1;
  int32_t r[2] = {-4 * PAGE, -4 * PAGE};
  for (int pg = 0; pg < npg; ++pg) {
    if (MODE == kPool) {
      int pidx = tok0 / PAGE + pg;
      int64_t page = -1;
      if (pidx < p.max_pages) page = p.table[(int64_t)c.b * p.max_pages + pidx];
      if (page < 0 || page >= p.n_pool_pages) {
        record_error(p.err, kErrPageRange);
        continue;   // row stays negative: the TMA box is zero-filled
      }
      r[pg] = (int32_t)(((page * p.n_kv + c.kvh) * 2) * PAGE);
    } else if (MODE == kZoned) {
      // cache.rs:185-237, 681-747: zone z holds pages of bs_z slots laid out
      // [layer][kv_head][slot][head_dim]; pages are consecutive in the arena.
      const int zone = tok0 < 4096 ? 0 : (tok0 < 131072 ? 1 : 2);
      const int64_t bs = zone == 0 ? 32 : (zone == 1 ? 128 : 1024);
      const int64_t zs = zone == 0 ? 0 : (zone == 1 ? 4096 : 131072);
      const int64_t zpage = zone == 0 ? 0 : (zone == 1 ? 128 : 1120);
      const int64_t lp = p.n_layers * (int64_t)p.n_kv;       // rows per slot across layers*heads
      const int64_t zrow = zone == 0 ? 0 : (zone == 1 ? 128 * lp * 32 : 128 * lp * 32 + 992 * lp * 128);
      const int64_t local = (tok0 - zs) / bs, slot = (tok0 - zs) % bs;
      if (zpage + local >= p.n_pool_pages) {
        record_error(p.err, kErrPageRange);
        continue;
      }
      r[pg] = (int32_t)(zrow + local * lp * bs + ((int64_t)p.layer * p.n_kv + c.kvh) * bs + slot +
                        pg * PAGE);
    } else {
      r[pg] = c.kvh * p.kv_stride + tok0 + pg * PAGE;
    }
  }
  s.rows[slot][lane][0] = r[0];
  s.rows[slot][lane][1] = r[1];
  s.rows[slot][lane][2] = npg;
}

template <int MODE>
__device__ __forceinline__ void issue(Smem& s, int stage, int k, const CUtensorMap* mk,
                                      const CUtensorMap* mv) {
  const int32_t* e = s.rows[(k / RING) & 1][k % RING];
  int npg = e[2];
  uint8_t* base = s.kv[stage];
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(&s.full[stage], (uint32_t)(npg * 4 * PAGE * 128));
  for (int pg = 0; pg < npg; ++pg) {
    int32_t rk = e[pg];
    int32_t rv = (MODE == kPool) ? rk + PAGE : rk;
    uint8_t* d = base + pg * PAGE * 128;
    tma_load_2d(d + 0 * SUB, mk, 0, rk, &s.full[stage]);
    tma_load_2d(d + 1 * SUB, mk, 32, rk, &s.full[stage]);
    tma_load_2d(d + 2 * SUB, mv, 0, rv, &s.full[stage]);
    tma_load_2d(d + 3 * SUB, mv, 32, rv, &s.full[stage]);
  }
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 2)
decode_f32_kernel(const Params p, const __grid_constant__ CUtensorMap map_k,
                  const __grid_constant__ CUtensorMap map_v) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int H = p.n_kv * GROUP;

  if (t == 0) {
    prefetch_tensormap(&map_k);
    prefetch_tensormap(&map_v);
    for (int i = 0; i < STAGES; ++i) mbar_init(&s.full[i], 1);
    fence_barrier_init();
  }

  // ---- sequence lengths and flat chunk prefix (block scan) ----
  for (int b = t; b < p.batch; b += THREADS) {
    int L = p.seq_lens ? p.seq_lens[b] : p.uniform_len;
    s.lens[b] = L > 0 ? L : 0;
  }
  __syncthreads();
  constexpr int PER = MAX_SEQS / THREADS;
  int local[PER];
  int run = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    int b = t * PER + j;
    int c = (b < p.batch) ? chunks_of(s.lens[b]) * p.n_kv : 0;
    local[j] = run;
    run += c;
  }
  int incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s.warp_tot[warp] = incl;
  __syncthreads();
  int woff = 0;
  for (int w = 0; w < warp; ++w) woff += s.warp_tot[w];
  int excl = woff + incl - run;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    int b = t * PER + j;
    if (b <= p.batch && b < MAX_SEQS + 1) s.prefix[b] = excl + local[j];
  }
  if (t == THREADS - 1 && p.batch == MAX_SEQS) s.prefix[MAX_SEQS] = excl + run;
  __syncthreads();

  // zero the outputs of empty sequences
  for (int b = blockIdx.x; b < p.batch; b += gridDim.x) {
    if (s.lens[b] == 0)
      for (int e = t; e < H * HD; e += THREADS) p.out[(int64_t)b * H * HD + e] = 0.0f;
  }

  const int total = s.prefix[p.batch];
  const int W = (total + gridDim.x - 1) / gridDim.x;
  const int begin = blockIdx.x * W;
  const int end = min(total, begin + W);
  if (begin >= end) return;
  const int n = end - begin;

  if (warp == 0) {
    fill_rows<MODE>(s, p, 0, begin, end, lane);
    fill_rows<MODE>(s, p, 1, begin + RING, end, lane);
  }
  __syncthreads();
  if (t == 0)
    for (int k = 0; k < STAGES && k < n; ++k) issue<MODE>(s, k, k, &map_k, &map_v);

  Cursor cur;
  seek(cur, s, p.batch, p.n_kv, begin);

  float q0[HD], q1[HD];
  float o[4][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int hq = t >> 6, tq = (t >> 4) & 3, c16 = t & 15, half = c16 >> 3, cc = c16 & 7;
  int aborted_at = -1;

  for (int k = 0; k < n; ++k) {
    const int stage = k % STAGES;
    const bool seg_start = (k == 0) || (cur.chunk == 0);
    const bool seg_end = (k == n - 1) || (cur.chunk == cur.nchunks - 1);
    if (seg_start) {
      const float* qp = p.q + ((int64_t)cur.b * H + cur.kvh * GROUP + 2 * warp) * HD;
#pragma unroll
      for (int d = 0; d < HD; d += 4) {
        float4 a = __ldg(reinterpret_cast<const float4*>(qp + d));
        float4 bq = __ldg(reinterpret_cast<const float4*>(qp + HD + d));
        q0[d] = a.x * p.qscale; q0[d + 1] = a.y * p.qscale;
        q0[d + 2] = a.z * p.qscale; q0[d + 3] = a.w * p.qscale;
        q1[d] = bq.x * p.qscale; q1[d + 1] = bq.y * p.qscale;
        q1[d + 2] = bq.z * p.qscale; q1[d + 3] = bq.w * p.qscale;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }
    // page rows for chunks [k + RING, k + 2*RING) into the ring slot just freed
    if (warp == 0 && k % RING == 0 && k > 0)
      fill_rows<MODE>(s, p, ((k / RING) + 1) & 1, begin + k + RING, end, lane);

    const int nv = min(CHUNK, cur.len - cur.chunk * CHUNK);
    bool ok = mbar_wait_bounded(&s.full[stage], (uint32_t)((k / STAGES) & 1));
    const uint8_t* st = s.kv[stage];

    // ---- scores: warp -> heads (2w, 2w+1), lane -> token ----
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float4 kk = *reinterpret_cast<const float4*>(st + swz128(lane, c));
      a0 = fmaf(q0[4 * c], kk.x, a0); a0 = fmaf(q0[4 * c + 1], kk.y, a0);
      a0 = fmaf(q0[4 * c + 2], kk.z, a0); a0 = fmaf(q0[4 * c + 3], kk.w, a0);
      b0 = fmaf(q1[4 * c], kk.x, b0); b0 = fmaf(q1[4 * c + 1], kk.y, b0);
      b0 = fmaf(q1[4 * c + 2], kk.z, b0); b0 = fmaf(q1[4 * c + 3], kk.w, b0);
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float4 kk = *reinterpret_cast<const float4*>(st + SUB + swz128(lane, c));
      a1 = fmaf(q0[32 + 4 * c], kk.x, a1); a1 = fmaf(q0[33 + 4 * c], kk.y, a1);
      a1 = fmaf(q0[34 + 4 * c], kk.z, a1); a1 = fmaf(q0[35 + 4 * c], kk.w, a1);
      b1 = fmaf(q1[32 + 4 * c], kk.x, b1); b1 = fmaf(q1[33 + 4 * c], kk.y, b1);
      b1 = fmaf(q1[34 + 4 * c], kk.z, b1); b1 = fmaf(q1[35 + 4 * c], kk.w, b1);
    }
    const bool valid = lane < nv;
    float s0 = valid ? a0 + a1 : -INFINITY;
    float s1 = valid ? b0 + b1 : -INFINITY;

    // ---- online softmax (log2 domain: q carries scale*log2 e) ----
    float mx0 = warp_max(s0), mx1 = warp_max(s1);
    float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
    float p0 = exp2f(s0 - mn0), p1 = exp2f(s1 - mn1);
    l0 = fmaf(l0, al0, p0);
    l1 = fmaf(l1, al1, p1);
    m0 = mn0;
    m1 = mn1;
    *reinterpret_cast<float2*>(&s.p[lane][2 * warp]) = make_float2(p0, p1);
    if (lane == 0) {
      s.alpha[2 * warp] = al0;
      s.alpha[2 * warp + 1] = al1;
    }
    if (__syncthreads_or(!ok)) { aborted_at = k; break; }

    // ---- PV: thread -> heads 4hq..4hq+3, dims 4*c16.., tokens tq mod 4 ----
    {
      float4 al = *reinterpret_cast<const float4*>(&s.alpha[4 * hq]);
      const float alv[4] = {al.x, al.y, al.z, al.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] *= alv[i];
      const uint8_t* vb = st + (2 + half) * SUB;
#pragma unroll
      for (int j = 0; j < CHUNK / 4; ++j) {
        const int tt = tq + 4 * j;
        if (tt < nv) {
          float4 pp = *reinterpret_cast<const float4*>(&s.p[tt][4 * hq]);
          float4 v = *reinterpret_cast<const float4*>(vb + swz128(tt, cc));
          const float pv[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            o[i][0] = fmaf(pv[i], v.x, o[i][0]);
            o[i][1] = fmaf(pv[i], v.y, o[i][1]);
            o[i][2] = fmaf(pv[i], v.z, o[i][2]);
            o[i][3] = fmaf(pv[i], v.w, o[i][3]);
          }
        }
      }
    }
    __syncthreads();
    if (t == 0 && k + STAGES < n) issue<MODE>(s, stage, k + STAGES, &map_k, &map_v);

    if (seg_end) {
      // ---- reduce l over lanes, o over token quarters ----
      float ls0 = warp_sum(l0), ls1 = warp_sum(l1);
      if (lane == 0) {
        s.lsum[2 * warp] = ls0;
        s.lsum[2 * warp + 1] = ls1;
        s.mmax[2 * warp] = m0;
        s.mmax[2 * warp + 1] = m1;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] += __shfl_xor_sync(0xffffffffu, o[i][j], 16);
      if ((warp & 1) && lane < 16) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          *reinterpret_cast<float4*>(&s.red[warp >> 1][lane][4 * i]) =
              make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
      }
      __syncthreads();
      const int pair = cur.b * p.n_kv + cur.kvh;
      const int pstart = s.prefix[cur.b] + cur.kvh * cur.nchunks;
      const int pend = pstart + cur.nchunks;
      const int cfirst = pstart / W, clast = (pend - 1) / W;
      const bool single = (cfirst == clast);
      const int slot = blockIdx.x + pair;
      const int h0 = 4 * (warp >> 1);
      if (!(warp & 1) && lane < 16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float4 r = *reinterpret_cast<const float4*>(&s.red[warp >> 1][lane][4 * i]);
          o[i][0] += r.x; o[i][1] += r.y; o[i][2] += r.z; o[i][3] += r.w;
        }
        if (single) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float inv = 1.0f / s.lsum[h0 + i];
            float* dst = p.out + ((int64_t)cur.b * H + cur.kvh * GROUP + h0 + i) * HD + 4 * lane;
            *reinterpret_cast<float4*>(dst) =
                make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float* dst = p.po + ((int64_t)slot * GROUP + h0 + i) * HD + 4 * lane;
            __stcg(reinterpret_cast<float4*>(dst), make_float4(o[i][0], o[i][1], o[i][2], o[i][3]));
          }
        }
      }
      if (!single) {
        if (t < GROUP) __stcg(&p.ml[(int64_t)slot * GROUP + t], make_float2(s.mmax[t], s.lsum[t]));
        __threadfence();
        __syncthreads();
        if (t == 0) {
          int old = atomicAdd(&p.cnt[pair], 1);
          int last = (old == clast - cfirst);
          if (last) atomicExch(&p.cnt[pair], 0);
          __threadfence();
          s.flag = last;
        }
        __syncthreads();
        if (s.flag) {
          const int h = t >> 4, c4 = (t & 15) * 4;
          float M = -INFINITY;
          for (int cb = cfirst; cb <= clast; ++cb) M = fmaxf(M, __ldcg(&p.ml[(int64_t)(cb + pair) * GROUP + h]).x);
          float den = 0.f;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int cb = cfirst; cb <= clast; ++cb) {
            float2 mlv = __ldcg(&p.ml[(int64_t)(cb + pair) * GROUP + h]);
            float w = exp2f(mlv.x - M);
            den = fmaf(w, mlv.y, den);
            float4 ov = ld_cg4(p.po + ((int64_t)(cb + pair) * GROUP + h) * HD + c4);
            acc.x = fmaf(w, ov.x, acc.x); acc.y = fmaf(w, ov.y, acc.y);
            acc.z = fmaf(w, ov.z, acc.z); acc.w = fmaf(w, ov.w, acc.w);
          }
          float inv = 1.0f / den;
          float* dst = p.out + ((int64_t)cur.b * H + cur.kvh * GROUP + h) * HD + c4;
          *reinterpret_cast<float4*>(dst) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
      }
    }
    advance(cur, s, p.batch, p.n_kv);
  }

  if (aborted_at >= 0) {
    record_error(p.err, kErrWaitTimeout);
    // drain the copies still in flight (chunks aborted_at .. aborted_at+STAGES-1)
    // before the CTA's shared memory is released; each wait is bounded too
    if (t == 0) {
      for (int c = aborted_at; c < n && c < aborted_at + STAGES; ++c)
        mbar_wait_bounded(&s.full[c % STAGES], (uint32_t)((c / STAGES) & 1));
    }
    __syncthreads();
  }
}

size_t smem_bytes() { return sizeof(Smem) + 1024; }

struct WsLayout {
  size_t cnt, ml, po, total;
};

WsLayout ws_layout(int batch, int n_kv) {
  int b = batch < MAX_SEQS ? batch : MAX_SEQS;
  size_t pairs = (size_t)b * n_kv;
  size_t slots = MAX_GRID + pairs;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  WsLayout w;
  w.cnt = 0;
  w.ml = al(pairs * sizeof(int32_t));
  w.po = w.ml + al(slots * GROUP * sizeof(float2));
  w.total = w.po + al(slots * GROUP * HD * sizeof(float));
  return w;
}

template <int MODE>
int32_t launch(const Params& base, const CUtensorMap& mk, const CUtensorMap& mv, int batch,
               const int32_t* seq_lens, const float* q, float* out, const int32_t* table,
               void* ws, cudaStream_t stream) {
  DeviceInfo* dev = nullptr;
  int32_t st = device_info(&dev);
  if (st) return st;
  static int occ_cache[64] = {0};
  int di = dev->device < 64 ? dev->device : 0;
  size_t smem = smem_bytes();
  if (!occ_cache[di]) {
    st = check_cuda(cudaFuncSetAttribute(decode_f32_kernel<MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "cudaFuncSetAttribute(decode_f32)");
    if (st) return st;
    int occ = 0;
    st = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_f32_kernel<MODE>,
                                                                  THREADS, smem),
                    "occupancy(decode_f32)");
    if (st) return st;
    occ_cache[di] = occ > 0 ? occ : 1;
  }
  int grid = dev->num_sms * occ_cache[di];
  if (grid > MAX_GRID) grid = MAX_GRID;
  WsLayout w = ws_layout(batch, base.n_kv);
  for (int b0 = 0; b0 < batch; b0 += MAX_SEQS) {
    Params p = base;
    int nb = batch - b0 < MAX_SEQS ? batch - b0 : MAX_SEQS;
    p.batch = nb;
    p.seq_lens = seq_lens ? seq_lens + b0 : nullptr;
    int H = base.n_kv * GROUP;
    p.q = q + (int64_t)b0 * H * HD;
    p.out = out + (int64_t)b0 * H * HD;
    p.table = table ? table + (int64_t)b0 * base.max_pages : nullptr;
    p.cnt = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + w.cnt);
    p.ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(ws) + w.ml);
    p.po = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + w.po);
    p.err = dev->err_word;
    decode_f32_kernel<MODE><<<grid, THREADS, smem, stream>>>(p, mk, mv);
    st = check_cuda(cudaGetLastError(), "decode_f32 launch");
    if (st) return st;
  }
  return NYION_OK;
}

int32_t check_common(int32_t n_heads, int32_t n_kv_heads, int32_t head_dim) {
  if (n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads)
    return fail(NYION_ERR_INVALID, "n_heads (%d) must be a positive multiple of n_kv_heads (%d)",
                n_heads, n_kv_heads);
  if (head_dim != HD || n_heads / n_kv_heads != GROUP)
    return fail(NYION_ERR_UNSUPPORTED,
                "this build has kernels for head_dim 64 and GQA group 8 (got head_dim %d, group %d)",
                head_dim, n_heads / n_kv_heads);
  return NYION_OK;
}

}  // namespace f32dec
}  // namespace nyion

using namespace nyion;
using namespace nyion::f32dec;

extern "C" size_t nyion_attn_decode_workspace_size(int32_t batch, int32_t n_kv_heads,
                                                   int32_t n_heads, int32_t head_dim) {
  (void)n_heads;
  (void)head_dim;
  if (batch <= 0 || n_kv_heads <= 0) return 0;
  return ws_layout(batch, n_kv_heads).total;
}

extern "C" int32_t nyion_attn_decode_paged_f32(const float* q, const float* kv_pool,
                                               int64_t n_pool_pages, const int32_t* page_table,
                                               int32_t max_pages, const int32_t* seq_lens,
                                               float* out, int32_t batch, int32_t n_heads,
                                               int32_t n_kv_heads, int32_t head_dim,
                                               int32_t page_tokens, float scale, void* workspace,
                                               size_t workspace_bytes, void* stream) {
  int32_t st = check_common(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!q || !kv_pool || !page_table || !seq_lens || !out)
    return fail(NYION_ERR_INVALID, "decode_paged_f32: null pointer argument");
  if (batch <= 0 || max_pages <= 0 || n_pool_pages <= 0)
    return fail(NYION_ERR_INVALID, "decode_paged_f32: batch, max_pages and n_pool_pages must be > 0");
  if (page_tokens != PAGE)
    return fail(NYION_ERR_UNSUPPORTED, "decode_paged_f32: page_tokens must be 16 (got %d)", page_tokens);
  uint64_t rows = (uint64_t)n_pool_pages * n_kv_heads * 2 * PAGE;
  if (rows > (1ull << 31))
    return fail(NYION_ERR_INVALID, "decode_paged_f32: pool of %lld pages exceeds 2^31 rows",
                (long long)n_pool_pages);
  size_t need = ws_layout(batch, n_kv_heads).total;
  if (!workspace) {
    st = internal_workspace(need, &workspace);
    if (st) return st;
  } else if (workspace_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "decode_paged_f32: workspace %zu < %zu bytes", workspace_bytes, need);
  }
  CUtensorMap map;
  st = encode_rows_tmap(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, kv_pool, HD, rows, 32, PAGE,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  Params p{};
  p.n_kv = n_kv_heads;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  return launch<kPool>(p, map, map, batch, seq_lens, q, out, page_table, workspace,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int32_t nyion_attn_decode_zoned_f32(float* out, const float* q, const float* k_arena,
                                               const float* v_arena, int64_t n_arena_pages,
                                               int32_t n_layers, int32_t layer_idx,
                                               int64_t seq_len, int64_t q_pos, int32_t n_heads,
                                               int32_t n_kv_heads, int32_t head_dim,
                                               void* stream) {
  int32_t st = check_common(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!out || !q || !k_arena || !v_arena)
    return fail(NYION_ERR_INVALID, "decode_zoned_f32: null pointer argument");
  if (seq_len <= 0 || q_pos < 0 || n_layers <= 0 || layer_idx < 0 || layer_idx >= n_layers ||
      n_arena_pages <= 0)
    return fail(NYION_ERR_INVALID, "decode_zoned_f32: bad seq_len/q_pos/layer/arena arguments");
  // ops.rs:183 valid_end = min(q_pos, seq_len - 1): tokens [0, valid_end] are attended
  int64_t valid_end = q_pos < seq_len - 1 ? q_pos : seq_len - 1;
  if (valid_end + 1 > (1ll << 30)) return fail(NYION_ERR_INVALID, "decode_zoned_f32: context too long");
  // rows in the arena: zone pages [0, n_arena_pages) of 32 / 128 / 1024 slots
  const int64_t lp = (int64_t)n_layers * n_kv_heads;
  int64_t z0 = n_arena_pages < 128 ? n_arena_pages : 128;
  int64_t z1 = n_arena_pages - z0 < 992 ? n_arena_pages - z0 : 992;
  int64_t z2 = n_arena_pages - z0 - z1;
  uint64_t rows = (uint64_t)(z0 * 32 + z1 * 128 + z2 * 1024) * lp;
  if (rows > (1ull << 31)) return fail(NYION_ERR_INVALID, "decode_zoned_f32: arena exceeds 2^31 rows");
  CUtensorMap mk, mv;
  st = encode_rows_tmap(&mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, k_arena, HD, rows, 32, PAGE,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  st = encode_rows_tmap(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, v_arena, HD, rows, 32, PAGE,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  void* ws = nullptr;
  st = internal_workspace(ws_layout(1, n_kv_heads).total, &ws);
  if (st) return st;
  Params p{};
  p.n_kv = n_kv_heads;
  p.n_layers = n_layers;
  p.layer = layer_idx;
  p.n_pool_pages = n_arena_pages;
  p.uniform_len = (int32_t)(valid_end + 1);
  p.qscale = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  return launch<kZoned>(p, mk, mv, 1, nullptr, q, out, nullptr, ws, static_cast<cudaStream_t>(stream));
}

// ---- reference CUDA C ABI (swamp-gpu/kernels/fused_attention.cu) -------------

static int32_t contig_decode(const float* d_q, const float* d_k, const float* d_v, float* d_out,
                             int n_heads, int n_kv_heads, int seq_len, int head_dim, int kv_stride,
                             void* ws, cudaStream_t stream) {
  int32_t st = check_common(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!d_q || !d_k || !d_v || !d_out) return fail(NYION_ERR_INVALID, "null pointer argument");
  if (seq_len <= 0 || kv_stride < seq_len)
    return fail(NYION_ERR_INVALID, "seq_len %d must be in [1, kv_stride=%d]", seq_len, kv_stride);
  uint64_t rows = (uint64_t)n_kv_heads * kv_stride;
  CUtensorMap mk, mv;
  st = encode_rows_tmap(&mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d_k, HD, rows, 32, PAGE,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  st = encode_rows_tmap(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d_v, HD, rows, 32, PAGE,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  if (!ws) {
    st = internal_workspace(ws_layout(1, n_kv_heads).total, &ws);
    if (st) return st;
  }
  Params p{};
  p.n_kv = n_kv_heads;
  p.kv_stride = kv_stride;
  p.uniform_len = seq_len;
  p.qscale = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  return launch<kContig>(p, mk, mv, 1, nullptr, d_q, d_out, nullptr, ws, stream);
}

extern "C" int gpu_attention_streamed(const float* d_q, const float* d_k_cache,
                                      const float* d_v_cache, float* d_output, int n_heads,
                                      int n_kv_heads, int seq_len, int head_dim, int kv_stride,
                                      void* stream) {
  return contig_decode(d_q, d_k_cache, d_v_cache, d_output, n_heads, n_kv_heads, seq_len, head_dim,
                       kv_stride, nullptr, static_cast<cudaStream_t>(stream)) == NYION_OK ? 0 : -1;
}

extern "C" int gpu_attention_device(const float* d_q, const float* d_k_cache,
                                    const float* d_v_cache, float* d_output, int n_heads,
                                    int n_kv_heads, int seq_len, int head_dim, int kv_stride) {
  return gpu_attention_streamed(d_q, d_k_cache, d_v_cache, d_output, n_heads, n_kv_heads, seq_len,
                                head_dim, kv_stride, nullptr);
}

extern "C" int gpu_attention_forward(const float* q, const float* k_cache, const float* v_cache,
                                     float* output, int n_heads, int n_kv_heads, int seq_len,
                                     int head_dim) {
  if (!q || !k_cache || !v_cache || !output) {
    fail(NYION_ERR_INVALID, "gpu_attention_forward: null pointer argument");
    return -1;
  }
  size_t qb = (size_t)n_heads * head_dim * sizeof(float);
  size_t kvb = (size_t)n_kv_heads * seq_len * head_dim * sizeof(float);
  float *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr;
  int rc = -1;
  if (check_cuda(cudaMalloc(&dq, qb), "cudaMalloc q") || check_cuda(cudaMalloc(&dk, kvb), "cudaMalloc k") ||
      check_cuda(cudaMalloc(&dv, kvb), "cudaMalloc v") || check_cuda(cudaMalloc(&dout, qb), "cudaMalloc out"))
    goto done;
  if (check_cuda(cudaMemcpy(dq, q, qb, cudaMemcpyHostToDevice), "copy q") ||
      check_cuda(cudaMemcpy(dk, k_cache, kvb, cudaMemcpyHostToDevice), "copy k") ||
      check_cuda(cudaMemcpy(dv, v_cache, kvb, cudaMemcpyHostToDevice), "copy v"))
    goto done;
  if (contig_decode(dq, dk, dv, dout, n_heads, n_kv_heads, seq_len, head_dim, seq_len, nullptr,
                    nullptr) != NYION_OK)
    goto done;
  if (check_cuda(cudaMemcpy(output, dout, qb, cudaMemcpyDeviceToHost), "copy out")) goto done;
  rc = 0;
done:
  cudaFree(dq);
  cudaFree(dk);
  cudaFree(dv);
  cudaFree(dout);
  return rc;
}

struct AttnGraph {
  cudaGraphExec_t exec;
  void* ws;
};

extern "C" void* gpu_graph_create_attention(const float* d_q, const float* d_k_cache,
                                            const float* d_v_cache, float* d_scores,
                                            float* d_output, int n_heads, int n_kv_heads,
                                            int seq_len, int head_dim, int kv_stride) {
  (void)d_scores;
  DeviceInfo* dev = nullptr;
  if (device_info(&dev)) return nullptr;
  size_t wsb = ws_layout(1, n_kv_heads > 0 ? n_kv_heads : 1).total;
  void* ws = nullptr;
  if (check_cuda(cudaMalloc(&ws, wsb), "cudaMalloc(graph workspace)")) return nullptr;
  if (check_cuda(cudaMemset(ws, 0, wsb), "cudaMemset(graph workspace)")) { cudaFree(ws); return nullptr; }
  cudaStream_t s;
  if (check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) {
    cudaFree(ws);
    return nullptr;
  }
  // one eager launch sets the kernel attributes outside capture
  if (contig_decode(d_q, d_k_cache, d_v_cache, d_output, n_heads, n_kv_heads, seq_len, head_dim,
                    kv_stride, ws, s) != NYION_OK ||
      check_cuda(cudaStreamSynchronize(s), "warm-up")) {
    cudaStreamDestroy(s);
    cudaFree(ws);
    return nullptr;
  }
  cudaGraph_t g = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool ok = check_cuda(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "BeginCapture") == 0;
  if (ok) {
    int32_t rc = contig_decode(d_q, d_k_cache, d_v_cache, d_output, n_heads, n_kv_heads, seq_len,
                               head_dim, kv_stride, ws, s);
    cudaError_t e = cudaStreamEndCapture(s, &g);
    ok = rc == NYION_OK && check_cuda(e, "EndCapture") == 0;
  }
  if (ok) ok = check_cuda(cudaGraphInstantiate(&exec, g, 0), "cudaGraphInstantiate") == 0;
  if (g) cudaGraphDestroy(g);
  cudaStreamDestroy(s);
  if (!ok) {
    cudaFree(ws);
    return nullptr;
  }
  AttnGraph* h = new AttnGraph{exec, ws};
  return h;
}

extern "C" int gpu_graph_replay_attention(void* graph_handle, void* stream) {
  if (!graph_handle) {
    fail(NYION_ERR_INVALID, "gpu_graph_replay_attention: null handle");
    return -1;
  }
  AttnGraph* h = static_cast<AttnGraph*>(graph_handle);
  return check_cuda(cudaGraphLaunch(h->exec, static_cast<cudaStream_t>(stream)), "cudaGraphLaunch") ? -1 : 0;
}

extern "C" void gpu_graph_destroy(void* graph_handle) {
  if (!graph_handle) return;
  AttnGraph* h = static_cast<AttnGraph*>(graph_handle);
  cudaGraphExecDestroy(h->exec);
  cudaFree(h->ws);
  delete h;
}
