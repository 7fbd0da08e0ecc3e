// decode_f32.cu — fp32 GQA decode attention over a paged KV pool (any number
// of KV heads; 4 KV heads take the whole-page kernel of decode_pages.cu), the
// short-context zone-arena kernel, and the reference's CUDA C ABI entry points
// (their single-sequence row-cache work runs in decode_contig.cu).
//
// Restates the maths of ops::attention (swamp-engine/src/ops.rs:170-278):
// s_t = scale * <q_h, K_t>, p = softmax(s), o_h = sum_t p_t V_t, query head h
// reading KV head h / (n_heads / n_kv_heads) — as a single-pass online
// softmax on B200:
//
//   * work = (sequence, KV head, 32-token chunk) triples, flattened and cut
//     into equal contiguous ranges, one per persistent CTA (stream-K style),
//     so every SM streams the same number of KV bytes whatever the batch and
//     context mix;
//   * a producer warp brings each chunk (two 16-token pages of K and V,
//     16 KB) into a 12-stage ring (full/empty mbarrier pair per stage).  In
//     the paged pool one 5-D TMA tensor copy moves a whole (page, KV head)
//     block — K and V, both 128-byte halves of every row, 8 KB — so a chunk
//     is two copies; page-table reads for the next 32 chunks are issued 16
//     chunks before they are needed, off the copy-issue critical path;
//   * six consumer warps take the chunks round-robin.  One warp computes a
//     whole chunk for all 8 query heads of the GQA group on the tensor cores
//     (mma.sync m16n8k16 bf16, fp32 accumulate), so every K/V byte is read
//     from shared memory once.  fp32 accuracy comes from splitting every
//     operand into bf16 hi + lo: the A operand stacks the hi rows (0..7) over
//     the lo rows (8..15) and the B operand is issued once with hi and once
//     with lo, so all four cross products accumulate and the residual is
//     ~2^-17 relative per operand.  K fragments come from ldmatrix on the
//     fp32 tile (dims permuted identically in q), P is reused from the score
//     accumulators as the A operand of P.V (no shared-memory round trip);
//   * every consumer warp keeps its own log-sum-exp partial (m, l, o) per
//     (sequence, KV head) segment and publishes it to the workspace when it
//     leaves the segment; a per-segment counter tells the last contributor
//     (whichever CTA and warp) to merge them and reset the counter to zero.
//     No barrier spans the consumer warps, so a slow warp never stalls the
//     others.  A segment served by one warp alone is written out directly.
#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace f32dec {

constexpr int HD = 64;
constexpr int GROUP = 8;              // query heads per KV head
constexpr int CHUNK = 32;             // tokens per pipeline stage
constexpr int PAGE = 16;              // tokens per page (TMA box height)
constexpr int NC = 6;                 // consumer warps
constexpr int STAGES = 12;            // two per consumer warp
constexpr int THREADS = (NC + 1) * 32;
constexpr int SUB = CHUNK * 128;      // 4096 B; a page block is 2*SUB: four 16-row x 128 B subtiles
constexpr int PAGE_BYTES = 8192;      // one (page, KV head) block in shared memory
constexpr int STAGE_BYTES = 4 * SUB;  // per page (8 KB): K dims 0-31 | K 32-63 | V 0-31 | V 32-63
constexpr int MAX_SEQS = 512;         // sequences per launch
constexpr int MAX_GRID = 1024;
constexpr int RING = 32;              // chunks per page-row prefetch batch

struct Params {
  const float* q;           // [batch][n_kv*GROUP][HD]
  float* out;               // [batch][n_kv*GROUP][HD]
  const int32_t* table;     // pool: [batch][max_pages]
  const int32_t* seq_lens;  // [batch]
  int32_t batch, n_kv, max_pages;
  int64_t n_pool_pages;
  float qscale;             // scale * log2(e)
  int32_t* cnt;             // [batch*n_kv] merge counters (start at 0, left at 0)
  float2* ml;               // [(MAX_GRID + pairs) * NC][GROUP] (m, l) partials
  float* po;                // [(MAX_GRID + pairs) * NC][GROUP][HD] o partials (relative to m)
  int32_t* err;
};

struct Smem {
  uint8_t kv[STAGES][STAGE_BYTES];   // first member: 1024-byte aligned
  uint64_t full[STAGES];             // TMA bytes landed
  uint64_t empty[STAGES];            // the consuming warp is done with the stage
  int32_t prefix[MAX_SEQS + 1];      // flat chunk index where sequence b starts
  int32_t lens[MAX_SEQS];
  int32_t rows[2][RING][3];          // per chunk: K row of page 0, page 1, page count
  int32_t warp_tot[THREADS / 32];
  int32_t abort_;
};

__device__ __forceinline__ int chunks_of(int len) { return (len + CHUNK - 1) / CHUNK; }

struct Cursor {
  int b, kvh, chunk, nchunks, len;
};

__device__ __forceinline__ void seek(Cursor& c, const Smem& s, int batch, int i) {
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
}

// Page rows of one chunk, prepared by a producer lane in two steps so the
// page-table load overlaps copy issue: rows_start() reads the table into
// registers, rows_finish() (16 chunks later) checks and stores them.
struct RowJob {
  int valid, npg, b, kvh, tok0;
  int64_t page[2];
};

__device__ __forceinline__ void rows_start(RowJob& j, const Smem& s, const Params& p, int i, int end) {
  j.valid = i < end;
  if (!j.valid) return;
  Cursor c;
  seek(c, s, p.batch, i);
  j.b = c.b;
  j.kvh = c.kvh;
  j.tok0 = c.chunk * CHUNK;
  j.npg = (c.len - j.tok0 > PAGE) ? 2 : 1;
  j.page[0] = j.page[1] = -1;
#pragma unroll
  for (int pg = 0; pg < 2; ++pg) {
    const int pidx = j.tok0 / PAGE + pg;
    if (pg < j.npg && pidx < p.max_pages) j.page[pg] = p.table[(int64_t)c.b * p.max_pages + pidx];
  }
}

// Stores per chunk: the (page * n_kv + kv head) block index of the 5-D map
// for page 0 and page 1, and the page count.
__device__ __forceinline__ void rows_finish(Smem& s, const Params& p, const RowJob& j, int slot,
                                            int lane) {
  if (!j.valid) return;
  int32_t r[2] = {-4 * PAGE, -4 * PAGE};
#pragma unroll
  for (int pg = 0; pg < 2; ++pg) {
    if (pg >= j.npg) continue;
    const int64_t page = j.page[pg];
    if (page < 0 || page >= p.n_pool_pages) {
      record_error(p.err, kErrPageRange);
      continue;   // negative coordinate: the TMA box is zero-filled
    }
    r[pg] = (int32_t)(page * p.n_kv + j.kvh);
  }
  s.rows[slot][lane][0] = r[0];
  s.rows[slot][lane][1] = r[1];
  s.rows[slot][lane][2] = j.npg;
}

__device__ __forceinline__ void issue(Smem& s, int stage, int k, const CUtensorMap* map) {
  const int32_t* e = s.rows[(k / RING) & 1][k % RING];
  const int npg = e[2];
  uint8_t* base = s.kv[stage];
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(&s.full[stage], (uint32_t)(npg * PAGE_BYTES));
  // (x, slot row, 128-B half, K/V, block): K_lo, K_hi, V_lo, V_hi subtiles
  for (int pg = 0; pg < npg; ++pg) tma_load_5d(base + pg * PAGE_BYTES, map, 0, 0, 0, 0, e[pg], &s.full[stage]);
}

__global__ void __launch_bounds__(THREADS, 1)
decode_f32_kernel(const Params p, const __grid_constant__ CUtensorMap map) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int H = p.n_kv * GROUP;

  if (t == 0) {
    prefetch_tensormap(&map);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    s.abort_ = 0;
    fence_barrier_init();
  }

  // ---- sequence lengths and flat chunk prefix (block scan) ----
  for (int b = t; b < p.batch; b += THREADS) {
    int L = p.seq_lens[b];
    s.lens[b] = L > 0 ? L : 0;
  }
  __syncthreads();
  constexpr int PER = (MAX_SEQS + THREADS - 1) / THREADS;
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
    if (b <= p.batch) s.prefix[b] = excl + local[j];
  }
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

  if (warp == NC) {
    // ================= producer warp =================
    RowJob job;
    rows_start(job, s, p, begin + lane, end);
    rows_finish(s, p, job, 0, lane);
    rows_start(job, s, p, begin + RING + lane, end);
    __syncwarp();
    for (int k = 0; k < n; ++k) {
      const int stage = k % STAGES;
      if (k % RING == RING / 2) {
        // rows for chunks [k - RING/2 + RING, ... + RING) into the other slot
        rows_finish(s, p, job, ((k / RING) + 1) & 1, lane);
        __syncwarp();
      } else if (k % RING == 0 && k > 0) {
        rows_start(job, s, p, begin + k + RING + lane, end);
      }
      bool ok = true;
      if (k >= STAGES) ok = mbar_wait_bounded(&s.empty[stage], (uint32_t)(((k / STAGES) - 1) & 1));
      if (!__all_sync(0xffffffffu, ok)) {
        record_error(p.err, kErrWaitTimeout);
        if (lane == 0) {
          atomicExch(&s.abort_, 1);
          // the last copy issued into each stage must land before the CTA exits
          for (int c = k - 1; c >= 0 && c >= k - STAGES; --c)
            mbar_wait_bounded(&s.full[c % STAGES], (uint32_t)((c / STAGES) & 1));
        }
        return;
      }
      if (lane == 0) issue(s, stage, k, &map);
      __syncwarp();
    }
    return;
  }

  // ================= consumer warps =================
  const int cw = warp;
  const int g = lane >> 2, tig = lane & 3;
  // ldmatrix row addresses for K k-step ks: subtile ks>>1 (2 KB each) of the
  // page, logical chunk 4*(ks&1) + (lane>>3), row lane&7 of the 8-token
  // n-tile; n-tile nt adds (nt>>1) pages and (nt&1) * 8 rows as immediates
  uint32_t koff[4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const uint32_t r = lane & 7, chunk = 4 * (ks & 1) + (lane >> 3);
    koff[ks] = (ks >> 1) * (SUB / 2) + r * 128 + (((chunk ^ r) & 7) << 4);
  }
  // V B-fragment words: token 16kt + 2tig + e (e in {0,1,8,9}) = page kt, row
  // 2tig + e; dim 8nt + g in subtile nt>>2.  voff[nt&3][e&1] is the lane part.
  uint32_t voff[4][2];
#pragma unroll
  for (int n4 = 0; n4 < 4; ++n4)
#pragma unroll
    for (int e1 = 0; e1 < 2; ++e1) {
      const uint32_t row = 2 * tig + e1, chunk = 2 * n4 + (g >> 2);
      voff[n4][e1] = PAGE_BYTES / 2 + row * 128 + (((chunk ^ row) & 7) << 4) + (g & 3) * 4;
    }

  // q fragments (A operand of S = Q K^T): rows g = hi, g+8 = lo of head g; the
  // k positions (2tig, 2tig+1, 2tig+8, 2tig+9) of k-step ks hold dims
  // 16ks + (tig, 4+tig, 8+tig, 12+tig), the order ldmatrix delivers K.
  auto load_q = [&](const Cursor& c, float (&x)[16]) {
    const float* qp = p.q + ((int64_t)c.b * H + c.kvh * GROUP + g) * HD;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
      for (int e = 0; e < 4; ++e) x[4 * ks + e] = __ldg(qp + 16 * ks + 4 * e + tig);
  };
  float qn[16];
  Cursor nxt;
  seek(nxt, s, p.batch, begin);
  load_q(nxt, qn);

  int i = begin;
  while (i < end) {
    const Cursor sg = nxt;
    const int pstart = i - sg.chunk;
    const int pend = pstart + sg.nchunks;
    const int seg_hi = min(end, pend);
    uint32_t qa[4][4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      split_bf16x2(qn[4 * ks] * p.qscale, qn[4 * ks + 1] * p.qscale, qa[ks][0], qa[ks][1]);
      split_bf16x2(qn[4 * ks + 2] * p.qscale, qn[4 * ks + 3] * p.qscale, qa[ks][2], qa[ks][3]);
    }
    if (seg_hi < end) {   // next segment's q loads fly while this one computes
      seek(nxt, s, p.batch, seg_hi);
      load_q(nxt, qn);
    }
    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) o[nt][j] = 0.f;
    float m = -INFINITY, l = 0.f;

    const int k0 = i - begin;
    const int kfirst = k0 + ((cw - k0 % NC) + NC) % NC;
    for (int k = kfirst; k < seg_hi - begin; k += NC) {
      const int stage = k % STAGES;
      const int nv = min(CHUNK, sg.len - (begin + k - pstart) * CHUNK);
      if (!s.abort_) {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s.full[stage], (uint32_t)((k / STAGES) & 1)))) {
          record_error(p.err, kErrWaitTimeout);
          if (lane == 0) atomicExch(&s.abort_, 1);
        }
      }
      const uint32_t sb = smem_u32(s.kv[stage]);

      // ---- pull the whole chunk into registers, then hand the stage back ----
      uint32_t kf[4][4][4];   // [ks][nt] ldmatrix.x4: K[8nt+g][16ks + {0,4,8,12} + tig]
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          ldsm_x4(sb + koff[ks] + (nt >> 1) * PAGE_BYTES + (nt & 1) * 1024, kf[ks][nt][0],
                  kf[ks][nt][1], kf[ks][nt][2], kf[ks][nt][3]);
      float vf[2][8][4];      // [kt][nt] V[16kt + 2tig + {0,1,8,9}][8nt + g]
#pragma unroll
      for (int kt = 0; kt < 2; ++kt)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const uint32_t a0 = sb + voff[nt & 3][0] + (nt >> 2) * (SUB / 2) + kt * PAGE_BYTES;
          const uint32_t a1 = sb + voff[nt & 3][1] + (nt >> 2) * (SUB / 2) + kt * PAGE_BYTES;
          vf[kt][nt][0] = lds32(a0);
          vf[kt][nt][1] = lds32(a1);
          vf[kt][nt][2] = lds32(a0 + 1024);
          vf[kt][nt][3] = lds32(a1 + 1024);
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[stage]);

      // ---- S = Q K^T for the chunk's 32 tokens (4 n-tiles of 8) ----
      float sc[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[nt][j] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          uint32_t bh0, bl0, bh1, bl1;
          split_bf16x2(__uint_as_float(kf[ks][nt][0]), __uint_as_float(kf[ks][nt][1]), bh0, bl0);
          split_bf16x2(__uint_as_float(kf[ks][nt][2]), __uint_as_float(kf[ks][nt][3]), bh1, bl1);
          mma_bf16(sc[nt], qa[ks], bh0, bh1);
          mma_bf16(sc[nt], qa[ks], bl0, bl1);
        }
      }
      // s[nt][j]: head g, token 8nt + 2tig + j
      float sv[4][2];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        sv[nt][0] = sc[nt][0] + sc[nt][2];
        sv[nt][1] = sc[nt][1] + sc[nt][3];
        if (nv < CHUNK) {
          if (8 * nt + 2 * tig >= nv) sv[nt][0] = -INFINITY;
          if (8 * nt + 2 * tig + 1 >= nv) sv[nt][1] = -INFINITY;
        }
      }
      // ---- online softmax (log2 domain: q carries scale * log2 e) ----
      float mx = sv[0][0];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) mx = fmaxf(mx, fmaxf(sv[nt][0], sv[nt][1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m, mx);
      const float al = exp2f(m - mn);
      float ps = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        sv[nt][0] = exp2f(sv[nt][0] - mn);
        sv[nt][1] = exp2f(sv[nt][1] - mn);
        ps += sv[nt][0] + sv[nt][1];
      }
      l = fmaf(l, al, ps);
      m = mn;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) o[nt][j] *= al;

      // ---- O += P V: k = tokens (2 k-steps of 16), n = dims (8 n-tiles) ----
#pragma unroll
      for (int kt = 0; kt < 2; ++kt) {
        if (16 * kt >= nv) break;
        uint32_t pa[4];
        split_bf16x2(sv[2 * kt][0], sv[2 * kt][1], pa[0], pa[1]);
        split_bf16x2(sv[2 * kt + 1][0], sv[2 * kt + 1][1], pa[2], pa[3]);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          float v0 = vf[kt][nt][0], v1 = vf[kt][nt][1], v2 = vf[kt][nt][2], v3 = vf[kt][nt][3];
          if (nv < CHUNK) {
            // tokens past the sequence end may hold anything: P is 0 there, V must be finite
            const int r = 16 * kt + 2 * tig;
            if (r >= nv) v0 = 0.f;
            if (r + 1 >= nv) v1 = 0.f;
            if (r + 8 >= nv) v2 = 0.f;
            if (r + 9 >= nv) v3 = 0.f;
          }
          uint32_t bh0, bl0, bh1, bl1;
          split_bf16x2(v0, v1, bh0, bl0);
          split_bf16x2(v2, v3, bh1, bl1);
          mma_bf16(o[nt], pa, bh0, bh1);
          mma_bf16(o[nt], pa, bl0, bl1);
        }
      }
    }

    i = seg_hi;
    if (kfirst >= seg_hi - begin) continue;   // this warp had no chunk in the segment

    // ---- publish this warp's partial (plain stores; counted at the end) ----
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int pair = sg.b * p.n_kv + sg.kvh;
    const int cfirst = pstart / W, clast = (pend - 1) / W;
    int contributors = 0;   // (CTA, warp) pairs that own at least one chunk of the segment
    for (int c = cfirst; c <= clast; ++c) {
      const int lo = max(pstart, c * W), hi = min(pend, (c + 1) * W);
      contributors += min(NC, hi - lo);
    }
    float* dst = p.out + ((int64_t)sg.b * H + sg.kvh * GROUP) * HD;
    if (contributors == 1) {
      const float inv = 1.0f / l;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
        *reinterpret_cast<float2*>(dst + g * HD + 8 * nt + 2 * tig) =
            make_float2((o[nt][0] + o[nt][2]) * inv, (o[nt][1] + o[nt][3]) * inv);
      continue;
    }
    const int64_t slot = ((int64_t)blockIdx.x + pair) * NC + cw;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
      __stcg(reinterpret_cast<float2*>(p.po + (slot * GROUP + g) * HD + 8 * nt + 2 * tig),
             make_float2(o[nt][0] + o[nt][2], o[nt][1] + o[nt][3]));
    if (tig == 0) __stcg(&p.ml[slot * GROUP + g], make_float2(m, l));
    // counting and merging wait until this warp has consumed all its chunks
  }

  // ---- after the last chunk: count in, and merge where this warp is last ----
  __threadfence();
  __syncwarp();
  for (int i2 = begin; i2 < end;) {
    Cursor sg;
    seek(sg, s, p.batch, i2);
    const int pstart = i2 - sg.chunk, pend = pstart + sg.nchunks, seg_hi = min(end, pend);
    const int k0 = i2 - begin;
    const int kfirst = k0 + ((cw - k0 % NC) + NC) % NC;
    i2 = seg_hi;
    if (kfirst >= seg_hi - begin) continue;
    const int cfirst = pstart / W, clast = (pend - 1) / W;
    int contributors = 0;
    for (int c = cfirst; c <= clast; ++c) {
      const int lo = max(pstart, c * W), hi = min(pend, (c + 1) * W);
      contributors += min(NC, hi - lo);
    }
    if (contributors == 1) continue;   // written directly
    const int pair = sg.b * p.n_kv + sg.kvh;
    int last = 0;
    if (lane == 0) {
      const int old = atomicAdd(&p.cnt[pair], 1);
      last = (old == contributors - 1);
      if (last) atomicExch(&p.cnt[pair], 0);
      __threadfence();
    }
    if (!__shfl_sync(0xffffffffu, last, 0)) continue;
    float* dst = p.out + ((int64_t)sg.b * H + sg.kvh * GROUP) * HD;
    // lane -> head lane>>2, dims 16*(lane&3) .. +15.  Contributors are the
    // warps (lo + q) % NC, q < min(NC, hi - lo), of each CTA c in
    // [cfirst, clast]; they are folded in one online pass with four partial
    // loads in flight at a time.
    const int mh = lane >> 2, md = 16 * (lane & 3);
    float M = -INFINITY, den = 0.f;
    float4 acc[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = cfirst; c <= clast; ++c) {
      const int lo = max(pstart, c * W) - c * W, hi = min(pend, (c + 1) * W) - c * W;
      const int nw = min(NC, hi - lo);
      for (int q0 = 0; q0 < nw; q0 += 4) {
        float2 mlv[4];
        float4 ov[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (q0 + u < nw) {
            const int64_t sl = ((int64_t)c + pair) * NC + ((lo + q0 + u) % NC);
            mlv[u] = __ldcg(&p.ml[sl * GROUP + mh]);
#pragma unroll
            for (int e = 0; e < 4; ++e) ov[u][e] = ld_cg4(p.po + (sl * GROUP + mh) * HD + md + 4 * e);
          } else {
            mlv[u] = make_float2(-INFINITY, 0.f);
#pragma unroll
            for (int e = 0; e < 4; ++e) ov[u][e] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (q0 + u >= nw) continue;
          const float Mn = fmaxf(M, mlv[u].x);
          const float sa = exp2f(M - Mn), sb = exp2f(mlv[u].x - Mn);
          den = den * sa + mlv[u].y * sb;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[e].x = fmaf(acc[e].x, sa, ov[u][e].x * sb);
            acc[e].y = fmaf(acc[e].y, sa, ov[u][e].y * sb);
            acc[e].z = fmaf(acc[e].z, sa, ov[u][e].z * sb);
            acc[e].w = fmaf(acc[e].w, sa, ov[u][e].w * sb);
          }
          M = Mn;
        }
      }
    }
    const float inv = 1.0f / den;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      *reinterpret_cast<float4*>(dst + mh * HD + md + 4 * e) =
          make_float4(acc[e].x * inv, acc[e].y * inv, acc[e].z * inv, acc[e].w * inv);
  }
}

size_t smem_bytes() { return sizeof(Smem) + 1024; }

struct WsLayout {
  size_t cnt, ml, po, total;
};

WsLayout ws_layout(int batch, int n_kv) {
  int b = batch < MAX_SEQS ? batch : MAX_SEQS;
  size_t pairs = (size_t)b * n_kv;
  size_t slots = (MAX_GRID + pairs) * NC;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  WsLayout w;
  w.cnt = 0;
  w.ml = al((size_t)MAX_SEQS * n_kv * sizeof(int32_t));   // counters: fixed size, see pages_workspace_bytes
  w.po = w.ml + al(slots * GROUP * sizeof(float2));
  w.total = w.po + al(slots * GROUP * HD * sizeof(float));
  if (n_kv == 4) {   // the whole-page kernel's layout (decode_pages.cu) is used instead
    const size_t pw = pages_workspace_bytes(batch);
    if (pw > w.total) w.total = pw;
  }
  return w;
}

int32_t launch(const Params& base, const CUtensorMap& map, int batch,
               const int32_t* seq_lens, const float* q, float* out, const int32_t* table,
               void* ws, cudaStream_t stream) {
  DeviceInfo* dev = nullptr;
  int32_t st = device_info(&dev);
  if (st) return st;
  const size_t smem = smem_bytes();
  int occ = 1;
  st = kernel_setup(reinterpret_cast<const void*>(decode_f32_kernel), smem, THREADS, &occ);
  if (st) return st;
  int grid = dev->num_sms * occ;
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
    decode_f32_kernel<<<grid, THREADS, smem, stream>>>(p, map);
    st = check_cuda(cudaGetLastError(), "decode_f32 launch");
    if (st) return st;
  }
  return NYION_OK;
}

// Pool: (x: 32 floats, slot row: 16 x 256 B, half: 2 x 128 B, K/V: 2 x 4096 B,
// block = page * n_kv + kv head: 8192 B); one box = one whole block.
int32_t pool_map(CUtensorMap* m, const float* pool, int64_t n_blocks) {
  const uint64_t dims[5] = {32, (uint64_t)PAGE, 2, 2, (uint64_t)n_blocks};
  const uint64_t strides[4] = {HD * 4, 128, PAGE * HD * 4, 2 * PAGE * HD * 4};
  const uint32_t box[5] = {32, (uint32_t)PAGE, 2, 2, 1};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, pool, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

bool specialised(int32_t n_heads, int32_t n_kv_heads, int32_t head_dim) {
  return head_dim == HD && n_kv_heads > 0 && n_heads == n_kv_heads * GROUP;
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

// ---- short contexts in the zone layout (ops::attention at <= 512 tokens) ----
// The executor's Full strategy runs up to 512 tokens and config 1 is 128: a
// one-launch kernel with no split-KV merge.  CTA = KV head, 256 threads.
// Scores: thread = token (its 256-byte K row in one batch of 16-byte loads,
// two rounds above 256 tokens), dots for the 8 query heads against q in shared
// memory.  Softmax: warp = head.  P.V: thread = (dim pair, token group), 32
// V loads in flight per round, the 8 groups summed through shared memory.
// With `importance` (ops::attention_tracked) each token's weights of the 8
// heads are added to importance[t] (double atomics: the 4 KV-head CTAs).
// Tokens < 4096 all sit in zone 0 (pages of 32 slots, [layer][kv head][slot]
// [64] per page).
constexpr int SMALL_TOK = 512;

template <int MAXT>
__global__ void __launch_bounds__(256) zoned_small_kernel(const float* __restrict__ q, const float* __restrict__ k_arena,
                                                          const float* __restrict__ v_arena, float* __restrict__ out,
                                                          double* __restrict__ importance, int n, int n_layers,
                                                          int layer, int n_kv, float sl2) {
  __shared__ float qs[GROUP][HD];
  __shared__ float ps[GROUP][MAXT];
  __shared__ float red[8][GROUP][HD];
  __shared__ float ls[GROUP];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int kvh = blockIdx.x, t = threadIdx.x, w = t >> 5, lane = t & 31;
  const int64_t lp = (int64_t)n_layers * n_kv;
  auto row = [&](int tok) { return ((int64_t)(tok >> 5) * lp * 32 + ((int64_t)layer * n_kv + kvh) * 32 + (tok & 31)) * HD; };
  // Up to 256 tokens every global load goes out at once: q, the K row of token
  // t and the V pairs of tokens 32 w .. 32 w + 31 (V does not depend on the scores).
  constexpr bool ONE_BATCH = MAXT <= 256;
  float4 kk0[HD / 4];
  float2 vv0[ONE_BATCH ? 32 : 1];
  if (ONE_BATCH) {
    const float q0 = q[(int64_t)kvh * GROUP * HD + t], q1 = q[(int64_t)kvh * GROUP * HD + t + 256];
    if (t < n) {
      const float4* kr = reinterpret_cast<const float4*>(k_arena + row(t));
#pragma unroll
      for (int c = 0; c < HD / 4; ++c) kk0[c] = __ldg(kr + c);
    }
#pragma unroll
    for (int u = 0; u < (ONE_BATCH ? 32 : 1); ++u) {
      const int j = 32 * w + u;
      vv0[u] = j < n ? __ldg(reinterpret_cast<const float2*>(v_arena + row(j)) + lane) : make_float2(0.f, 0.f);
    }
    qs[t / HD][t % HD] = q0 * sl2;
    qs[(t + 256) / HD][(t + 256) % HD] = q1 * sl2;
  } else {
    for (int i = t; i < GROUP * HD; i += 256) qs[i / HD][i % HD] = q[(int64_t)kvh * GROUP * HD + i] * sl2;
  }
  __syncthreads();
  for (int tok = t; tok < MAXT; tok += 256) {
    float acc[GROUP];
#pragma unroll
    for (int h = 0; h < GROUP; ++h) acc[h] = 0.f;
    if (tok < n) {
      float4 kk[HD / 4];
      if (ONE_BATCH) {
#pragma unroll
        for (int c = 0; c < HD / 4; ++c) kk[c] = kk0[c];
      } else {
        const float4* kr = reinterpret_cast<const float4*>(k_arena + row(tok));
#pragma unroll
        for (int c = 0; c < HD / 4; ++c) kk[c] = __ldg(kr + c);
      }
#pragma unroll
      for (int c = 0; c < HD / 4; ++c)
#pragma unroll
        for (int h = 0; h < GROUP; ++h) {
          const float* qq = &qs[h][4 * c];
          acc[h] = fmaf(qq[0], kk[c].x, fmaf(qq[1], kk[c].y, fmaf(qq[2], kk[c].z, fmaf(qq[3], kk[c].w, acc[h]))));
        }
    }
#pragma unroll
    for (int h = 0; h < GROUP; ++h) ps[h][tok] = tok < n ? acc[h] : -INFINITY;
  }
  __syncthreads();
  {
    float mx = -INFINITY;
    for (int j = lane; j < MAXT; j += 32) mx = fmaxf(mx, ps[w][j]);
    mx = warp_max(mx);
    float l = 0.f;
    for (int j = lane; j < MAXT; j += 32) {
      const float pe = exp2f(ps[w][j] - mx);
      ps[w][j] = pe;
      l += pe;
    }
    l = warp_sum(l);
    if (lane == 0) ls[w] = l;
  }
  __syncthreads();
  if (importance) {
    for (int tok = t; tok < n; tok += 256) {
      double a = 0.0;
#pragma unroll
      for (int h = 0; h < GROUP; ++h) a += (double)(ps[h][tok] * (1.0f / ls[h]));
      atomicAdd(importance + tok, a);
    }
  }
  {
    const int dp = lane, tg = w;                      // dims 2dp, 2dp+1; tokens tg * n_per .. + n_per
    const int n_per = MAXT <= 256 ? 32 : (n + 7) / 8;
    float2 acc[GROUP];
#pragma unroll
    for (int h = 0; h < GROUP; ++h) acc[h] = make_float2(0.f, 0.f);
    for (int u0 = 0; u0 < n_per; u0 += 32) {
      float2 vv[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int j = tg * n_per + u0 + u;
        if (ONE_BATCH)
          vv[u] = vv0[ONE_BATCH ? u : 0];   // n_per = 32: loaded at the start
        else
          vv[u] = (u0 + u < n_per && j < n) ? __ldg(reinterpret_cast<const float2*>(v_arena + row(j)) + dp)
                                            : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int j = tg * n_per + u0 + u;
        if (u0 + u < n_per && j < n) {
#pragma unroll
          for (int h = 0; h < GROUP; ++h) {
            const float pe = ps[h][j];
            acc[h].x = fmaf(pe, vv[u].x, acc[h].x);
            acc[h].y = fmaf(pe, vv[u].y, acc[h].y);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      red[tg][h][2 * dp] = acc[h].x;
      red[tg][h][2 * dp + 1] = acc[h].y;
    }
  }
  __syncthreads();
  for (int i = t; i < GROUP * HD; i += 256) {
    const int h = i / HD, d = i % HD;
    float o = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) o += red[g][h][d];
    out[((int64_t)kvh * GROUP + h) * HD + d] = o / ls[h];
  }
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
  if (!specialised(n_heads, n_kv_heads, head_dim) && generic_shape_ok(n_heads, n_kv_heads, head_dim)) {
    // other shapes: the generic kernel (library-owned workspace)
    if (!q || !kv_pool || !page_table || !seq_lens || !out)
      return fail(NYION_ERR_INVALID, "decode_paged_f32: null pointer argument");
    if (batch <= 0 || max_pages <= 0 || n_pool_pages <= 0)
      return fail(NYION_ERR_INVALID, "decode_paged_f32: batch, max_pages and n_pool_pages must be > 0");
    if (page_tokens != PAGE)
      return fail(NYION_ERR_UNSUPPORTED, "decode_paged_f32: page_tokens must be 16 (got %d)", page_tokens);
    GenericCall c;
    c.who = "decode_paged_f32";
    c.q = q;
    c.k = kv_pool;
    c.table = page_table;
    c.max_pages = max_pages;
    c.n_pool_pages = n_pool_pages;
    c.n_heads = n_heads;
    c.n_kv = n_kv_heads;
    c.head_dim = head_dim;
    c.rows = batch;
    c.lens = seq_lens;
    c.scale = scale;
    c.out = out;
    c.max_tokens = (int64_t)max_pages * PAGE;
    c.fmt = kGenF32;
    c.layout = kGenPaged;
    return generic_decode(c, static_cast<cudaStream_t>(stream));
  }
  int32_t st = check_common(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!q || !kv_pool || !page_table || !seq_lens || !out)
    return fail(NYION_ERR_INVALID, "decode_paged_f32: null pointer argument");
  if (batch <= 0 || max_pages <= 0 || n_pool_pages <= 0)
    return fail(NYION_ERR_INVALID, "decode_paged_f32: batch, max_pages and n_pool_pages must be > 0");
  if (page_tokens != PAGE)
    return fail(NYION_ERR_UNSUPPORTED, "decode_paged_f32: page_tokens must be 16 (got %d)", page_tokens);
  uint64_t rows = (uint64_t)n_pool_pages * n_kv_heads;   // (page, kv head) blocks
  if (rows > (1ull << 31))
    return fail(NYION_ERR_INVALID, "decode_paged_f32: pool of %lld pages exceeds 2^31 rows",
                (long long)n_pool_pages);
  size_t need = ws_layout(batch, n_kv_heads).total;
  if (!workspace) {
    st = internal_workspace(need, &workspace, kWsCounters, ws_layout(batch, n_kv_heads).ml,
                            static_cast<cudaStream_t>(stream));
    if (st) return st;
  } else if (workspace_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "decode_paged_f32: workspace %zu < %zu bytes", workspace_bytes, need);
  }
  const float qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  // 4 KV heads: a page is one 32 KB block, streamed whole (decode_pages.cu)
  if (n_kv_heads == 4)
    return launch_pages(q, kv_pool, n_pool_pages, page_table, max_pages, seq_lens, out, batch, qscale,
                        workspace, static_cast<cudaStream_t>(stream));
  CUtensorMap map;
  st = pool_map(&map, kv_pool, n_pool_pages * n_kv_heads);
  if (st) return st;
  Params p{};
  p.n_kv = n_kv_heads;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.qscale = qscale;
  return launch(p, map, batch, seq_lens, q, out, page_table, workspace,
                       static_cast<cudaStream_t>(stream));
}

namespace nyion {
int64_t zoned_small_max() { return f32dec::SMALL_TOK; }

int32_t zoned_small(float* out, const float* q, const float* k_arena, const float* v_arena, int64_t n_arena_pages,
                    int32_t n_layers, int32_t layer_idx, int64_t n_tokens, int32_t n_kv_heads, int32_t head_dim,
                    double* importance, void* stream) {
  const int64_t pages = (n_tokens + 31) / 32;
  if (pages > n_arena_pages)
    return fail(NYION_ERR_INVALID, "decode_zoned_f32: %lld tokens need %lld pages, the arena has %lld",
                (long long)n_tokens, (long long)pages, (long long)n_arena_pages);
  const float sl2 = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  auto kern = n_tokens <= 256 ? f32dec::zoned_small_kernel<256> : f32dec::zoned_small_kernel<f32dec::SMALL_TOK>;
  return check_cuda(launch_pdl(kern, dim3((unsigned)n_kv_heads), dim3(256), 0, static_cast<cudaStream_t>(stream), q,
                               k_arena, v_arena, out, importance, (int)n_tokens, (int)n_layers, (int)layer_idx,
                               (int)n_kv_heads, sl2),
                    "decode_zoned_f32 short-context launch");
}
}  // namespace nyion

extern "C" int32_t nyion_attn_decode_zoned_f32(float* out, const float* q, const float* k_arena,
                                               const float* v_arena, int64_t n_arena_pages,
                                               int32_t n_layers, int32_t layer_idx,
                                               int64_t seq_len, int64_t q_pos, int32_t n_heads,
                                               int32_t n_kv_heads, int32_t head_dim,
                                               void* stream) {
  const bool generic = !specialised(n_heads, n_kv_heads, head_dim) && generic_shape_ok(n_heads, n_kv_heads, head_dim);
  int32_t st = generic ? NYION_OK : check_common(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!out || !q || !k_arena || !v_arena)
    return fail(NYION_ERR_INVALID, "decode_zoned_f32: null pointer argument");
  if (seq_len <= 0 || q_pos < 0 || n_layers <= 0 || layer_idx < 0 || layer_idx >= n_layers ||
      n_arena_pages <= 0)
    return fail(NYION_ERR_INVALID, "decode_zoned_f32: bad seq_len/q_pos/layer/arena arguments");
  // ops.rs:183 valid_end = min(q_pos, seq_len - 1): tokens [0, valid_end] are attended
  int64_t valid_end = q_pos < seq_len - 1 ? q_pos : seq_len - 1;
  if (valid_end + 1 > (1ll << 30)) return fail(NYION_ERR_INVALID, "decode_zoned_f32: context too long");
  if (generic) {
    GenericCall c;
    c.who = "decode_zoned_f32";
    c.q = q;
    c.k = k_arena;
    c.v = v_arena;
    c.n_heads = n_heads;
    c.n_kv = n_kv_heads;
    c.head_dim = head_dim;
    c.rows = 1;
    c.u_begin = 0;
    c.u_end = (int32_t)(valid_end + 1);
    c.n_layers = n_layers;
    c.layer = layer_idx;
    c.n_pages = n_arena_pages;
    c.out = out;
    c.max_tokens = valid_end + 1;
    c.fmt = kGenF32;
    c.layout = kGenZoned;
    return generic_decode(c, static_cast<cudaStream_t>(stream));
  }
  if (valid_end + 1 <= zoned_small_max())
    return zoned_small(out, q, k_arena, v_arena, n_arena_pages, n_layers, layer_idx, valid_end + 1, n_kv_heads,
                       head_dim, nullptr, stream);
  const float sl2 = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  return contig_zoned_f32(q, k_arena, v_arena, out, n_kv_heads, n_layers, layer_idx, n_arena_pages,
                          (int)(valid_end + 1), sl2, nullptr, 0, static_cast<cudaStream_t>(stream));
}

// ---- reference CUDA C ABI (swamp-gpu/kernels/fused_attention.cu) -------------

static int32_t contig_decode(const float* d_q, const float* d_k, const float* d_v, float* d_out,
                             int n_heads, int n_kv_heads, int seq_len, int head_dim, int kv_stride,
                             void* ws, cudaStream_t stream) {
  const bool generic = !specialised(n_heads, n_kv_heads, head_dim) && generic_shape_ok(n_heads, n_kv_heads, head_dim);
  int32_t st = generic ? NYION_OK : check_common(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!d_q || !d_k || !d_v || !d_out) return fail(NYION_ERR_INVALID, "null pointer argument");
  if (seq_len <= 0 || kv_stride < seq_len)
    return fail(NYION_ERR_INVALID, "seq_len %d must be in [1, kv_stride=%d]", seq_len, kv_stride);
  if (generic) {
    GenericCall c;
    c.who = "gpu_attention";
    c.q = d_q;
    c.k = d_k;
    c.v = d_v;
    c.n_heads = n_heads;
    c.n_kv = n_kv_heads;
    c.head_dim = head_dim;
    c.rows = 1;
    c.u_begin = 0;
    c.u_end = seq_len;
    c.stride = kv_stride;
    c.out = d_out;
    c.max_tokens = seq_len;
    c.fmt = kGenF32;
    c.layout = kGenRows;
    return generic_decode(c, stream);
  }
  const float sl2 = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  return contig_rows_f32(d_q, d_k, d_v, d_out, n_kv_heads, kv_stride, seq_len, sl2, ws,
                         ws ? contig_workspace_bytes(n_kv_heads, seq_len) : 0, stream);
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

extern "C" void* gpu_graph_create_attention(const float* d_q, const float* d_k_cache,
                                            const float* d_v_cache, float* d_scores,
                                            float* d_output, int n_heads, int n_kv_heads,
                                            int seq_len, int head_dim, int kv_stride) {
  (void)d_scores;
  DeviceInfo* dev = nullptr;
  if (device_info(&dev)) return nullptr;
  const size_t wsb = contig_workspace_bytes(n_kv_heads > 0 ? n_kv_heads : 1, seq_len);
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

// ---- allocation-free variant of the paged fp32 decode -----------------------
//
// For callers that cannot allocate device memory at decode time: a
// latency-critical serving loop that must never hit cudaFree's implicit device
// synchronisation, a host whose HBM is entirely handed out by its own arena so
// an extra cudaMalloc would fail or fragment it, or a plugin host whose rules
// forbid a library from allocating behind its back.  The split-KV scratch (merge counters and log-sum-exp partials) lives
// in one file-scope device array instead, sized kNoAllocScratchBytes; every
// GPU that loads this library reserves it until the process exits.
//
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress (and sets the kernel's shared-memory attribute); make
// that first call before any stream capture.  All calls on a device share the
// one array, so calls that overlap on the GPU (for example on different
// streams) race and corrupt each other's partials: serialise
// them.  The merge counters are cleared at the start of every call.
// Device-side page-id range errors of this variant go to its own error word,
// a second file-scope device variable; nyion_attn_device_error reads and
// clears it together with the shared word, and allocates nothing when only
// this entry point has run on the device.  The cached addresses belong to the
// CUDA context that resolved them: after cudaDeviceReset the library (this
// entry point included) must not be used again in the process.
namespace nyion {
namespace f32dec {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;   // 8 MiB per device
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ int32_t g_noalloc_err;

struct NoAllocDevice {
  bool ready = false;
  uint8_t* scratch = nullptr;   // device address of g_noalloc_scratch
  int32_t* err = nullptr;       // device address of g_noalloc_err
  int grid = 0;
  int sms = 0;
};
static NoAllocDevice g_noalloc_dev[64];
static std::mutex g_noalloc_mu;

static int32_t noalloc_setup(NoAllocDevice** out) {
  int dev = -1;
  int32_t st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  if (dev < 0 || dev >= 64) return fail(NYION_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    void* sp = nullptr;
    void* ep = nullptr;
    st = check_cuda(cudaGetSymbolAddress(&sp, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
    if (st) return st;
    st = check_cuda(cudaGetSymbolAddress(&ep, g_noalloc_err), "cudaGetSymbolAddress(error word)");
    if (st) return st;
    int sms = 0, major = 0;
    st = check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
    if (st) return st;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (major != 10) return fail(NYION_ERR_UNSUPPORTED, "device %d is not sm_100a", dev);
    int occ = 1;
    st = kernel_setup(reinterpret_cast<const void*>(decode_f32_kernel), smem_bytes(), THREADS, &occ);
    if (st) return st;
    d.scratch = static_cast<uint8_t*>(sp);
    d.err = static_cast<int32_t*>(ep);
    d.grid = sms * (occ > 0 ? occ : 1);
    if (d.grid > MAX_GRID) d.grid = MAX_GRID;
    d.sms = sms;
    d.ready = true;
  }
  *out = &d;
  return NYION_OK;
}

}  // namespace f32dec

int32_t* noalloc_error_word_if_ready() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(f32dec::g_noalloc_mu);
  return f32dec::g_noalloc_dev[dev].ready ? f32dec::g_noalloc_dev[dev].err : nullptr;
}

}  // namespace nyion

extern "C" int32_t nyion_attn_decode_paged_f32_noalloc(
    const float* q, const float* kv_pool, int64_t n_pool_pages, const int32_t* page_table,
    int32_t max_pages, const int32_t* seq_lens, float* out, int32_t batch, int32_t n_heads,
    int32_t n_kv_heads, int32_t head_dim, int32_t page_tokens, float scale, void* stream) {
  int32_t st = check_common(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!q || !kv_pool || !page_table || !seq_lens || !out)
    return fail(NYION_ERR_INVALID, "decode_paged_f32_noalloc: null pointer argument");
  if (batch <= 0 || max_pages <= 0 || n_pool_pages <= 0)
    return fail(NYION_ERR_INVALID, "decode_paged_f32_noalloc: batch, max_pages and n_pool_pages must be > 0");
  if (page_tokens != PAGE)
    return fail(NYION_ERR_UNSUPPORTED, "decode_paged_f32_noalloc: page_tokens must be 16 (got %d)", page_tokens);
  if (batch > MAX_SEQS)
    return fail(NYION_ERR_INVALID, "decode_paged_f32_noalloc: batch %d exceeds %d sequences per call",
                batch, MAX_SEQS);
  if ((uint64_t)n_pool_pages * n_kv_heads > (1ull << 31))
    return fail(NYION_ERR_INVALID, "decode_paged_f32_noalloc: pool too large");
  NoAllocDevice* d = nullptr;
  st = noalloc_setup(&d);
  if (st) return st;
  cudaStream_t s0 = static_cast<cudaStream_t>(stream);
  if (n_kv_heads == 4 && pages_workspace_bytes(batch) <= kNoAllocScratchBytes) {
    // 4 KV heads: the whole-page kernel on the static scratch, counters cleared first
    st = check_cuda(cudaMemsetAsync(d->scratch, 0, pages_counter_bytes(), s0), "clear merge counters");
    if (st) return st;
    const float qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
    return launch_pages(q, kv_pool, n_pool_pages, page_table, max_pages, seq_lens, out, batch, qscale, d->scratch,
                        s0, d->err, d->sms);
  }
  // scratch layout for this launch: counters | (m, l) partials | o partials
  const size_t pairs = (size_t)batch * n_kv_heads;
  const size_t slots = ((size_t)d->grid + pairs) * NC;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t off_ml = al(pairs * sizeof(int32_t));
  const size_t off_po = off_ml + al(slots * GROUP * sizeof(float2));
  const size_t need = off_po + slots * GROUP * HD * sizeof(float);
  if (need > kNoAllocScratchBytes)
    return fail(NYION_ERR_WORKSPACE,
                "decode_paged_f32_noalloc: %d sequences x %d KV heads need %zu bytes of scratch; "
                "the static scratch holds %zu (use nyion_attn_decode_paged_f32 with a workspace)",
                batch, n_kv_heads, need, kNoAllocScratchBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = check_cuda(cudaMemsetAsync(d->scratch, 0, pairs * sizeof(int32_t), s), "clear merge counters");
  if (st) return st;
  CUtensorMap map;
  st = pool_map(&map, kv_pool, n_pool_pages * n_kv_heads);
  if (st) return st;
  Params p{};
  p.q = q;
  p.out = out;
  p.table = page_table;
  p.seq_lens = seq_lens;
  p.batch = batch;
  p.n_kv = n_kv_heads;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  p.cnt = reinterpret_cast<int32_t*>(d->scratch);
  p.ml = reinterpret_cast<float2*>(d->scratch + off_ml);
  p.po = reinterpret_cast<float*>(d->scratch + off_po);
  p.err = d->err;
  decode_f32_kernel<<<d->grid, THREADS, smem_bytes(), s>>>(p, map);
  return check_cuda(cudaGetLastError(), "decode_f32_noalloc launch");
}
