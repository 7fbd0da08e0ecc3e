// decode_pages.cu — batched fp32 paged decode, streaming whole pages.
//
// Same maths as decode_f32.cu (ops::attention, swamp-engine/src/ops.rs:170-278,
// over a 16-token page table), organised around the HBM access pattern: a
// page of the pool holds all 4 KV heads (4 x 8 KB, contiguous), and reading
// each page in one piece sustains ~97% of the measured copy bandwidth where
// 8 KB slices of pages read at different times reach ~85%.  So:
//
//   * unit of work = (sequence, page): 16 tokens x 4 KV heads = 32 KB, copied
//     by ONE 5-D TMA box (x 32 floats, token 16, 128-B half 2, K/V 2, KV head 4)
//     into a 6-stage ring; units flattened over the batch and cut into equal
//     contiguous ranges, one persistent CTA per SM;
//   * 8 consumer warps = 4 KV heads x 2 page parities: warp (kvh, par) takes
//     the units k = par, par + 2, ... of its CTA and reads only its head's
//     8 KB block; with an even ring depth every stage is always consumed by
//     the same four warps, so each warp sees each stage's phases in order;
//   * per unit: S = Q K^T and O += P V on mma.sync bf16 with fp32 operands
//     split hi + lo (all four cross products; ~2^-17 relative residual),
//     online softmax in the log2 domain;
//   * at each sequence boundary the two parity warps of a KV head fold their
//     partials in shared memory; a sequence held by one CTA is written there,
//     otherwise each CTA leaves one (m, l, o) partial and a counter lets the
//     last CTA's two warps merge them, all loads in flight together (no
//     inter-CTA wait).
#include <math.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace pages {

constexpr int HD = 64;
constexpr int GROUP = 8;
constexpr int PAGE = 16;
constexpr int NKV = 4;                       // KV heads per page (this kernel's geometry)
constexpr int NCW = 2 * NKV;                 // consumer warps
constexpr int STAGES = 6;
static_assert(STAGES % 2 == 0, "a stage must always belong to one page parity");
constexpr int THREADS = (NCW + 1) * 32;
constexpr int BLOCK = 8192;                  // one KV head of a page: K 0-31 | K 32-63 | V 0-31 | V 32-63
constexpr int STAGE_BYTES = NKV * BLOCK;
constexpr int MAX_SEQS = 512;
constexpr int MAX_GRID = 296;          // one CTA per SM on B200 (148), with room

struct Params {
  const float* q;           // [batch][32][64]
  float* out;               // [batch][32][64]
  const int32_t* table;     // [batch][max_pages]
  const int32_t* seq_lens;  // [batch]
  int32_t batch, max_pages;
  int64_t n_pool_pages;
  float qscale;             // scale * log2(e)
  int32_t* cnt;             // [batch * NKV] merge counters (start at 0, left at 0)
  float2* ml;               // [(MAX_GRID + batch) * NKV][GROUP] (m, l) per CTA partial
  float* po;                // [(MAX_GRID + batch) * NKV][GROUP][HD] o relative to m
  int32_t* err;
};

// per KV head: the parity-1 warp's partial handed to the parity-0 warp
struct Xch {
  float o[GROUP][HD];
  float2 ml[GROUP];
  int32_t flag;
};

struct Smem {
  uint8_t kv[STAGES][STAGE_BYTES];   // first member: 1024-byte aligned
  uint64_t full[STAGES];
  uint64_t empty[STAGES];            // 4 arrivals: the parity's KV-head warps
  int32_t prefix[MAX_SEQS + 1];      // flat unit index where sequence b starts
  int32_t lens[MAX_SEQS];
  int32_t warp_tot[THREADS / 32];
  Xch xch[NKV];
  int32_t abort_;
};

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ int pages_of(int len) { return (len + PAGE - 1) / PAGE; }

// sequence holding flat unit u (prefix[b] <= u < prefix[b + 1])
__device__ __forceinline__ int seq_of(const Smem& s, int batch, int u) {
  int lo = 0, hi = batch;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s.prefix[mid] <= u) lo = mid; else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(THREADS, 1)
decode_pages_kernel(const Params p, const __grid_constant__ CUtensorMap map) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  constexpr int H = NKV * GROUP;

  if (t == 0) {
    prefetch_tensormap(&map);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], NKV);
    }
    s.abort_ = 0;
    fence_barrier_init();
  }
  // programmatic dependent launch: the next grid in the stream may be
  // scheduled now; nothing global is read before the previous grid completed
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- sequence lengths and flat page prefix (block scan) ----
  for (int b = t; b < p.batch; b += THREADS) {
    const int L = p.seq_lens[b];
    s.lens[b] = L > 0 ? L : 0;
  }
  __syncthreads();
  constexpr int PER = (MAX_SEQS + THREADS - 1) / THREADS;
  int local[PER];
  int run = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int b = t * PER + j;
    const int c = (b < p.batch) ? pages_of(s.lens[b]) : 0;
    local[j] = run;
    run += c;
  }
  int incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s.warp_tot[warp] = incl;
  __syncthreads();
  int woff = 0;
  for (int w = 0; w < warp; ++w) woff += s.warp_tot[w];
  const int excl = woff + incl - run;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int b = t * PER + j;
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

  if (warp == NCW) {
    // ================= producer warp =================
    // lane l holds the block coordinate (page * 4) of units begin + 32 r + l,
    // one block of 32 loaded ahead; -4 (all out of range) zero-fills a bad page
    auto coord = [&](int u) -> int32_t {
      if (u >= end) return -NKV;
      const int b = seq_of(s, p.batch, u);
      const int pi = u - s.prefix[b];
      const int64_t page = pi < p.max_pages ? p.table[(int64_t)b * p.max_pages + pi] : -1;
      if (page < 0 || page >= p.n_pool_pages) {
        record_error(p.err, kErrPageRange);
        return -NKV;
      }
      return (int32_t)(page * NKV);
    };
    int32_t cur = coord(begin + lane);
    int32_t nxt = coord(begin + 32 + lane);
    for (int k = 0; k < n; ++k) {
      if ((k & 31) == 0 && k > 0) {
        cur = nxt;
        nxt = coord(begin + k + 32 + lane);
      }
      const int32_t c4 = __shfl_sync(0xffffffffu, cur, k & 31);
      const int stage = k % STAGES;
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
      if (lane == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&s.full[stage], STAGE_BYTES);
        tma_load_5d(s.kv[stage], &map, 0, 0, 0, 0, c4, &s.full[stage]);
      }
      __syncwarp();
    }
    return;
  }

  // ================= consumer warps =================
  const int kvh = warp & (NKV - 1), par = warp / NKV;
  const int g = lane >> 2, tig = lane & 3;
  // ldmatrix row addresses for K k-step ks: 128-B half ks>>1 (2 KB each),
  // logical chunk 4*(ks&1) + (lane>>3), row lane&7 of the 8-token n-tile;
  // n-tile nt adds nt * 8 rows (1 KB)
  uint32_t koff[4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const uint32_t r = lane & 7, chunk = 4 * (ks & 1) + (lane >> 3);
    koff[ks] = (ks >> 1) * 2048 + r * 128 + (((chunk ^ r) & 7) << 4);
  }
  // V B-fragment words: token 2tig + e (e in {0,1,8,9}), dim 8nt + g in the
  // 128-B half nt>>2.  voff[nt&3][e&1] is the lane part.
  uint32_t voff[4][2];
#pragma unroll
  for (int n4 = 0; n4 < 4; ++n4)
#pragma unroll
    for (int e1 = 0; e1 < 2; ++e1) {
      const uint32_t row = 2 * tig + e1, chunk = 2 * n4 + (g >> 2);
      voff[n4][e1] = BLOCK / 2 + row * 128 + (((chunk ^ row) & 7) << 4) + (g & 3) * 4;
    }
  const uint32_t head_base = (uint32_t)kvh * BLOCK;

  // q fragments (A operand): rows g = hi, g+8 = lo of head g; k positions
  // (2tig, 2tig+1, 2tig+8, 2tig+9) of k-step ks hold dims 16ks + (tig, 4+tig,
  // 8+tig, 12+tig), the order ldmatrix delivers K
  auto load_q = [&](int b, float (&x)[16]) {
    const float* qp = p.q + ((int64_t)b * H + kvh * GROUP + g) * HD;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
#pragma unroll
      for (int e = 0; e < 4; ++e) x[4 * ks + e] = __ldg(qp + 16 * ks + 4 * e + tig);
  };
  float qn[16];
  int nb = seq_of(s, p.batch, begin);
  load_q(nb, qn);

  int i = begin;
  while (i < end) {
    const int b = nb;
    const int pstart = s.prefix[b], pend = s.prefix[b + 1];
    const int seg_hi = min(end, pend);
    const int len = s.lens[b];
    uint32_t qa[4][4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      split_bf16x2(qn[4 * ks] * p.qscale, qn[4 * ks + 1] * p.qscale, qa[ks][0], qa[ks][1]);
      split_bf16x2(qn[4 * ks + 2] * p.qscale, qn[4 * ks + 3] * p.qscale, qa[ks][2], qa[ks][3]);
    }
    if (seg_hi < end) {   // the next sequence's q loads fly while this one computes
      nb = seq_of(s, p.batch, seg_hi);
      load_q(nb, qn);
    }
    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) o[nt][j] = 0.f;
    float m = -INFINITY, l = 0.f;

    const int k0 = i - begin;
    const int kfirst = k0 + ((par - k0) & 1);
    for (int k = kfirst; k < seg_hi - begin; k += 2) {
      const int stage = k % STAGES;
      const int nv = min(PAGE, len - (begin + k - pstart) * PAGE);
      if (!s.abort_) {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s.full[stage], (uint32_t)((k / STAGES) & 1)))) {
          record_error(p.err, kErrWaitTimeout);
          if (lane == 0) atomicExch(&s.abort_, 1);
        }
      }
      const uint32_t sb = smem_u32(s.kv[stage]) + head_base;

      // ---- pull this head's 16 tokens into registers, then release ----
      uint32_t kf[4][2][4];   // [ks][nt] ldmatrix.x4: K[8nt+g][16ks + {0,4,8,12} + tig]
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          ldsm_x4(sb + koff[ks] + nt * 1024, kf[ks][nt][0], kf[ks][nt][1], kf[ks][nt][2], kf[ks][nt][3]);
      float vf[8][4];         // [nt] V[2tig + {0,1,8,9}][8nt + g]
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const uint32_t a0 = sb + voff[nt & 3][0] + (nt >> 2) * 2048;
        const uint32_t a1 = sb + voff[nt & 3][1] + (nt >> 2) * 2048;
        vf[nt][0] = lds32(a0);
        vf[nt][1] = lds32(a1);
        vf[nt][2] = lds32(a0 + 1024);
        vf[nt][3] = lds32(a1 + 1024);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[stage]);

      // ---- S = Q K^T for the page's 16 tokens (2 n-tiles of 8) ----
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[nt][j] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          uint32_t bh0, bl0, bh1, bl1;
          split_bf16x2(__uint_as_float(kf[ks][nt][0]), __uint_as_float(kf[ks][nt][1]), bh0, bl0);
          split_bf16x2(__uint_as_float(kf[ks][nt][2]), __uint_as_float(kf[ks][nt][3]), bh1, bl1);
          mma_bf16(sc[nt], qa[ks], bh0, bh1);
          mma_bf16(sc[nt], qa[ks], bl0, bl1);
        }
      }
      // sv[nt][j]: head g, token 8nt + 2tig + j
      float sv[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        sv[nt][0] = sc[nt][0] + sc[nt][2];
        sv[nt][1] = sc[nt][1] + sc[nt][3];
        if (nv < PAGE) {
          if (8 * nt + 2 * tig >= nv) sv[nt][0] = -INFINITY;
          if (8 * nt + 2 * tig + 1 >= nv) sv[nt][1] = -INFINITY;
        }
      }
      // ---- online softmax (log2 domain: q carries scale * log2 e) ----
      float mx = fmaxf(fmaxf(sv[0][0], sv[0][1]), fmaxf(sv[1][0], sv[1][1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m, mx);
      const float al = exp2f(m - mn);
      float ps = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
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

      // ---- O += P V: k = the 16 tokens, n = dims (8 n-tiles) ----
      uint32_t pa[4];
      split_bf16x2(sv[0][0], sv[0][1], pa[0], pa[1]);
      split_bf16x2(sv[1][0], sv[1][1], pa[2], pa[3]);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        float v0 = vf[nt][0], v1 = vf[nt][1], v2 = vf[nt][2], v3 = vf[nt][3];
        if (nv < PAGE) {
          // slots past the sequence end may hold anything: P is 0 there, V must be finite
          const int r = 2 * tig;
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

    i = seg_hi;

    // ---- fold the two parity warps' partials of (b, kvh) in shared memory ----
    // (a warp without a page of b here contributes l = 0); the parity-0 warp
    // then writes the result, or publishes one partial per CTA when other
    // CTAs hold pages of b too
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    Xch& xc = s.xch[kvh];
    if (par == 1) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
        *reinterpret_cast<float2*>(&xc.o[g][8 * nt + 2 * tig]) =
            make_float2(o[nt][0] + o[nt][2], o[nt][1] + o[nt][3]);
      if (tig == 0) xc.ml[g] = make_float2(m, l);
    }
    named_bar_sync(1 + kvh, 64);
    if (par == 0) {
      const float2 ml1 = xc.ml[g];
      const float M = fmaxf(m, ml1.x);                // finite: one of the two owns a page
      const float a0 = l > 0.f ? exp2f(m - M) : 0.f, a1 = ml1.y > 0.f ? exp2f(ml1.x - M) : 0.f;
      const float L = l * a0 + ml1.y * a1;
      const int cfirst = pstart / W, clast = (pend - 1) / W;
      if (cfirst == clast) {                          // every page of b is in this CTA
        const float inv = 1.0f / L;
        float* dst = p.out + ((int64_t)b * H + kvh * GROUP + g) * HD;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const float2 o1 = *reinterpret_cast<const float2*>(&xc.o[g][8 * nt + 2 * tig]);
          *reinterpret_cast<float2*>(dst + 8 * nt + 2 * tig) =
              make_float2(((o[nt][0] + o[nt][2]) * a0 + o1.x * a1) * inv,
                          ((o[nt][1] + o[nt][3]) * a0 + o1.y * a1) * inv);
        }
      } else {
        const int64_t slot = ((int64_t)blockIdx.x + b) * NKV + kvh;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const float2 o1 = *reinterpret_cast<const float2*>(&xc.o[g][8 * nt + 2 * tig]);
          __stcg(reinterpret_cast<float2*>(p.po + (slot * GROUP + g) * HD + 8 * nt + 2 * tig),
                 make_float2((o[nt][0] + o[nt][2]) * a0 + o1.x * a1, (o[nt][1] + o[nt][3]) * a0 + o1.y * a1));
        }
        if (tig == 0) __stcg(&p.ml[slot * GROUP + g], make_float2(M, L));
      }
    }
    named_bar_sync(1 + kvh, 64);                      // the exchange buffer is free again
  }

  // ---- after the last unit: the parity-0 warp of each KV head counts the CTA
  // in for the (at most two) sequences it shares with other CTAs; where the
  // CTA is last, both warps of the head merge the CTA partials (heads 4 par ..
  // 4 par + 3) with every partial's loads in flight together.  The named
  // barrier just passed orders both warps' partial stores before lane 0's
  // acq_rel atomic, which releases them at gpu scope and, in the last CTA,
  // acquires the other CTAs' partials for both warps (next barrier) ----
  const int b_first = seq_of(s, p.batch, begin), b_last = seq_of(s, p.batch, end - 1);
#pragma unroll 1
  for (int e = 0; e < 2; ++e) {
    const int b = e == 0 ? b_first : b_last;
    if (e == 1 && b_last == b_first) break;
    const int pstart = s.prefix[b], pend = s.prefix[b + 1];
    const int cfirst = pstart / W, clast = (pend - 1) / W;
    if (cfirst == clast) continue;                    // written above
    if (par == 0 && lane == 0) {
      int old;
      asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + b * NKV + kvh) : "memory");
      const int last = (old == clast - cfirst);
      if (last) atomicExch(&p.cnt[b * NKV + kvh], 0);
      s.xch[kvh].flag = last;
    }
    named_bar_sync(1 + kvh, 64);
    const int last = s.xch[kvh].flag;
    named_bar_sync(1 + kvh, 64);
    if (!last) continue;
    // lane -> head 4 par + lane / 8, dims 8 (lane % 8) .. +7
    const int h = 4 * par + (lane >> 3), d = 8 * (lane & 7);
    constexpr int CB = 6;
    float M = -INFINITY, den = 0.f;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int cb = cfirst; cb <= clast; cb += CB) {
      float2 mlv[CB];
      float4 ov[CB][2];
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        if (cb + j <= clast) {
          const int64_t sl = ((int64_t)(cb + j) + b) * NKV + kvh;
          mlv[j] = __ldcg(&p.ml[sl * GROUP + h]);
          ov[j][0] = ld_cg4(p.po + (sl * GROUP + h) * HD + d);
          ov[j][1] = ld_cg4(p.po + (sl * GROUP + h) * HD + d + 4);
        } else {
          mlv[j] = make_float2(-INFINITY, 0.f);
          ov[j][0] = ov[j][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        if (!(mlv[j].y > 0.f)) continue;
        const float Mn = fmaxf(M, mlv[j].x);
        const float sa = exp2f(M - Mn), sbv = exp2f(mlv[j].x - Mn);
        den = den * sa + mlv[j].y * sbv;
        const float v[8] = {ov[j][0].x, ov[j][0].y, ov[j][0].z, ov[j][0].w,
                            ov[j][1].x, ov[j][1].y, ov[j][1].z, ov[j][1].w};
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) acc[q8] = fmaf(acc[q8], sa, v[q8] * sbv);
        M = Mn;
      }
    }
    const float inv = 1.0f / den;
    float* dst = p.out + ((int64_t)b * H + kvh * GROUP + h) * HD + d;
    *reinterpret_cast<float4*>(dst) = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
  }
}

size_t smem_bytes() { return sizeof(Smem) + 1024; }

}  // namespace pages

// ---- host side -------------------------------------------------------------

size_t pages_workspace_bytes(int batch) {
  const size_t b = (size_t)(batch < pages::MAX_SEQS ? batch : pages::MAX_SEQS);
  const size_t slots = (pages::MAX_GRID + b) * pages::NKV;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  // the counter block is sized for MAX_SEQS sequences whatever the batch, so
  // that calls of different batch sizes sharing a workspace (and the chunks
  // of a batch above MAX_SEQS) keep their counters in the same bytes
  return al((size_t)pages::MAX_SEQS * pages::NKV * sizeof(int32_t)) + al(slots * pages::GROUP * sizeof(float2)) +
         slots * pages::GROUP * pages::HD * sizeof(float);
}

size_t pages_counter_bytes() {
  return ((size_t)pages::MAX_SEQS * pages::NKV * sizeof(int32_t) + 255) & ~size_t(255);
}

int32_t launch_pages(const float* q, const float* kv_pool, int64_t n_pool_pages, const int32_t* page_table,
                     int32_t max_pages, const int32_t* seq_lens, float* out, int32_t batch, float qscale,
                     void* ws, cudaStream_t stream, int32_t* err_word, int num_sms) {
  using namespace pages;
  // the allocation-free entry passes its own error word and SM count (device_info may allocate)
  DeviceInfo local{};
  DeviceInfo* dev = &local;
  int32_t st = NYION_OK;
  if (err_word) {
    st = check_cuda(cudaGetDevice(&local.device), "cudaGetDevice");
    if (st) return st;
    local.num_sms = num_sms;
    local.err_word = err_word;
  } else {
    st = device_info(&dev);
    if (st) return st;
  }
  if ((uint64_t)n_pool_pages * NKV > (1ull << 31))
    return fail(NYION_ERR_INVALID, "decode_paged_f32: pool too large");
  CUtensorMap map;
  {
    // (x: 32 floats, slot: 16 x 256 B, half: 2 x 128 B, K/V: 2 x 4096 B,
    //  block = page * 4 + KV head: 8192 B); one box = one whole page
    const uint64_t dims[5] = {32, (uint64_t)PAGE, 2, 2, (uint64_t)n_pool_pages * NKV};
    const uint64_t strides[4] = {HD * 4, 128, PAGE * HD * 4, 2 * PAGE * HD * 4};
    const uint32_t box[5] = {32, (uint32_t)PAGE, 2, 2, (uint32_t)NKV};
    st = encode_tmap(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, kv_pool, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  const size_t smem = smem_bytes();
  int occ = 1;
  st = kernel_setup(reinterpret_cast<const void*>(decode_pages_kernel), smem, THREADS, &occ);
  if (st) return st;
  int grid = dev->num_sms * occ;
  if (grid > MAX_GRID) grid = MAX_GRID;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  for (int b0 = 0; b0 < batch; b0 += MAX_SEQS) {
    const int nb = batch - b0 < MAX_SEQS ? batch - b0 : MAX_SEQS;
    const size_t slots = (MAX_GRID + (size_t)nb) * NKV;
    Params p{};
    p.q = q + (int64_t)b0 * NKV * GROUP * HD;
    p.out = out + (int64_t)b0 * NKV * GROUP * HD;
    p.table = page_table + (int64_t)b0 * max_pages;
    p.seq_lens = seq_lens + b0;
    p.batch = nb;
    p.max_pages = max_pages;
    p.n_pool_pages = n_pool_pages;
    p.qscale = qscale;
    uint8_t* w = static_cast<uint8_t*>(ws);
    p.cnt = reinterpret_cast<int32_t*>(w);
    p.ml = reinterpret_cast<float2*>(w + al((size_t)MAX_SEQS * NKV * sizeof(int32_t)));
    p.po = reinterpret_cast<float*>(w + al((size_t)MAX_SEQS * NKV * sizeof(int32_t)) +
                                    al(slots * GROUP * sizeof(float2)));
    p.err = dev->err_word;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    st = check_cuda(cudaLaunchKernelEx(&cfg, decode_pages_kernel, p, map), "decode_pages launch");
    if (st) return st;
  }
  return NYION_OK;
}

}  // namespace nyion
