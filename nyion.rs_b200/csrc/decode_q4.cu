// decode_q4.cu — the 4-bit KV path: block quantizer / dequantizer, Q4 paged
// decode producing log-sum-exp partials, the fp32 ring partial, and the
// partial combine.
//
// Block format (swamp-engine/src/cache.rs:637-663, 375-394): 32 values ->
// 20 bytes [f16 d][f16 dmin][16 bytes of nibbles], element i in byte i/2,
// low nibble for even i; d = absmax / 7, q = clamp(round((x - dmin) / d), 0, 15),
// dequant x' = f32(d) * q + f32(dmin).
//
// Q4 decode on B200.  A nibble n becomes the fp16 value 1 + n/16 with one
// shift and one LOP3 per pair of values ((w << s) & 0x03C003C0 | 0x3C003C00),
// so the block's dot product  sum q_i (d n_i + dmin)  becomes
//   d * 16 * (sum q_i (1 + n_i/16) - sum q_i) + dmin * sum q_i,
// with sum q_i (1 + n_i/16) on the tensor cores (mma.sync m16n8k16 f16, fp32
// accumulate; q split into fp16 hi + lo rows) and the rest a per-score fix-up.
// P.V uses the same identity: v = 16 d (1 + n/16) + (dmin - 16 d), so
// o = sum_t (16 p_t d_t) v'_t  +  sum_t p_t (dmin_t - 16 d_t) per block.
// Only the nibbles of V are staged again in shared memory, as a swizzled fp16
// tile for ldmatrix.trans; K nibbles go straight from a 4-byte load into the
// B fragments.  The dims inside a 32-value block are visited in a fixed
// permutation (pairs (0,4), (1,5), (2,6), (3,7) of each 8-value group) that q
// and the output share.
#include <cuda_fp16.h>
#include <math.h>

#include <mutex>
#include <string.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace q4 {

constexpr int HD = 64;
constexpr int GROUP = 8;
constexpr int BLK = 20;                 // bytes per 32-value block
constexpr int ROWB = 2 * BLK;           // bytes per token row (head_dim 64)
constexpr int PAGE = 16;                // tokens per page
constexpr int NKV = 4;                  // KV heads per page in this build
constexpr int PAGE_KV = 2 * PAGE * ROWB;      // 1280 B: K rows then V rows of one KV head
constexpr int PAGE_BYTES = NKV * PAGE_KV;     // 5120 B: one whole page
constexpr int CHUNK = 64;               // tokens per stage (4 pages)
constexpr int STAGE_BYTES = 4 * PAGE_BYTES;   // 20 KB
constexpr int STAGES = 3;                // x 2 CTAs per SM
constexpr int NC = 8;                   // consumer warps: 4 KV heads x 2 token halves
constexpr int THREADS = (NC + 1) * 32;
constexpr int MAX_SEQS = 512;
constexpr int MAX_GRID = 1024;
constexpr int RING = 32;

// ============================================================================
// quantizer / dequantizer (bit-exact with cache.rs)
// ============================================================================

// One thread per (row, block): src [n_rows][head_dim] f32 -> dst [n_rows][nblk][20].
__global__ void quantize_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                int64_t n_rows, int head_dim) {
  const int nblk = (head_dim + 31) / 32;
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= n_rows * nblk) return;
  const int64_t row = id / nblk;
  const int blk = (int)(id % nblk);
  const int start = blk * 32;
  const int len = min(32, head_dim - start);
  const float* x = src + row * head_dim + start;
  float v[32];
  float mx = 0.0f, mn = 3.40282347e+38f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = (i < len) ? x[i] : 0.0f;
    if (i < len) {
      mx = fmaxf(mx, fabsf(v[i]));
      mn = fminf(mn, v[i]);
    }
  }
  const float d = mx > 1e-10f ? __fdiv_rn(mx, 7.0f) : 0.0f;
  const float dmin = mn;
  const unsigned short hd = __half_as_ushort(__float2half_rn(d));
  const unsigned short hm = __half_as_ushort(__float2half_rn(dmin));
  uint32_t w[5];
  w[0] = (uint32_t)hd | ((uint32_t)hm << 16);
  w[1] = w[2] = w[3] = w[4] = 0u;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    uint32_t q = 0;
    if (i < len && d > 1e-10f) {
      float r = roundf(__fdiv_rn(__fsub_rn(v[i], dmin), d));
      r = fminf(fmaxf(r, 0.0f), 15.0f);
      q = (uint32_t)r;
    }
    // nibble i lives in byte 4 + i/2: word 1 + i/8, bit (i % 8) * 4
    w[1 + i / 8] |= q << ((i % 8) * 4);
  }
  uint32_t* out = reinterpret_cast<uint32_t*>(dst + id * BLK);
#pragma unroll
  for (int j = 0; j < 5; ++j) out[j] = w[j];
}

__global__ void dequant_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst,
                               int64_t n_rows, int head_dim) {
  const int nblk = (head_dim + 31) / 32;
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= n_rows * nblk) return;
  const int64_t row = id / nblk;
  const int blk = (int)(id % nblk);
  const int start = blk * 32;
  const int len = min(32, head_dim - start);
  const uint32_t* in = reinterpret_cast<const uint32_t*>(src + id * BLK);
  const float d = __half2float(__ushort_as_half((unsigned short)(in[0] & 0xffffu)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(in[0] >> 16)));
  float* y = dst + row * head_dim + start;
  for (int i = 0; i < len; ++i) {
    const uint32_t q = (in[1 + i / 8] >> ((i % 8) * 4)) & 0xfu;
    y[i] = __fadd_rn(__fmul_rn(d, (float)q), dmin);   // separate mul and add
  }
}

// ============================================================================
// Q4 paged decode -> log-sum-exp partials
// ============================================================================

struct Params {
  const float* q;              // [batch][H][HD]
  const uint8_t* pool;         // [n_pool_pages][NKV][K|V][PAGE][40]
  const int32_t* table;        // [batch][max_pages]
  const int32_t* tok_begin;    // [batch] or null -> u_begin
  const int32_t* tok_end;      // [batch] or null -> u_end
  const int32_t* seq_lens;     // window mode: [batch] lengths; Q4 range = window minus ring
  int32_t window, ring_tokens; // window mode when seq_lens != null
  int32_t u_begin, u_end;
  int32_t batch, max_pages;
  int64_t n_pool_pages;
  float qscale;                // scale * log2(e)
  float* part;                 // [batch][H][HD + 2] result of the reduce: o / l, m (natural log), l
  float* cta_part;             // [MAX_GRID + batch][NKV][GROUP][HD + 2]: o (relative to m), m (log2), l
  int32_t* meta;               // [batch][2]: first and last CTA covering sequence b
  int32_t* err;
};

struct Smem {
  uint8_t kv[STAGES][STAGE_BYTES];
  uint8_t vt[NC][32 * 128];          // per warp: V chunk as fp16 [32 tokens][64], swizzled
  float hdr[NC][32][8];              // per warp and token: K factors | V factors, halves swapped for
                                     // tokens with bit 2 set (conflict-free 16-byte accesses)
  uint64_t full[STAGES], empty[STAGES];
  int32_t prefix[MAX_SEQS + 1];      // flat chunk index where sequence b starts
  int32_t c0[MAX_SEQS];              // first chunk (absolute, in 64-token units) of sequence b
  int32_t beg[MAX_SEQS], end[MAX_SEQS];
  int32_t rows[2][RING][5];          // per chunk: 4 page ids (or -1) and the sequence index
  int32_t warp_tot[THREADS / 32];
  int32_t abort_;
};

__device__ __forceinline__ int seek_seq(const Smem& s, int batch, int i) {
  int lo = 0, hi = batch;
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (s.prefix[mid] <= i) lo = mid; else hi = mid;
  }
  return lo;
}

struct RowJob {
  int valid, b;
  int32_t page[4];
};

__device__ __forceinline__ void rows_start(RowJob& j, const Smem& s, const Params& p, int i,
                                           int end) {
  j.valid = i < end;
  if (!j.valid) return;
  j.b = seek_seq(s, p.batch, i);
  const int chunk = s.c0[j.b] + (i - s.prefix[j.b]);
#pragma unroll
  for (int pg = 0; pg < 4; ++pg) {
    const int tok0 = chunk * CHUNK + pg * PAGE;
    const int pidx = chunk * 4 + pg;
    j.page[pg] = -2;   // not needed
    if (tok0 < s.end[j.b] && tok0 + PAGE > s.beg[j.b])
      j.page[pg] = (pidx < p.max_pages) ? p.table[(int64_t)j.b * p.max_pages + pidx] : -1;
  }
}

__device__ __forceinline__ void rows_finish(Smem& s, const Params& p, const RowJob& j, int slot,
                                            int lane) {
  if (!j.valid) return;
#pragma unroll
  for (int pg = 0; pg < 4; ++pg) {
    int32_t v = j.page[pg];
    if (v == -1 || (v >= 0 && v >= p.n_pool_pages)) {
      record_error(p.err, kErrPageRange);
      v = -2;    // skipped: the stage slot keeps stale bytes, all its tokens are masked out
    } else if (v < -2) {
      record_error(p.err, kErrPageRange);
      v = -2;
    }
    s.rows[slot][lane][pg] = v;
  }
  s.rows[slot][lane][4] = j.b;
}

// fp16x2 {1 + n_a/16, 1 + n_b/16} from the nibbles at bits [s+0..3] and [s+16..19] of w
template <int SHIFT>
__device__ __forceinline__ uint32_t nib2h(uint32_t w) {
  const uint32_t x = SHIFT >= 0 ? (w << SHIFT) : (w >> (-SHIFT));
  return (x & 0x03C003C0u) | 0x3C003C00u;
}

__device__ __forceinline__ float2 hdr2f(uint32_t w) {   // (d, dmin) of a block header word
  return make_float2(__half2float(__ushort_as_half((unsigned short)(w & 0xffffu))),
                     __half2float(__ushort_as_half((unsigned short)(w >> 16))));
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ void sts_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ void sts_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// dim visited at position c (0..63) of a row: pairs (0,4),(1,5),(2,6),(3,7) per 8-group
__device__ __forceinline__ int perm_dim(int c) {
  const int base = c & ~7, e = c & 7;
  return base + ((e & 1) ? 4 : 0) + (e >> 1);
}

__device__ __forceinline__ void named_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NC * 32) : "memory");
}

__global__ void __launch_bounds__(THREADS, 2) decode_q4_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                     ~uintptr_t(127));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int H = NKV * GROUP;

  if (t == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], NC);
    }
    s.abort_ = 0;
    fence_barrier_init();
  }
  // programmatic dependent launch: nothing global is read before the previous grid
  // in the stream completed, and the next grid (the ring partial or the reduce) is
  // released only after that, so it may read this kernel's inputs without waiting
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int b = t; b < p.batch; b += THREADS) {
    int lo, hi;
    if (p.seq_lens) {
      // config-3 split: Q4 tokens [max(0, L - window), max(that, L - ring))
      const int L = p.seq_lens[b];
      lo = max(0, L - p.window);
      hi = max(lo, L - p.ring_tokens);
    } else {
      lo = p.tok_begin ? p.tok_begin[b] : p.u_begin;
      hi = p.tok_end ? p.tok_end[b] : p.u_end;
    }
    lo = max(lo, 0);
    if (hi < lo) hi = lo;
    s.beg[b] = lo;
    s.end[b] = hi;
    s.c0[b] = lo / CHUNK;
  }
  __syncthreads();
  constexpr int PER = (MAX_SEQS + THREADS - 1) / THREADS;
  int local[PER];
  int run = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int b = t * PER + j;
    int c = 0;
    if (b < p.batch && s.end[b] > s.beg[b]) c = (s.end[b] + CHUNK - 1) / CHUNK - s.c0[b];
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

  const int total = s.prefix[p.batch];
  const int W = (total + gridDim.x - 1) / gridDim.x;
  if (blockIdx.x == 0) {
    for (int b = t; b < p.batch; b += THREADS) {
      const int lo = s.prefix[b], hi = s.prefix[b + 1];
      p.meta[2 * b] = hi > lo ? lo / W : 0;
      p.meta[2 * b + 1] = hi > lo ? (hi - 1) / W : -1;   // -1: empty range
    }
  }
  const int begin = blockIdx.x * W;
  const int end = min(total, begin + W);
  if (begin >= end) return;
  const int n = end - begin;

  if (warp == NC) {
    // ================= producer warp: whole pages by bulk copy =================
    RowJob job;
    rows_start(job, s, p, begin + lane, end);
    rows_finish(s, p, job, 0, lane);
    rows_start(job, s, p, begin + RING + lane, end);
    __syncwarp();
    for (int k = 0; k < n; ++k) {
      const int stage = k % STAGES;
      if (k % RING == RING / 2) {
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
          for (int c = k - 1; c >= 0 && c >= k - STAGES; --c)
            mbar_wait_bounded(&s.full[c % STAGES], (uint32_t)((c / STAGES) & 1));
        }
        return;
      }
      if (lane == 0) {
        const int32_t* e = s.rows[(k / RING) & 1][k % RING];
        uint32_t bytes = 0;
#pragma unroll
        for (int pg = 0; pg < 4; ++pg) bytes += (e[pg] >= 0) ? PAGE_BYTES : 0;
        // an all-skipped chunk still completes the phase through the arrive itself
        mbar_arrive_expect_tx(&s.full[stage], bytes);
#pragma unroll
        for (int pg = 0; pg < 4; ++pg)
          if (e[pg] >= 0)
            bulk_load(s.kv[stage] + pg * PAGE_BYTES, p.pool + (int64_t)e[pg] * PAGE_BYTES,
                      PAGE_BYTES, &s.full[stage]);
      }
      __syncwarp();
    }
    return;
  }

  // ================= consumer warps =================
  const int kvh = warp & 3, th = warp >> 2;
  const int g = lane >> 2, tig = lane & 3;
  const uint32_t vt = smem_u32(s.vt[warp]);
  const uint32_t hd = smem_u32(s.hdr[warp]);
  // ldmatrix.trans row addresses of the V tile for k-step kt, n-tile pair np:
  // matrix m = lane>>3: tokens 16kt + 8(m&1) + (lane&7), 16-B chunk 2np + (m>>1)
  uint32_t voff[2][4];
#pragma unroll
  for (int kt = 0; kt < 2; ++kt)
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      const uint32_t tok = 16 * kt + 8 * ((lane >> 3) & 1) + (lane & 7);
      const uint32_t ch = 2 * np + (lane >> 4);
      voff[kt][np] = tok * 128 + (((ch ^ tok) & 7) << 4);
    }

  int i = begin;
  while (i < end) {
    const int b = seek_seq(s, p.batch, i);
    const int seg_hi = min(end, s.prefix[b + 1]);
    const int sb = s.beg[b], se = s.end[b];
    // q fragments, dims permuted: k-step (blk, ks) pairs dims 32blk + 8tig + {ks*2 + (0,4)} in
    // a0/a1 and {ks*2 + (1,5)} in a2/a3, hi rows 0-7 and lo rows 8-15
    uint32_t qa[2][2][4];
    float qs[2];      // sum of the (hi + lo) q values of head g over each block
    {
      const float* qp = p.q + ((int64_t)b * H + kvh * GROUP + g) * HD;
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        float x[8];
        const float4 a = __ldg(reinterpret_cast<const float4*>(qp + 32 * blk + 8 * tig));
        const float4 c = __ldg(reinterpret_cast<const float4*>(qp + 32 * blk + 8 * tig + 4));
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = c.x; x[5] = c.y; x[6] = c.z; x[7] = c.w;
        float sum = 0.f;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          uint32_t h0, l0, h1, l1;
          split_f16x2(x[2 * ks] * p.qscale, x[2 * ks + 4] * p.qscale, h0, l0);
          split_f16x2(x[2 * ks + 1] * p.qscale, x[2 * ks + 5] * p.qscale, h1, l1);
          qa[blk][ks][0] = h0; qa[blk][ks][1] = l0; qa[blk][ks][2] = h1; qa[blk][ks][3] = l1;
          const float2 fh0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
          const float2 fl0 = __half22float2(*reinterpret_cast<const __half2*>(&l0));
          const float2 fh1 = __half22float2(*reinterpret_cast<const __half2*>(&h1));
          const float2 fl1 = __half22float2(*reinterpret_cast<const __half2*>(&l1));
          sum += (fh0.x + fl0.x) + (fh0.y + fl0.y) + (fh1.x + fl1.x) + (fh1.y + fl1.y);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        qs[blk] = sum;
      }
    }
    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) o[nt][j] = 0.f;
    float cb[2] = {0.f, 0.f};   // sum_t p_t (dmin - 16 d) per V block (this thread's tokens)
    float m = -INFINITY, l = 0.f;

    for (int k = i - begin; k < seg_hi - begin; ++k) {
      const int stage = k % STAGES;
      const int chunk = s.c0[b] + (begin + k - s.prefix[b]);
      const int pos0 = chunk * CHUNK + 32 * th;       // absolute position of this warp's token 0
      if (!s.abort_) {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s.full[stage], (uint32_t)((k / STAGES) & 1)))) {
          record_error(p.err, kErrWaitTimeout);
          if (lane == 0) atomicExch(&s.abort_, 1);
        }
      }
      const bool any = (pos0 < se) && (pos0 + 32 > sb);
      const bool inner = (pos0 >= sb) && (pos0 + 32 <= se);   // no token of this warp is masked
      if (any) {
        const uint32_t kb = smem_u32(s.kv[stage]) + 2 * th * PAGE_BYTES + kvh * PAGE_KV;
        // token t of this warp: page 2th + t/16 (offset (t/16)*PAGE_BYTES), row t%16
        // ---- V nibbles of token `lane` -> fp16 tile row `lane` ----
        {
          const uint32_t vr = kb + (lane >> 4) * PAGE_BYTES + PAGE * ROWB + (lane & 15) * ROWB;
#pragma unroll
          for (int blk = 0; blk < 2; ++blk)
#pragma unroll
            for (int wq = 0; wq < 4; ++wq) {
              const uint32_t w = lds_u32(vr + blk * BLK + 4 + 4 * wq);
              const uint32_t ch = 4 * blk + wq;
              sts_v4(vt + lane * 128 + (((ch ^ lane) & 7) << 4), nib2h<6>(w), nib2h<2>(w),
                     nib2h<-2>(w), nib2h<-6>(w));
            }
          // block headers of token `lane` as the fp32 factors the score and P.V steps use:
          // score = sum_blk 16 d (q.(1 + n/16)) + (dmin - 16 d) qs; zero for masked tokens
          const uint32_t kr = vr - PAGE * ROWB;
          const float2 k0 = hdr2f(lds_u32(kr)), k1 = hdr2f(lds_u32(kr + BLK));
          const float2 v0 = hdr2f(lds_u32(vr)), v1 = hdr2f(lds_u32(vr + BLK));
          const bool live = inner || ((pos0 + lane >= sb) && (pos0 + lane < se));
          const float a0 = 16.0f * k0.x, a1 = 16.0f * k1.x, b0 = 16.0f * v0.x, b1 = 16.0f * v1.x;
          const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
          const uint32_t sw = ((lane >> 2) & 1) << 4;
          sts_f4(hd + lane * 32 + sw, live ? make_float4(a0, k0.y - a0, a1, k1.y - a1) : zero);
          sts_f4(hd + lane * 32 + (sw ^ 16), live ? make_float4(b0, v0.y - b0, b1, v1.y - b1) : zero);
        }
        __syncwarp();   // V tile rows and headers written by all lanes
        // ---- S = Q K^T: 4 n-tiles of 8 tokens, 2 blocks x 2 k-steps ----
        float sc[4][2][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int tk = 8 * nt + g;
          const uint32_t kr = kb + (tk >> 4) * PAGE_BYTES + (tk & 15) * ROWB;
#pragma unroll
          for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[nt][blk][j] = 0.f;
            const uint32_t w = lds_u32(kr + blk * BLK + 4 + 4 * tig);
            mma_f16(sc[nt][blk], qa[blk][0], nib2h<6>(w), nib2h<2>(w));
            mma_f16(sc[nt][blk], qa[blk][1], nib2h<-2>(w), nib2h<-6>(w));
          }
        }
        float sv[4][2];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int tt = 8 * nt + 2 * tig + e;
            const float4 h = lds_f4(hd + tt * 32 + (((tt >> 2) & 1) << 4));   // a0, c0, a1, c1
            const float t0 = sc[nt][0][e] + sc[nt][0][2 + e];            // sum q (1 + n/16), hi + lo rows
            const float t1 = sc[nt][1][e] + sc[nt][1][2 + e];
            sv[nt][e] = fmaf(h.x, t0, fmaf(h.z, t1, fmaf(h.y, qs[0], h.w * qs[1])));
          }
        if (!inner) {   // the sequence range starts or ends inside this warp's 32 tokens
#pragma unroll
          for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int pos = pos0 + 8 * nt + 2 * tig + e;
              if (pos < sb || pos >= se) sv[nt][e] = -INFINITY;
            }
        }
        // ---- online softmax ----
        float mx = sv[0][0];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mx = fmaxf(mx, fmaxf(sv[nt][0], sv[nt][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        // lazy rescale: the reference max m moves only when the chunk max passes it by
        // more than 2 (log2 units), so p <= 4 and most chunks skip the rescale
        if (mx > m + 2.0f) {
          const float al = exp2f(m - mx);                               // m = -inf: 0
          l *= al;
#pragma unroll
          for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int j = 0; j < 4; ++j) o[nt][j] *= al;
          cb[0] *= al;
          cb[1] *= al;
          m = mx;
        }
        const float mref = m == -INFINITY ? 0.f : m;                    // all masked so far: p = 0
        float ps = 0.f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          sv[nt][0] = exp2f(sv[nt][0] - mref);
          sv[nt][1] = exp2f(sv[nt][1] - mref);
          ps += sv[nt][0] + sv[nt][1];
        }
        l += ps;
        // ---- P'_blk = 16 p d_V (A operand), correction terms ----
        uint32_t pa[2][2][4];   // [blk][kt]
#pragma unroll
        for (int kt = 0; kt < 2; ++kt) {
          float pv[2][4];       // [blk][token e: 16kt + 2tig + {0,1,8,9}]
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int nt = 2 * kt + (e >> 1);
            const int tt = 8 * nt + 2 * tig + (e & 1);
            const float pe = sv[nt][e & 1];
            // 16 d_V and dmin_V - 16 d_V of both blocks (zero for masked tokens, whose
            // stage bytes may be stale)
            const float4 h = lds_f4(hd + tt * 32 + ((((tt >> 2) & 1) ^ 1) << 4));
            pv[0][e] = pe * h.x;
            pv[1][e] = pe * h.z;
            cb[0] = fmaf(pe, h.y, cb[0]);
            cb[1] = fmaf(pe, h.w, cb[1]);
          }
#pragma unroll
          for (int blk = 0; blk < 2; ++blk) {
            split_f16x2(pv[blk][0], pv[blk][1], pa[blk][kt][0], pa[blk][kt][1]);
            split_f16x2(pv[blk][2], pv[blk][3], pa[blk][kt][2], pa[blk][kt][3]);
          }
        }
        // ---- O += P' V': k = 16 tokens, n-tiles of 8 (permuted) dims ----
#pragma unroll
        for (int kt = 0; kt < 2; ++kt)
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vt + voff[kt][np], b0, b1, b2, b3);
            const int blk = np >> 1;
            mma_f16(o[2 * np], pa[blk][kt], b0, b1);
            mma_f16(o[2 * np + 1], pa[blk][kt], b2, b3);
          }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[stage]);
    }

    // ---- segment end: the two token halves of each KV head merge in shared
    //      memory, one partial per (CTA, sequence, KV head) goes to the workspace ----
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      cb[blk] += __shfl_xor_sync(0xffffffffu, cb[blk], 1);
      cb[blk] += __shfl_xor_sync(0xffffffffu, cb[blk], 2);
    }
    named_sync();                       // every warp is done with its V tile
    float* mine = reinterpret_cast<float*>(s.vt[warp]);   // [GROUP][HD + 2]
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = 8 * nt + 2 * tig + e;
        mine[g * (HD + 2) + perm_dim(c)] = o[nt][e] + o[nt][2 + e] + cb[nt >> 2];
      }
    if (tig == 0) {
      mine[g * (HD + 2) + HD] = m;
      mine[g * (HD + 2) + HD + 1] = l;
    }
    named_sync();
    if (th == 0) {
      // lane -> head lane>>2, dims 16*(lane&3) .. +15; partner warp holds the other half
      const float* a0 = reinterpret_cast<const float*>(s.vt[warp]);
      const float* a1 = reinterpret_cast<const float*>(s.vt[warp + 4]);
      const int mh = lane >> 2, md = 16 * (lane & 3);
      const float m0 = a0[mh * (HD + 2) + HD], l0 = a0[mh * (HD + 2) + HD + 1];
      const float m1 = a1[mh * (HD + 2) + HD], l1 = a1[mh * (HD + 2) + HD + 1];
      const float M = fmaxf(m0, m1);
      const float w0 = (l0 > 0.f) ? exp2f(m0 - M) : 0.f, w1 = (l1 > 0.f) ? exp2f(m1 - M) : 0.f;
      float* dst = p.cta_part + ((((int64_t)blockIdx.x + b) * NKV + kvh) * GROUP + mh) * (HD + 2);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float v0 = (l0 > 0.f) ? a0[mh * (HD + 2) + md + e] : 0.f;
        const float v1 = (l1 > 0.f) ? a1[mh * (HD + 2) + md + e] : 0.f;
        __stcg(dst + md + e, w0 * v0 + w1 * v1);
      }
      if ((lane & 3) == 0) {
        __stcg(dst + HD, M);
        __stcg(dst + HD + 1, w0 * l0 + w1 * l1);
      }
    }
    named_sync();                       // partner tiles are read before the next segment writes them
    i = seg_hi;
  }
}

// ============================================================================
// reduce of the per-CTA partials: one CTA per (sequence, query head) row
// ============================================================================
// 8 warps take the covering CTAs round-robin (lane = 2 dims, four partial
// loads in flight), then warp 0 folds the 8 warp results.  Output is the
// partial format (o/l, m natural, l) or, with `final_out`, o/l alone.
struct RingArgs {
  const float* q;          // [batch][H][HD]
  const float* ring;       // [batch][NKV][K|V][ring_tokens][HD]
  const int32_t* seq_lens; // [batch]
  int32_t ring_tokens, window;
  float qscale;            // scale * log2(e)
};

constexpr int RING_MAX = 128;   // ring tokens of one sequence (larger rings: error)

// fp32 ring tokens [max(max(0, L - window), L - ring), L) of config 3 (slot pos %
// ring), one (sequence, KV head) per CTA, all 8 query heads of the group.  Every
// global load of the CTA goes out in one batch: q, each thread's half K row
// (eight 16-byte loads) and its sixteen 8-byte V pairs (V does not depend on the
// scores).  Scores: thread = (token, half row), dots for the 8 heads against q in
// shared memory (each half padded by 16 bytes, so the two halves a warp reads
// fall in different banks), halves joined by a shuffle.  Softmax: warp = head.
// P.V: thread = (dim pair, 16-token group), 8 heads accumulated, the 8 groups
// summed at the merge.
struct RingSmem {
  float qs[GROUP][2][36];    // [head][half][32 dims + 4 pad]
  float ps[GROUP][RING_MAX];
  float red[8][GROUP][HD];   // [16-token group][head][dim] partial P.V sums
  float mls[GROUP][2];       // (m log2, l) per head
};

// The ring tokens' partial of (sequence b, KV head kvh), all 8 query heads,
// left in shared memory: o[h][d] = sum_g red[g][h][d] (relative to mls[h][0]),
// l = mls[h][1].  Returns the number of ring tokens attended.
__device__ int ring_partial_cta(const RingArgs& ra, int b, int kvh, RingSmem& sm) {
  constexpr int TOK = RING_MAX;
  const int t = threadIdx.x, w = t >> 5, lane = t & 31;
  const int R = ra.ring_tokens;
  const int Ls = ra.seq_lens[b];
  const int lo = max(max(0, Ls - ra.window), Ls - R);
  const int n = min(max(0, Ls - lo), TOK);
  const int lo_slot = lo % R;
  auto slot_of = [&](int j) { const int sl = lo_slot + j; return sl >= R ? sl - R : sl; };   // j < R
  const float* qb = ra.q + ((int64_t)b * NKV * GROUP + kvh * GROUP) * HD;
  const float* kb = ra.ring + ((int64_t)(b * NKV + kvh) * 2 + 0) * R * HD;
  const float* vb = ra.ring + ((int64_t)(b * NKV + kvh) * 2 + 1) * R * HD;
  // ---- all global loads in flight together ----
  const int j = t >> 1, half = t & 1;          // scores: token j, dims 32 half .. +31
  const int dp = lane, tg = w;                 // P.V: dims 2dp, 2dp+1; tokens 16tg .. 16tg+15
  const float q0 = qb[t], q1 = qb[t + 256];
  float4 k[8];
  if (j < n) {
    const float4* kr = reinterpret_cast<const float4*>(kb + (int64_t)slot_of(j) * HD + 32 * half);
#pragma unroll
    for (int c = 0; c < 8; ++c) k[c] = __ldg(kr + c);
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) k[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float2 v[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const int jj = 16 * tg + u;
    v[u] = jj < n ? __ldg(reinterpret_cast<const float2*>(vb + (int64_t)slot_of(jj) * HD) + dp)
                  : make_float2(0.f, 0.f);
  }
  sm.qs[t / HD][(t % HD) / 32][t % 32] = q0 * ra.qscale;
  sm.qs[(t + 256) / HD][((t + 256) % HD) / 32][(t + 256) % 32] = q1 * ra.qscale;
  __syncthreads();
  {
    float acc[GROUP];
#pragma unroll
    for (int h = 0; h < GROUP; ++h) acc[h] = 0.f;
    if (j < n) {
#pragma unroll
      for (int c = 0; c < 8; ++c)
#pragma unroll
        for (int h = 0; h < GROUP; ++h) {
          const float4 qq = *reinterpret_cast<const float4*>(&sm.qs[h][half][4 * c]);
          acc[h] = fmaf(qq.x, k[c].x, fmaf(qq.y, k[c].y, fmaf(qq.z, k[c].z, fmaf(qq.w, k[c].w, acc[h]))));
        }
    }
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      const float sc = acc[h] + __shfl_xor_sync(0xffffffffu, acc[h], 1);
      if (half == 0 && j < TOK) sm.ps[h][j] = j < n ? sc : -INFINITY;
    }
  }
  __syncthreads();
  {  // softmax of head w over the tokens
    float mx = -INFINITY;
    for (int j = lane; j < TOK; j += 32) mx = fmaxf(mx, sm.ps[w][j]);
    mx = warp_max(mx);
    float l = 0.f;
    for (int j = lane; j < TOK; j += 32) {
      const float pe = mx > -INFINITY ? exp2f(sm.ps[w][j] - mx) : 0.f;
      sm.ps[w][j] = pe;
      l += pe;
    }
    l = warp_sum(l);
    if (lane == 0) {
      sm.mls[w][0] = mx;
      sm.mls[w][1] = l;
    }
  }
  __syncthreads();
  {
    float2 acc[GROUP];
#pragma unroll
    for (int h = 0; h < GROUP; ++h) acc[h] = make_float2(0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 16; ++u)
#pragma unroll
      for (int h = 0; h < GROUP; ++h) {
        const float pe = sm.ps[h][16 * tg + u];
        acc[h].x = fmaf(pe, v[u].x, acc[h].x);
        acc[h].y = fmaf(pe, v[u].y, acc[h].y);
      }
#pragma unroll
    for (int h = 0; h < GROUP; ++h) {
      sm.red[tg][h][2 * dp] = acc[h].x;
      sm.red[tg][h][2 * dp + 1] = acc[h].y;
    }
  }
  __syncthreads();
  return n;
}

// ---- split-KV exchange over peer memory ----------------------------------
// Every rank owns a mailbox with the same layout.  A rank writes its partial
// of row r into slot [rank] of EVERY rank's mailbox (stores over NVLink) as
// 64-bit words: value bits low, the step's epoch high.  An aligned 64-bit
// store is single-copy atomic, so a reader that sees the epoch in a word sees
// its value: no fence and no separate flag (the scheme of NCCL's LL
// protocol).  A reader polls its row's words of every rank until all carry
// the epoch, then combines.  Each row's epoch is a counter kept by the row's
// CTA in its own mailbox header; buf = epoch & 1 double-buffers consecutive
// steps: a rank writes step s+1 only after reading every rank's step-s words,
// and every rank has read step s-1 before it writes step s.
constexpr int MAX_RANKS = 8;
struct Exchange {
  uint8_t* mbox[MAX_RANKS];   // mailbox of rank r ([rank] = this rank's own)
  int32_t world, rank, rows;  // world 0: no exchange
  long long timeout_ns;       // bound on the wait for the other ranks
};
__host__ __device__ constexpr size_t mbox_data_off(int rows) {
  return (size_t(rows) * 4 + 255) & ~size_t(255);          // after the per-row epochs
}
__host__ __device__ constexpr size_t mbox_bytes(int rows) {
  return mbox_data_off(rows) + size_t(2) * MAX_RANKS * rows * (HD + 2) * 8;
}

__device__ __forceinline__ void st_word(uint64_t* p, float v, uint32_t epoch) {
  const uint64_t w = ((uint64_t)epoch << 32) | __float_as_uint(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// One CTA per (sequence, query head) row.  The covering CTAs' partials are
// taken by the 8 warps round-robin with up to RU of them loaded before any is
// folded (one L2 round trip for up to 8 RU CTAs); warp 0 combines.  Without an exchange the row is written as
// the partial format (o/l, m natural, l) or, with `final_out`, o/l alone;
// with an exchange it is sent to every rank and the ranks' partials of the
// row are combined into `final_out`.
constexpr int RU = 20;
__global__ void __launch_bounds__(256) q4_reduce_kernel(const float* __restrict__ cta_part,
                                                       const int32_t* __restrict__ meta, int batch,
                                                       float* __restrict__ part,
                                                       float* __restrict__ final_out,
                                                       const __grid_constant__ Exchange ex, int32_t* err) {
  __shared__ float red[8][HD + 2];
  pdl_wait();
  const int row = blockIdx.x;                 // b * 32 + h
  const int b = row / (NKV * GROUP), h = row % (NKV * GROUP);
  const int kvh = h / GROUP, hh = h % GROUP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cf = meta[2 * b], cl = meta[2 * b + 1];
  float M = -INFINITY, L = 0.f, o0 = 0.f, o1 = 0.f;
  for (int cbase = cf; cbase <= cl; cbase += 8 * RU) {
    float2 ml[RU], ov[RU];
#pragma unroll
    for (int u = 0; u < RU; ++u) {
      const int c = cbase + warp + 8 * u;
      if (c <= cl) {
        const float* src = cta_part + ((((int64_t)c + b) * NKV + kvh) * GROUP + hh) * (HD + 2);
        ml[u] = __ldcg(reinterpret_cast<const float2*>(src + HD));
        ov[u] = __ldcg(reinterpret_cast<const float2*>(src) + lane);
      } else {
        ml[u] = make_float2(-INFINITY, 0.f);
        ov[u] = make_float2(0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < RU; ++u) {
      if (!(ml[u].y > 0.f)) continue;
      const float Mn = fmaxf(M, ml[u].x);
      const float sa = exp2f(M - Mn), sb = exp2f(ml[u].x - Mn);
      L = L * sa + ml[u].y * sb;
      o0 = o0 * sa + ov[u].x * sb;
      o1 = o1 * sa + ov[u].y * sb;
      M = Mn;
    }
  }
  red[warp][2 * lane] = o0;
  red[warp][2 * lane + 1] = o1;
  if (lane == 0) {
    red[warp][HD] = M;
    red[warp][HD + 1] = L;
  }
  constexpr int nparts = 8;
  __syncthreads();
  if (warp != 0) return;
  float Mt = -INFINITY;
  for (int w = 0; w < nparts; ++w)
    if (red[w][HD + 1] > 0.f) Mt = fmaxf(Mt, red[w][HD]);
  float den = 0.f, a0 = 0.f, a1 = 0.f;
  for (int w = 0; w < nparts; ++w) {
    if (!(red[w][HD + 1] > 0.f)) continue;
    const float wt = exp2f(red[w][HD] - Mt);
    den = fmaf(wt, red[w][HD + 1], den);
    a0 = fmaf(wt, red[w][2 * lane], a0);
    a1 = fmaf(wt, red[w][2 * lane + 1], a1);
  }
  const float inv = den > 0.f ? 1.0f / den : 0.f;
  const float mnat = den > 0.f ? Mt * 0.6931471805599453f : -INFINITY;   // log2 -> natural units
  if (ex.world == 0) {
    if (final_out) {
      final_out[(int64_t)row * HD + 2 * lane] = a0 * inv;
      final_out[(int64_t)row * HD + 2 * lane + 1] = a1 * inv;
    } else {
      float* dst = part + (int64_t)row * (HD + 2);
      dst[2 * lane] = a0 * inv;
      dst[2 * lane + 1] = a1 * inv;
      if (lane == 0) {
        dst[HD] = mnat;
        dst[HD + 1] = den;
      }
    }
    return;
  }

  // ---- exchange: this rank's row partial to every rank, then combine ----
  int* epochs = reinterpret_cast<int*>(ex.mbox[ex.rank]);     // [rows] steps done per row
  uint32_t epoch = 0;
  if (lane == 0) epoch = (uint32_t)(*reinterpret_cast<volatile int*>(epochs + row)) + 1u;
  epoch = __shfl_sync(0xffffffffu, epoch, 0);
  const int buf = epoch & 1;
  const size_t slot = ((size_t)(buf * MAX_RANKS + ex.rank) * ex.rows + row) * (HD + 2);
  for (int r = 0; r < ex.world; ++r) {
    uint64_t* dst = reinterpret_cast<uint64_t*>(ex.mbox[r] + mbox_data_off(ex.rows)) + slot;
    st_word(dst + 2 * lane, a0 * inv, epoch);
    st_word(dst + 2 * lane + 1, a1 * inv, epoch);
    if (lane == 0) {
      st_word(dst + HD, mnat, epoch);
      st_word(dst + HD + 1, den, epoch);
    }
  }
  // every rank's words of this row, from this rank's own mailbox
  const uint64_t* box = reinterpret_cast<const uint64_t*>(ex.mbox[ex.rank] + mbox_data_off(ex.rows));
  float v0[MAX_RANKS], v1[MAX_RANKS], vm[MAX_RANKS], vl[MAX_RANKS];
  bool ok = true;
  const unsigned long long t0 = global_ns();
#pragma unroll
  for (int r = 0; r < MAX_RANKS; ++r) {
    v0[r] = v1[r] = 0.f;
    vm[r] = -INFINITY;
    vl[r] = 0.f;
    if (r >= ex.world || !ok) continue;
    const uint64_t* src = box + ((size_t)(buf * MAX_RANKS + r) * ex.rows + row) * (HD + 2);
    uint32_t spins = 0;
    while (true) {
      const uint64_t w0 = ld_word(src + 2 * lane), w1 = ld_word(src + 2 * lane + 1);
      const uint64_t wm = ld_word(src + HD), wl = ld_word(src + HD + 1);
      const bool here = (uint32_t)(w0 >> 32) == epoch && (uint32_t)(w1 >> 32) == epoch &&
                        (uint32_t)(wm >> 32) == epoch && (uint32_t)(wl >> 32) == epoch;
      if (__all_sync(0xffffffffu, here)) {
        v0[r] = __uint_as_float((uint32_t)w0);
        v1[r] = __uint_as_float((uint32_t)w1);
        vm[r] = __uint_as_float((uint32_t)wm);
        vl[r] = __uint_as_float((uint32_t)wl);
        break;
      }
      if (++spins > 32) __nanosleep(64);
      if ((long long)(global_ns() - t0) > ex.timeout_ns) {
        ok = false;
        break;
      }
    }
  }
  if (!ok && lane == 0) record_error(err, kErrWaitTimeout);
  float Mr = -INFINITY;
#pragma unroll
  for (int r = 0; r < MAX_RANKS; ++r)
    if (vl[r] > 0.f) Mr = fmaxf(Mr, vm[r]);
  float dr = 0.f, c0 = 0.f, c1 = 0.f;
#pragma unroll
  for (int r = 0; r < MAX_RANKS; ++r) {
    if (!(vl[r] > 0.f)) continue;
    const float wt = vl[r] * expf(vm[r] - Mr);
    dr += wt;
    c0 = fmaf(wt, v0[r], c0);
    c1 = fmaf(wt, v1[r], c1);
  }
  const float ir = dr > 0.f ? 1.0f / dr : 0.f;
  final_out[(int64_t)row * HD + 2 * lane] = c0 * ir;
  final_out[(int64_t)row * HD + 2 * lane + 1] = c1 * ir;
  if (lane == 0) *reinterpret_cast<volatile int*>(epochs + row) = (int)epoch;
}

// Config 3: the fp32 ring tokens' partial and the reduce in one launch.  CTA =
// (sequence, KV head), warp = query head.  Launched with programmatic dependent
// launch after the 4-bit decode, whose CTAs release it only after their own
// wait on the grid before them, so the ring inputs are complete: the ring part
// runs while decode CTAs drain, then the CTA waits for the decode to complete
// and folds the covering CTAs' partials (up to RU loaded per round trip) into
// the ring's.  Writes o / l.
__global__ void __launch_bounds__(256) q4_reduce_ring_kernel(const float* __restrict__ cta_part,
                                                            const int32_t* __restrict__ meta,
                                                            float* __restrict__ final_out, const RingArgs ra) {
  __shared__ RingSmem sm;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int b = blockIdx.x / NKV, kvh = blockIdx.x % NKV;
  const int hh = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = ring_partial_cta(ra, b, kvh, sm);
  asm volatile("griddepcontrol.wait;" ::: "memory");   // the decode's partials and meta are complete
  float M = -INFINITY, L = 0.f, o0 = 0.f, o1 = 0.f;
  if (n > 0 && sm.mls[hh][1] > 0.f) {
    M = sm.mls[hh][0];
    L = sm.mls[hh][1];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      o0 += sm.red[g][hh][2 * lane];
      o1 += sm.red[g][hh][2 * lane + 1];
    }
  }
  const int cf = meta[2 * b], cl = meta[2 * b + 1];
  for (int cbase = cf; cbase <= cl; cbase += RU) {
    float2 ml[RU], ov[RU];
#pragma unroll
    for (int u = 0; u < RU; ++u) {
      const int c = cbase + u;
      if (c <= cl) {
        const float* src = cta_part + ((((int64_t)c + b) * NKV + kvh) * GROUP + hh) * (HD + 2);
        ml[u] = __ldcg(reinterpret_cast<const float2*>(src + HD));
        ov[u] = __ldcg(reinterpret_cast<const float2*>(src) + lane);
      } else {
        ml[u] = make_float2(-INFINITY, 0.f);
        ov[u] = make_float2(0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < RU; ++u) {
      if (!(ml[u].y > 0.f)) continue;
      const float Mn = fmaxf(M, ml[u].x);
      const float sa = exp2f(M - Mn), sb = exp2f(ml[u].x - Mn);
      L = L * sa + ml[u].y * sb;
      o0 = o0 * sa + ov[u].x * sb;
      o1 = o1 * sa + ov[u].y * sb;
      M = Mn;
    }
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  float* dst = final_out + ((int64_t)b * NKV * GROUP + kvh * GROUP + hh) * HD;
  *reinterpret_cast<float2*>(dst + 2 * lane) = make_float2(o0 * inv, o1 * inv);
}

// ============================================================================
// log-sum-exp combine: parts [G][rows][HD+2] -> out [rows][HD]
// ============================================================================
__global__ void lse_combine_kernel(const float* __restrict__ parts, int G, int64_t rows,
                                   float* __restrict__ out) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 16) + (threadIdx.x >> 4);
  const int d4 = (threadIdx.x & 15) * 4;
  if (r >= rows) return;
  float M = -INFINITY;
  for (int gi = 0; gi < G; ++gi) {
    const float* pp = parts + ((int64_t)gi * rows + r) * (HD + 2);
    if (pp[HD + 1] > 0.f) M = fmaxf(M, pp[HD]);
  }
  float den = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (M != -INFINITY) {
    for (int gi = 0; gi < G; ++gi) {
      const float* pp = parts + ((int64_t)gi * rows + r) * (HD + 2);
      const float lg = pp[HD + 1];
      if (!(lg > 0.f)) continue;
      const float w = lg * expf(pp[HD] - M);
      den += w;
      acc.x = fmaf(w, pp[d4], acc.x);
      acc.y = fmaf(w, pp[d4 + 1], acc.y);
      acc.z = fmaf(w, pp[d4 + 2], acc.z);
      acc.w = fmaf(w, pp[d4 + 3], acc.w);
    }
  }
  const float inv = den > 0.f ? 1.0f / den : 0.f;
  *reinterpret_cast<float4*>(out + r * HD + d4) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

size_t smem_bytes() { return sizeof(Smem) + 128; }
// two CTAs per SM: 2 x (dynamic + 1 KB reserved) within the 228 KB of an SM
static_assert(sizeof(Smem) + 128 + 1024 <= 114 * 1024, "decode_q4 shared memory must allow 2 CTAs per SM");

struct WsLayout {
  size_t meta, cta_part, total;
};

WsLayout ws_layout(int batch) {
  const int b = batch < MAX_SEQS ? batch : MAX_SEQS;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  WsLayout w;
  w.meta = 0;
  w.cta_part = al((size_t)b * 2 * sizeof(int32_t));
  w.total = w.cta_part + al((size_t)(MAX_GRID + b) * NKV * GROUP * (HD + 2) * sizeof(float));
  return w;
}

int32_t check_shape(int32_t n_heads, int32_t n_kv_heads, int32_t head_dim) {
  if (n_kv_heads != NKV || n_heads != NKV * GROUP || head_dim != HD)
    return fail(NYION_ERR_UNSUPPORTED,
                "the 4-bit kernels of this build take 32 query heads, 4 KV heads, head_dim 64 "
                "(got %d/%d/%d)", n_heads, n_kv_heads, head_dim);
  return NYION_OK;
}

int32_t launch_partial(Params base, int batch, const int32_t* tok_begin, const int32_t* tok_end,
                       const float* q, float* part, const int32_t* table, void* ws,
                       cudaStream_t stream, float* final_out = nullptr, RingArgs ra = RingArgs{},
                       const Exchange& ex = Exchange{}) {
  DeviceInfo* dev = nullptr;
  int32_t st = device_info(&dev);
  if (st) return st;
  const size_t smem = smem_bytes();
  int occ = 1;
  st = kernel_setup(reinterpret_cast<const void*>(decode_q4_kernel), smem, THREADS, &occ);
  if (st) return st;
  const int grid = dev->num_sms * occ < MAX_GRID ? dev->num_sms * occ : MAX_GRID;
  const WsLayout w = ws_layout(batch);
  for (int b0 = 0; b0 < batch; b0 += MAX_SEQS) {
    Params p = base;
    const int nb = batch - b0 < MAX_SEQS ? batch - b0 : MAX_SEQS;
    p.batch = nb;
    p.tok_begin = tok_begin ? tok_begin + b0 : nullptr;
    p.tok_end = tok_end ? tok_end + b0 : nullptr;
    p.q = q + (int64_t)b0 * NKV * GROUP * HD;
    p.part = part + (int64_t)b0 * NKV * GROUP * (HD + 2);
    p.table = table + (int64_t)b0 * base.max_pages;
    p.seq_lens = base.seq_lens ? base.seq_lens + b0 : nullptr;
    p.meta = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws) + w.meta);
    p.cta_part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + w.cta_part);
    p.err = dev->err_word;
    st = check_cuda(launch_pdl(decode_q4_kernel, dim3(grid), dim3(THREADS), smem, stream, p),
                    "decode_q4 launch");
    if (st) return st;
    float* fo = final_out ? final_out + (int64_t)b0 * NKV * GROUP * HD : nullptr;
    const float* cp = p.cta_part;
    const int32_t* mt = p.meta;
    if (ra.ring) {   // config 3: ring partial + reduce in one launch (final output only)
      RingArgs r = ra;
      r.q = q + (int64_t)b0 * NKV * GROUP * HD;
      r.ring = ra.ring + (int64_t)b0 * NKV * 2 * ra.ring_tokens * HD;
      r.seq_lens = ra.seq_lens + b0;
      st = check_cuda(launch_pdl(q4_reduce_ring_kernel, dim3(nb * NKV), dim3(256), 0, stream, cp, mt, fo, r),
                      "q4_reduce_ring launch");
    } else {
      st = check_cuda(launch_pdl(q4_reduce_kernel, dim3(nb * NKV * GROUP), dim3(256), 0, stream, cp, mt, nb, p.part,
                                 fo, ex, dev->err_word),
                      "q4_reduce launch");
    }
    if (st) return st;
  }
  return NYION_OK;
}

}  // namespace q4
}  // namespace nyion

using namespace nyion;
using namespace nyion::q4;

extern "C" int32_t nyion_attn_quantize_q4(const float* src, uint8_t* dst, int64_t n_rows,
                                          int32_t head_dim, void* stream) {
  if (!src || !dst || n_rows < 0 || head_dim <= 0)
    return fail(NYION_ERR_INVALID, "quantize_q4: bad arguments");
  if (n_rows == 0) return NYION_OK;
  const int64_t n = n_rows * ((head_dim + 31) / 32);
  quantize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(src, dst, n_rows,
                                                                                          head_dim);
  return check_cuda(cudaGetLastError(), "quantize_q4 launch");
}

extern "C" int32_t nyion_attn_dequant_q4(const uint8_t* src, float* dst, int64_t n_rows,
                                         int32_t head_dim, void* stream) {
  if (!src || !dst || n_rows < 0 || head_dim <= 0)
    return fail(NYION_ERR_INVALID, "dequant_q4: bad arguments");
  if (n_rows == 0) return NYION_OK;
  const int64_t n = n_rows * ((head_dim + 31) / 32);
  dequant_kernel<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(src, dst, n_rows,
                                                                                         head_dim);
  return check_cuda(cudaGetLastError(), "dequant_q4 launch");
}

extern "C" size_t nyion_attn_q4_workspace_size(int32_t batch) {
  return batch > 0 ? ws_layout(batch).total : 0;
}

extern "C" int32_t nyion_attn_decode_q4_partial(const float* q, const uint8_t* kv_pool,
                                                int64_t n_pool_pages, const int32_t* page_table,
                                                int32_t max_pages, const int32_t* tok_begin,
                                                const int32_t* tok_end, int32_t u_begin,
                                                int32_t u_end, float* part, int32_t batch,
                                                int32_t n_heads, int32_t n_kv_heads,
                                                int32_t head_dim, int32_t page_tokens, float scale,
                                                void* workspace, size_t workspace_bytes,
                                                void* stream) {
  int32_t st = check_shape(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!q || !kv_pool || !page_table || !part)
    return fail(NYION_ERR_INVALID, "decode_q4_partial: null pointer argument");
  if (page_tokens != PAGE)
    return fail(NYION_ERR_UNSUPPORTED, "decode_q4_partial: page_tokens must be 16");
  if (batch <= 0 || max_pages <= 0 || n_pool_pages <= 0)
    return fail(NYION_ERR_INVALID, "decode_q4_partial: batch, max_pages, n_pool_pages must be > 0");
  if (reinterpret_cast<uintptr_t>(kv_pool) % 16)
    return fail(NYION_ERR_INVALID, "decode_q4_partial: kv_pool must be 16-byte aligned");
  const size_t need = ws_layout(batch).total;
  if (!workspace) {
    st = internal_workspace(need, &workspace);
    if (st) return st;
  } else if (workspace_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "decode_q4_partial: workspace %zu < %zu", workspace_bytes, need);
  }
  Params p{};
  p.pool = kv_pool;
  p.u_begin = u_begin;
  p.u_end = u_end;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  return launch_partial(p, batch, tok_begin, tok_end, q, part, page_table, workspace,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int32_t nyion_attn_lse_combine(const float* parts, int32_t n_parts, int64_t rows,
                                          int32_t head_dim, float* out, void* stream) {
  if (!parts || !out || n_parts <= 0 || rows <= 0)
    return fail(NYION_ERR_INVALID, "lse_combine: bad arguments");
  if (head_dim != HD) return fail(NYION_ERR_UNSUPPORTED, "lse_combine: head_dim must be 64");
  lse_combine_kernel<<<(unsigned)((rows + 15) / 16), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      parts, n_parts, rows, out);
  return check_cuda(cudaGetLastError(), "lse_combine launch");
}

extern "C" int32_t nyion_attn_decode_q4_window_ring(
    const float* q, const uint8_t* kv_pool, int64_t n_pool_pages, const int32_t* page_table,
    int32_t max_pages, const int32_t* seq_lens, const float* ring, int32_t ring_tokens,
    int32_t window, float* out, int32_t batch, int32_t n_heads, int32_t n_kv_heads,
    int32_t head_dim, int32_t page_tokens, float scale, void* workspace, size_t workspace_bytes,
    void* stream) {
  int32_t st = check_shape(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!q || !kv_pool || !page_table || !seq_lens || !ring || !out)
    return fail(NYION_ERR_INVALID, "decode_q4_window_ring: null pointer argument");
  if (ring_tokens <= 0 || window <= 0 || batch <= 0)
    return fail(NYION_ERR_INVALID, "decode_q4_window_ring: ring_tokens, window, batch must be > 0");
  // workspace: [q4 partial workspace][2 partial arrays of batch*H*(HD+2) floats][tok ranges]
  // (the documented size; the fused ring reduce writes `out` directly and leaves the
  // partial arrays unused)
  const size_t q4ws = ws_layout(batch).total;
  const size_t rows = (size_t)batch * n_heads;
  const size_t parts_bytes = 2 * rows * (HD + 2) * sizeof(float);
  const size_t range_bytes = 2 * (size_t)batch * sizeof(int32_t);
  const size_t need = q4ws + parts_bytes + range_bytes;
  if (!workspace) {
    st = internal_workspace(need, &workspace);
    if (st) return st;
  } else if (workspace_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "decode_q4_window_ring: workspace %zu < %zu", workspace_bytes, need);
  }
  if (ring_tokens > RING_MAX)
    return fail(NYION_ERR_UNSUPPORTED, "decode_q4_window_ring: ring_tokens %d > %d", ring_tokens, RING_MAX);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  float* parts = reinterpret_cast<float*>(w + q4ws);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Params p{};
  p.pool = kv_pool;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.seq_lens = seq_lens;
  p.window = window;
  p.ring_tokens = ring_tokens;
  const float sc = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim));
  p.qscale = sc * 1.4426950408889634f;
  RingArgs ra{};
  ra.q = q;
  ra.ring = ring;
  ra.seq_lens = seq_lens;
  ra.ring_tokens = ring_tokens;
  ra.window = window;
  ra.qscale = p.qscale;
  return launch_partial(p, batch, nullptr, nullptr, q, parts, page_table, w, s, out, ra);
}


// ---- split-KV decode with the exchange fused into the reduce ---------------

extern "C" size_t nyion_attn_splitkv_mailbox_bytes(int32_t batch, int32_t n_heads) {
  if (batch <= 0 || n_heads <= 0) return 0;
  return q4::mbox_bytes(batch * n_heads);
}

extern "C" int32_t nyion_attn_mailbox_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(NYION_ERR_INVALID, "mailbox_alloc: bad arguments");
  *ptr = nullptr;
  int32_t st = check_cuda(cudaMalloc(ptr, bytes), "cudaMalloc(mailbox)");
  if (st) return st;
  st = check_cuda(cudaMemset(*ptr, 0, bytes), "cudaMemset(mailbox)");
  if (st) {
    cudaFree(*ptr);
    *ptr = nullptr;
  }
  return st;
}

extern "C" int32_t nyion_attn_mailbox_free(void* ptr) {
  return check_cuda(cudaFree(ptr), "cudaFree(mailbox)");
}

extern "C" int32_t nyion_attn_ipc_handle(void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return fail(NYION_ERR_INVALID, "ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  int32_t st = check_cuda(cudaIpcGetMemHandle(&h, dev_ptr), "cudaIpcGetMemHandle");
  if (st) return st;
  memcpy(handle_out, &h, sizeof(h));
  return NYION_OK;
}

extern "C" int32_t nyion_attn_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return fail(NYION_ERR_INVALID, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" int32_t nyion_attn_ipc_close(void* dev_ptr) {
  return check_cuda(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
}

extern "C" int32_t nyion_attn_decode_q4_splitkv(
    const float* q, const uint8_t* kv_pool, int64_t n_pool_pages, const int32_t* page_table,
    int32_t max_pages, int32_t u_begin, int32_t u_end, float* out, int32_t batch, int32_t n_heads,
    int32_t n_kv_heads, int32_t head_dim, int32_t page_tokens, float scale, void* const* mailboxes,
    int32_t world, int32_t rank, int32_t timeout_ms, void* workspace, size_t workspace_bytes,
    void* stream) {
  int32_t st = check_shape(n_heads, n_kv_heads, head_dim);
  if (st) return st;
  if (!q || !kv_pool || !page_table || !out || !mailboxes)
    return fail(NYION_ERR_INVALID, "decode_q4_splitkv: null pointer argument");
  if (page_tokens != PAGE) return fail(NYION_ERR_UNSUPPORTED, "decode_q4_splitkv: page_tokens must be 16");
  if (batch <= 0 || batch > MAX_SEQS || max_pages <= 0 || n_pool_pages <= 0)
    return fail(NYION_ERR_INVALID, "decode_q4_splitkv: batch must be in [1, %d]; max_pages, n_pool_pages > 0",
                MAX_SEQS);
  if (world < 1 || world > MAX_RANKS || rank < 0 || rank >= world)
    return fail(NYION_ERR_INVALID, "decode_q4_splitkv: rank %d of world %d (at most %d ranks)", rank, world,
                MAX_RANKS);
  if (reinterpret_cast<uintptr_t>(kv_pool) % 16)
    return fail(NYION_ERR_INVALID, "decode_q4_splitkv: kv_pool must be 16-byte aligned");
  Exchange ex{};
  for (int r = 0; r < world; ++r) {
    if (!mailboxes[r]) return fail(NYION_ERR_INVALID, "decode_q4_splitkv: mailbox of rank %d is null", r);
    ex.mbox[r] = static_cast<uint8_t*>(mailboxes[r]);
  }
  ex.world = world;
  ex.rank = rank;
  ex.rows = batch * n_heads;
  ex.timeout_ns = (long long)(timeout_ms > 0 ? timeout_ms : 2000) * 1000000LL;
  const size_t need = ws_layout(batch).total;
  if (!workspace) {
    st = internal_workspace(need, &workspace);
    if (st) return st;
  } else if (workspace_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "decode_q4_splitkv: workspace %zu < %zu", workspace_bytes, need);
  }
  Params p{};
  p.pool = kv_pool;
  p.u_begin = u_begin;
  p.u_end = u_end;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  // the partial buffer is not written in exchange mode; the CTA partials go
  // to the workspace and the combined rows to `out`
  return launch_partial(p, batch, nullptr, nullptr, q, out, page_table, workspace,
                        static_cast<cudaStream_t>(stream), out, RingArgs{}, ex);
}
