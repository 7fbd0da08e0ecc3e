// decode_q4.cu — the 4-bit KV path: block quantizer / dequantizer, the Q4
// paged decode with its split-KV merge (and, across GPUs, the exchange of the
// ranks' partials) inside the same launch, the fp32 ring partial of config 3,
// and the log-sum-exp partial combine.
//
// Block format (swamp-engine/src/cache.rs:637-663, 375-394): 32 values ->
// 20 bytes [f16 d][f16 dmin][16 bytes of nibbles], element i in byte i/2,
// low nibble for even i; d = absmax / 7, q = clamp(round((x - dmin) / d), 0, 15),
// dequant x' = f32(d) * q + f32(dmin).
//
// Q4 decode on B200.  A nibble n placed in the low mantissa bits of an fp16
// with a zero exponent field is the subnormal n * 2^-24 (bits 0-3) or
// n * 2^-20 (bits 4-7): one LOP3 (a mask) per pair of values, no offset to
// cancel, and the tensor cores multiply subnormal fp16 inputs exactly.  A
// 32-bit word of nibbles gives four fp16x2 registers with one shift and four
// masks.  The block's dot product  sum q_i (d n_i + dmin)  is
//   d * 2^16 * sum q'_i n'_i + dmin * sum q_i
// with q'_i = q_i * 2^8 (low nibbles) or 2^4 (high nibbles), so that every
// product q'_i n'_i is q_i n_i 2^-16, on mma.sync m16n8k16 f16 with fp32
// accumulation (q' split into fp16 hi + lo rows); the per-token factors and
// the dmin term are a per-score fix-up.  P.V:  o = sum_t (p_t d_t) n_t +
// sum_t p_t dmin_t  per block, with p d split into fp16 hi + lo rows (A) and
// the V nibbles as subnormal B fragments built in registers straight from two
// tokens' nibble words (one PRMT per pair of halfwords); the powers of two of
// the nibble positions are restored on the output.  The dims of the K side
// are visited in a fixed permutation (pairs (0,4), (1,5), (2,6), (3,7) of each
// 8-value group) that q shares; the V side's output column c of n-tile
// (block, j) is dim 32 block + 4 c + j.
//
// Work split: the (sequence, 64-token chunk) units of a call are flattened
// and cut into equal contiguous ranges, one persistent CTA per SM.  A CTA
// has one producer warp (whole 5 KB pages by bulk copy into a 4-stage ring)
// and 16 consumer warps in two groups that take alternate stages (stage s
// always goes to group s % 2); within a group, warp = (KV head, 32-token
// half of the chunk) computes its tokens for the 8 query heads of its KV
// head.  Every shared-memory access of the chunk loop is a per-lane base plus
// a constant: the V tile and the per-token factor table are padded (144- and
// 48-byte rows) instead of swizzled, which keeps ldmatrix and the 16-byte
// stores free of bank conflicts.
//
// Merge: at the end of a sequence's chunks the 4 warps of each KV head fold
// their partials in shared memory and the CTA writes one partial per
// (sequence, query head).  A sequence covered by several CTAs is merged in the
// same launch by the last CTA to finish: CTAs count in per group of about
// sqrt(n) CTAs (acq_rel atomic after a CTA barrier, no waiting), the last of
// a group merges the group's partials, and the last group to finish merges
// the group partials and writes the result — the (o/l, m, l) partial, the
// output, or, across GPUs, this rank's rows sent to every rank's mailbox
// over peer memory, the other ranks' rows awaited (bounded wait) and the
// combined output written.  One launch per call.
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
// Q4 paged decode with the split-KV merge (and the rank exchange) in-launch
// ============================================================================

#ifndef NYION_Q4_GROUPS
#define NYION_Q4_GROUPS 2
#endif
constexpr int GROUPS = NYION_Q4_GROUPS; // consumer groups: stage s is consumed by group s % GROUPS
constexpr int STAGES = GROUPS == 2 ? 8 : 6;   // 20 KB each
constexpr int NCW = GROUPS * NKV * 2;   // consumer warps: group x KV head x 32-token half
constexpr int NCT = NCW * 32;           // consumer threads
#ifndef NYION_Q4_PRODUCERS
#define NYION_Q4_PRODUCERS 1
#endif
// producer warps: producer w copies the chunks k = w (mod NPROD), each its own
// chain of stages and page-id ring.  Independent copy pipelines stream more
// bytes per SM with no math (4 pipelines: 4.6 TB/s against 3.9 for one), but
// this kernel is bound by its consumers and the extra warps cost it issue slots
// (config 5: 118 us with 4 producers, 116 with 2, 115 with 1)
constexpr int NPROD = NYION_Q4_PRODUCERS;
constexpr int THREADS = NCT + 32 * NPROD;
constexpr int MAX_SEQS = 512;
constexpr int MAX_GRID = 1024;
constexpr int RING = 32;                // chunks whose page ids the producer stages ahead
constexpr int PAIR_STRIDE = 80;         // bytes per token pair of a warp's factor table (64 + 16)
constexpr int ROWS = NKV * GROUP;       // query heads of a sequence
constexpr int MT = ROWS * 16;           // threads of the merge mapping (16 per query head)
constexpr int CP = HD + 4;              // floats per row of a CTA partial: o[64], m, l, 2 unused
constexpr int WK_BYTES = GROUP * CP * 4;   // per-warp region: factor table, then the segment partial
static_assert(16 * PAIR_STRIDE <= WK_BYTES, "the factor table fits the per-warp region");
static_assert(STAGES % GROUPS == 0, "a stage must always be consumed by the same warps");
static_assert(STAGES % NPROD == 0, "a stage must always be filled by the same producer");
static_assert(MT == ROWS * 16 && NCT >= MT, "merge mapping: 16 threads per query head, 4 dims each");

enum : int32_t { kModePart = 0, kModeFinal = 1, kModeExchange = 2, kModeRing = 3 };

// ---- split-KV exchange over peer memory ----------------------------------
// Every rank owns a mailbox with the same layout.  A rank writes its partial
// of row r into slot [rank] of EVERY rank's mailbox (stores over NVLink) as
// 64-bit words: value bits low, the step's epoch high.  An aligned 64-bit
// store is single-copy atomic, so a reader that sees the epoch in a word sees
// its value: no fence and no separate flag (the scheme of NCCL's LL
// protocol).  A reader polls its row's words of every rank until all carry
// the epoch, then combines.  Each row's epoch is a counter kept in this
// rank's own mailbox header; buf = epoch & 1 double-buffers consecutive
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
  int32_t mode;                // kModePart / Final / Exchange / Ring
  float* part;                 // kModePart: [batch][H][HD + 2] (o / l, m natural log, l)
  float* out;                  // kModeFinal, kModeExchange: [batch][H][HD]
  float* cta_part;             // [MAX_GRID + batch][ROWS][CP]: o (relative to m), m (log2), l
  int32_t* gcnt;               // [MAX_GRID + MAX_SEQS]: arrivals [b], merge tickets [MAX_SEQS + b] (zero between calls)
  int32_t* scnt;               // [MAX_SEQS] sequence counters (zero between calls)
  int32_t* meta;               // kModeRing: [batch][2] first and last CTA covering sequence b
  int32_t* err;
  Exchange ex;
};

struct Smem {
  uint8_t kv[STAGES][STAGE_BYTES];
  // per warp: the factor table of the chunk (token pair j at j * PAIR_STRIDE:
  // K {16 d0, dmin0 - 16 d0, 16 d1, dmin1 - 16 d1} then V, each value for both
  // tokens of the pair), then at the end of a sequence its partial [GROUP][CP]
  uint8_t wk[NCW][WK_BYTES];
  uint64_t full[STAGES], empty[STAGES];
  int32_t vmask[STAGES];             // bit pg: page pg of the stage was copied
  int32_t prefix[MAX_SEQS + 1];      // flat chunk index where sequence b starts
  int32_t c0[MAX_SEQS];              // first chunk (absolute, in 64-token units) of sequence b
  int32_t beg[MAX_SEQS], end[MAX_SEQS];
  int32_t rows[NPROD][2][RING][5];   // per producer and chunk: 4 page ids (or -1 / -2), the sequence
  int32_t warp_tot[THREADS / 32];
  int32_t flag;
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

__device__ __forceinline__ void rows_finish(int32_t (*rows)[RING][5], const Params& p, const RowJob& j, int slot,
                                            int lane) {
  if (!j.valid) return;
#pragma unroll
  for (int pg = 0; pg < 4; ++pg) {
    int32_t v = j.page[pg];
    if (v == -1 || v < -2 || (v >= 0 && v >= p.n_pool_pages)) {
      record_error(p.err, kErrPageRange);
      v = -2;    // not copied: the page's tokens are masked out by the consumers
    }
    rows[slot][lane][pg] = v;
  }
  rows[slot][lane][4] = j.b;
}

__device__ __forceinline__ float2 hdr2f(uint32_t w) {   // (d, dmin) of a block header word
  return make_float2(__half2float(__ushort_as_half((unsigned short)(w & 0xffffu))),
                     __half2float(__ushort_as_half((unsigned short)(w >> 16))));
}

// dim visited at position c (0..63) of a row: pairs (0,4),(1,5),(2,6),(3,7) per 8-group
__device__ __forceinline__ int perm_dim(int c) {
  const int base = c & ~7, e = c & 7;
  return base + ((e & 1) ? 4 : 0) + (e >> 1);
}

// 2^x by the MUFU instruction (ex2.approx.ftz: relative error ~2^-22, subnormal
// results flushed to zero, 2^-inf = 0)
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
}

__device__ __forceinline__ int atom_add_acq_rel(int32_t* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// byte offset of n-tile nt's token (8 nt + g) row, relative to token g's row of
// the warp's first page
__device__ __forceinline__ constexpr int nt_off(int nt) { return (nt >> 1) * PAGE_BYTES + (nt & 1) * 8 * ROWB; }

// (O, M, L) += (Oo, Mo, Lo): two partials (o relative to m in log2 units, l)
__device__ __forceinline__ void merge_pair(float4& O, float& M, float& L, float4 Oo, float Mo, float Lo) {
  if (!(Lo > 0.f)) return;
  if (!(L > 0.f)) {
    O = Oo;
    M = Mo;
    L = Lo;
    return;
  }
  const float Mn = fmaxf(M, Mo);
  const float sa = ex2_ftz(M - Mn), sb = ex2_ftz(Mo - Mn);
  L = L * sa + Lo * sb;
  O.x = O.x * sa + Oo.x * sb;
  O.y = O.y * sa + Oo.y * sb;
  O.z = O.z * sa + Oo.z * sb;
  O.w = O.w * sa + Oo.w * sb;
  M = Mn;
}

// Merge of n partials at slots first, first + stride, ... for this thread's
// (query head r, dims d4 .. d4 + 3): o relative to M (log2), L.  The loads of
// a batch of U slots are all in flight at once; the batch's maximum is taken
// first, so that its weights are independent exponentials (no chain through
// the running maximum).
__device__ __forceinline__ void merge_slots(const Params& p, int first, int stride, int n, int r, int d4,
                                            float4& O, float& M, float& L) {
  M = -INFINITY;
  L = 0.f;
  O = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int U = 8;
  for (int j0 = 0; j0 < n; j0 += U) {
    float2 ml[U];
    float4 ov[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (j0 + u < n) {
        const float* src = p.cta_part + ((int64_t)(first + (j0 + u) * stride) * ROWS + r) * CP;
        ml[u] = __ldcg(reinterpret_cast<const float2*>(src + HD));
        ov[u] = __ldcg(reinterpret_cast<const float4*>(src + d4));
      } else {
        ml[u] = make_float2(-INFINITY, 0.f);
        ov[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float Mn = M;
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (ml[u].y > 0.f) Mn = fmaxf(Mn, ml[u].x);
    if (Mn == -INFINITY) continue;   // nothing attended so far
    const float sa = L > 0.f ? ex2_ftz(M - Mn) : 0.f;
    L *= sa;
    O.x *= sa;
    O.y *= sa;
    O.z *= sa;
    O.w *= sa;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (!(ml[u].y > 0.f)) continue;
      const float w = ex2_ftz(ml[u].x - Mn);
      L = fmaf(w, ml[u].y, L);
      O.x = fmaf(w, ov[u].x, O.x);
      O.y = fmaf(w, ov[u].y, O.y);
      O.z = fmaf(w, ov[u].z, O.z);
      O.w = fmaf(w, ov[u].w, O.w);
    }
    M = Mn;
  }
}

__device__ __forceinline__ void store_slot(const Params& p, int slot, int r, int d4, float4 O, float M, float L) {
  float* dst = p.cta_part + ((int64_t)slot * ROWS + r) * CP;
  __stcg(reinterpret_cast<float4*>(dst + d4), O);
  if (d4 == 0) __stcg(reinterpret_cast<float2*>(dst + HD), make_float2(M, L));
}

// The result of sequence b for this thread's (query head r, dims d4 .. d4+3)
// from its merged (O relative to M in log2 units, L): the partial, the
// output, or the exchange with the other ranks (step `epoch`) and the
// combined output.
__device__ __noinline__ void finish_row(const Params& p, int b, int r, int d4, float4 O, float M, float L, uint32_t epoch) {
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  const float4 o = make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
  const float mnat = L > 0.f ? M * 0.6931471805599453f : -INFINITY;   // log2 -> natural units
  const int64_t row = (int64_t)b * ROWS + r;
  if (p.mode == kModePart) {
    float* dst = p.part + row * (HD + 2);
    dst[d4] = o.x;
    dst[d4 + 1] = o.y;
    dst[d4 + 2] = o.z;
    dst[d4 + 3] = o.w;
    if (d4 == 0) {
      dst[HD] = mnat;
      dst[HD + 1] = L;
    }
    return;
  }
  if (p.mode == kModeFinal || p.ex.world == 1) {   // one rank: this partial is the result
    *reinterpret_cast<float4*>(p.out + row * HD + d4) = o;
    return;
  }
  // ---- exchange: this rank's row into every rank's mailbox (its own included);
  //      q4_exchange_kernel, launched after this kernel, waits for the ranks'
  //      rows and combines them ----
  const Exchange& ex = p.ex;
  const int buf = epoch & 1;
  const size_t slot = ((size_t)(buf * MAX_RANKS + ex.rank) * ex.rows + row) * (HD + 2);
  for (int rk = 0; rk < ex.world; ++rk) {
    uint64_t* dst = reinterpret_cast<uint64_t*>(ex.mbox[rk] + mbox_data_off(ex.rows)) + slot;
    st_word(dst + d4, o.x, epoch);
    st_word(dst + d4 + 1, o.y, epoch);
    st_word(dst + d4 + 2, o.z, epoch);
    st_word(dst + d4 + 3, o.w, epoch);
    if (d4 == 0) {
      st_word(dst + HD, mnat, epoch);
      st_word(dst + HD + 1, L, epoch);
    }
  }
}

// The epoch of row r of sequence b for this step (exchange mode with more than
// one rank): one past the counter kept in this rank's mailbox header.  Issued
// early (it is consumed only by finish_block) so that its load overlaps the merge.
__device__ __forceinline__ uint32_t row_epoch(const Params& p, int b, int r) {
  if (p.mode != kModeExchange || p.ex.world == 1) return 0u;
  const int* epochs = reinterpret_cast<const int*>(p.ex.mbox[p.ex.rank]) + (int64_t)b * ROWS;
  return (uint32_t)(*reinterpret_cast<const volatile int*>(epochs + r)) + 1u;
}

// finish_row for the rows a CTA holds (thread -> row r when `valid`, with its
// step epoch from row_epoch); in exchange mode the row's epoch counter is
// advanced after the exchange.  No other CTA touches the row in this step, and
// the next step is a later launch, so no barrier is needed around the counter.
__device__ void finish_block(const Params& p, int b, bool valid, int r, int d4, float4 O, float M, float L,
                             uint32_t epoch) {
  if (!valid) return;
  finish_row(p, b, r, d4, O, M, L, epoch);
  if (epoch != 0u && d4 == 0)
    *reinterpret_cast<volatile int*>(reinterpret_cast<int*>(p.ex.mbox[p.ex.rank]) + (int64_t)b * ROWS + r) =
        (int)epoch;
}

// Bounded wait until *c >= target (acquire at gpu scope); false on timeout.
__device__ bool wait_count(const int32_t* c, int target, long long timeout_ns) {
  const unsigned long long t0 = global_ns();
  while (true) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
    if (v >= target) return true;
    if ((long long)(global_ns() - t0) > timeout_ns) return false;
    __nanosleep(64);
  }
}

// The rest of a segment's end, after the warps' partials are in shared memory:
// the CTA's partial of sequence b (finished here when the CTA covers b alone,
// else stored for the merge), the count-in and, in the merging CTAs, the merge,
// the exchange and the output.  Called by all consumer threads.
__device__ __forceinline__ void segment_end(const Params& p, Smem& s, int b, int pb, int W, int total, int seg_hi,
                                         int end) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int mr = t >> 4, md4 = (t & 15) * 4;
  const int pe_ = s.prefix[b + 1];
  const int first_b = pb / W, last_b = (pe_ - 1) / W, n_b = last_b - first_b + 1;
  {
    // a sequence this CTA covers alone is finished here: its rows' epochs load
    // while the partials are folded
    const uint32_t ep_self = (n_b == 1 && t < MT) ? row_epoch(p, b, mr) : 0u;
    // thread t < MT -> (query head mr = KV head mr / 8, head mr % 8; dims md4 ..):
    // the partials of warps kv, kv + 4, kv + 8, ...
    constexpr int NW = NCW / NKV;
    const int kv = (mr >> 3) & (NKV - 1), hh = mr & 7;
    float ms[NW], ls[NW];
    float4 os[NW];
#pragma unroll
    for (int j = 0; j < NW; ++j) {
      const float* src = reinterpret_cast<const float*>(s.wk[kv + 4 * j]) + hh * CP;
      ms[j] = src[HD];
      ls[j] = src[HD + 1];
      os[j] = *reinterpret_cast<const float4*>(src + md4);
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < NW; ++j)
      if (ls[j] > 0.f) M = fmaxf(M, ms[j]);
    float L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < NW; ++j) {
      if (!(ls[j] > 0.f)) continue;
      const float w = ex2_ftz(ms[j] - M);
      L = fmaf(w, ls[j], L);
      O.x = fmaf(w, os[j].x, O.x);
      O.y = fmaf(w, os[j].y, O.y);
      O.z = fmaf(w, os[j].z, O.z);
      O.w = fmaf(w, os[j].w, O.w);
    }
    if (n_b == 1 && p.mode != kModeRing) finish_block(p, b, t < MT, mr, md4, O, M, L, ep_self);   // this CTA alone
    else if (t < MT) store_slot(p, blockIdx.x + b, mr, md4, O, M, L);
  }
  consumer_sync();   // partials stored (and shared partials read) before the count-in
  if (n_b > 1 && p.mode != kModeRing) {
    // Row-parallel merge: every covering CTA counts in (gcnt[b]); of the
    // eligible ones, the last R to take a merge ticket (gcnt[MAX_SEQS + b]; R =
    // the query heads, or the eligible CTAs if fewer) each merge rows j, j + R,
    // ... of the sequence once every covering CTA has counted in (all CTAs of
    // the grid are resident, one per SM, so the wait ends; it is bounded all
    // the same).  The last covering CTA is not eligible when its range goes on
    // past this sequence: it reaches b first (b's last chunks lead its range)
    // and the other CTAs reach b only at the end of theirs, so a wait there
    // would hold back its later sequences and chain the sequences' merges.
    const bool more = seg_hi < end;
    const int n_m = n_b - (min(total, (last_b + 1) * W) > pe_ ? 1 : 0);
    const int R = min(n_m, ROWS);
    if (t == 0) {
      // the arrival is a release reduction (no reply awaited); only the
      // ticket's reply is waited for
      asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(&p.gcnt[b]) : "memory");
      s.flag = more ? -1 : atomicAdd(&p.gcnt[MAX_SEQS + b], 1);
    }
    consumer_sync();
    const int ticket = s.flag;
    consumer_sync();
    if (ticket >= n_m - R) {
      const int j = ticket - (n_m - R);
      // the rows this thread finishes after the merge (thread -> merged row slot
      // t / 16, row j + (t / 16) R, dims (t % 16) 4): their epochs load meanwhile
      const int nr = (ROWS - j + R - 1) / R;
      const uint32_t ep_row = (t >> 4) < nr ? row_epoch(p, b, j + (t >> 4) * R) : 0u;
      if (t == 0 && !wait_count(&p.gcnt[b], n_b, p.mode == kModeExchange ? p.ex.timeout_ns : 2000000000LL))
        record_error(p.err, kErrWaitTimeout);
      consumer_sync();
      // thread -> partial group pg = t / 16 (covering CTAs pg, pg + 32, ...), dims d4;
      // the 32 groups are folded pairwise (lanes 16 apart, by a shuffle), then the
      // first 16 threads fold the 16 warps' partials from shared memory
      const int pg = t >> 4, d4 = (t & 15) * 4;
      uint8_t* const wk = &s.wk[0][0];   // the per-warp regions as one flat scratch area
      float4* ro = reinterpret_cast<float4*>(wk);                         // [16 warps][16] o
      float2* rml = reinterpret_cast<float2*>(wk + 16 * 16 * 16);          // [16 warps][16] (m, l)
      float4* fo = reinterpret_cast<float4*>(wk + 16 * 16 * 24);          // [rows][16] merged o
      float2* fml = reinterpret_cast<float2*>(wk + 16 * 16 * 24 + ROWS * 16 * 16);   // [rows][16]
      static_assert(16 * 16 * 24 + ROWS * 16 * 24 <= NCW * WK_BYTES,
                    "merge scratch fits the warp regions");
      for (int rs = 0; rs < nr; ++rs) {
        const int r = j + rs * R;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        float M = -INFINITY, L = 0.f;
        if (t < MT) {   // whole warps
          merge_slots(p, first_b + b + pg, 32, n_b > pg ? (n_b - pg + 31) / 32 : 0, r, d4, O, M, L);
          const float Mo = __shfl_xor_sync(0xffffffffu, M, 16), Lo = __shfl_xor_sync(0xffffffffu, L, 16);
          const float4 Oo = make_float4(__shfl_xor_sync(0xffffffffu, O.x, 16), __shfl_xor_sync(0xffffffffu, O.y, 16),
                                        __shfl_xor_sync(0xffffffffu, O.z, 16), __shfl_xor_sync(0xffffffffu, O.w, 16));
          merge_pair(O, M, L, Oo, Mo, Lo);
          if (lane < 16) {
            ro[warp * 16 + lane] = O;
            rml[warp * 16 + lane] = make_float2(M, L);
          }
        }
        consumer_sync();
        // the 16 warps' partials of the row folded by warp 0: lane (h, c) = (lane / 16,
        // lane % 16) takes dims 4c .. 4c + 3 of warps 8h .. 8h + 7, all loads at once;
        // the common maximum first, then the weighted sums (independent
        // exponentials), the two halves summed by a shuffle
        if (warp == 0) {
          const int c = lane & 15, h = lane >> 4;
          float2 mo[8];
          float4 oo[8];
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            mo[w] = rml[(8 * h + w) * 16 + c];
            oo[w] = ro[(8 * h + w) * 16 + c];
          }
          float Mx = -INFINITY;
#pragma unroll
          for (int w = 0; w < 8; ++w)
            if (mo[w].y > 0.f) Mx = fmaxf(Mx, mo[w].x);
          Mx = fmaxf(Mx, __shfl_xor_sync(0xffffffffu, Mx, 16));
          float Lx = 0.f;
          float4 Ox = make_float4(0.f, 0.f, 0.f, 0.f);
          if (Mx > -INFINITY) {
#pragma unroll
            for (int w = 0; w < 8; ++w) {
              if (!(mo[w].y > 0.f)) continue;
              const float sc = ex2_ftz(mo[w].x - Mx);
              Lx = fmaf(sc, mo[w].y, Lx);
              Ox.x = fmaf(sc, oo[w].x, Ox.x);
              Ox.y = fmaf(sc, oo[w].y, Ox.y);
              Ox.z = fmaf(sc, oo[w].z, Ox.z);
              Ox.w = fmaf(sc, oo[w].w, Ox.w);
            }
          }
          Lx += __shfl_xor_sync(0xffffffffu, Lx, 16);
          Ox.x += __shfl_xor_sync(0xffffffffu, Ox.x, 16);
          Ox.y += __shfl_xor_sync(0xffffffffu, Ox.y, 16);
          Ox.z += __shfl_xor_sync(0xffffffffu, Ox.z, 16);
          Ox.w += __shfl_xor_sync(0xffffffffu, Ox.w, 16);
          if (h == 0) {
            fo[rs * 16 + c] = Ox;
            fml[rs * 16 + c] = make_float2(Mx, Lx);
          }
        }
        consumer_sync();
      }
      // thread -> merged row slot rs = t / 16 (row j + rs R), dims d4
      const int rs = t >> 4;
      const bool valid = rs < nr;
      const float2 ml = valid ? fml[rs * 16 + (t & 15)] : make_float2(-INFINITY, 0.f);
      finish_block(p, b, valid, valid ? j + rs * R : 0, d4,
                   valid ? fo[rs * 16 + (t & 15)] : make_float4(0.f, 0.f, 0.f, 0.f), ml.x, ml.y, ep_row);
      consumer_sync();
      if (t == 0 && atom_add_acq_rel(&p.scnt[b], 1) == R - 1) {
        // the last merger resets the counters: every CTA has counted in and
        // taken its ticket, and no CTA reads them again in this launch
        __stcg(&p.gcnt[b], 0);
        __stcg(&p.gcnt[MAX_SEQS + b], 0);
        __stcg(&p.scnt[b], 0);
      }
    }
  }
}

__global__ void __launch_bounds__(THREADS, 1) decode_q4_kernel(const __grid_constant__ Params p) {
  // every access needs 16-byte alignment at most (bulk copies, ldmatrix, 16-byte
  // stores, mbarriers): the dynamic shared window provides it, and using the
  // array directly keeps the shared state space visible to the compiler
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int H = ROWS;

  if (t == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], NKV * 2);
    }
    s.abort_ = 0;
    fence_barrier_init();
  }
  // programmatic dependent launch: nothing global is read before the previous grid
  // in the stream completed; the next grid may be scheduled from here on and
  // waits for this one the same way
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // one token range for every sequence (no per-sequence arrays): the chunk
  // offsets follow without a scan
  const bool uniform = !p.seq_lens && !p.tok_begin && !p.tok_end;
  if (uniform && warp == NCW) {
    // the page-table entries of this CTA's first chunks head for L2 while the
    // prologue runs (lane l: chunk begin + l; the same split as below)
    const int lo = max(p.u_begin, 0), hi = max(p.u_end, lo);
    const int c = hi > lo ? (hi + CHUNK - 1) / CHUNK - lo / CHUNK : 0;
    const int tot = p.batch * c;
    const int w = (tot + (int)gridDim.x - 1) / (int)gridDim.x;
    const int i = (int)blockIdx.x * w + lane;
    if (c > 0 && lane < w && i < tot) {
      const int pidx = (lo / CHUNK + i % c) * 4;
      if (pidx < p.max_pages)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.table + (int64_t)(i / c) * p.max_pages + pidx));
    }
  }
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
    if (uniform) {
      const int c = hi > lo ? (hi + CHUNK - 1) / CHUNK - lo / CHUNK : 0;
      s.prefix[b] = b * c;
      if (b == p.batch - 1) s.prefix[p.batch] = p.batch * c;
    }
  }
  __syncthreads();
  if (!uniform) {
    // exclusive prefix of the chunk counts: thread t owns sequence t
    static_assert(THREADS >= MAX_SEQS + 1, "one thread per sequence in the prefix scan");
    const int b = t;
    int c = 0;
    if (b < p.batch && s.end[b] > s.beg[b]) c = (s.end[b] + CHUNK - 1) / CHUNK - s.c0[b];
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s.warp_tot[warp] = incl;
    __syncthreads();
    int woff = 0;
    for (int w = 0; w < warp; ++w) woff += s.warp_tot[w];
    if (b <= p.batch) s.prefix[b] = woff + incl - c;
    __syncthreads();
  }

  const int total = s.prefix[p.batch];
  const int W = (total + gridDim.x - 1) / gridDim.x;
  if (p.mode == kModeRing && blockIdx.x == 0) {
    for (int b = t; b < p.batch; b += THREADS) {
      const int lo = s.prefix[b], hi = s.prefix[b + 1];
      p.meta[2 * b] = hi > lo ? lo / W : 0;
      p.meta[2 * b + 1] = hi > lo ? (hi - 1) / W : -1;   // -1: empty range
    }
  }
  const int begin = blockIdx.x * W;
  const int end = min(total, begin + W);

  if (warp >= NCW) {
    // ========== producer warps: whole pages by bulk copy; producer pw copies
    // ========== the chunks k = pw + NPROD it into stages k % STAGES ==========
    const int pw = warp - NCW;
    if (begin + pw >= end) return;
    const int nit = (end - begin - pw + NPROD - 1) / NPROD;   // this producer's chunks
    int32_t (*rows)[RING][5] = s.rows[pw];
    auto chunk_of = [&](int it) { return begin + pw + NPROD * it; };
    RowJob job;
    rows_start(job, s, p, chunk_of(lane), end);
    rows_finish(rows, p, job, 0, lane);
    rows_start(job, s, p, chunk_of(RING + lane), end);
    __syncwarp();
    for (int it = 0; it < nit; ++it) {
      if ((it & (RING - 1)) == RING / 2) {
        rows_finish(rows, p, job, ((it / RING) + 1) & 1, lane);
        __syncwarp();
      } else if ((it & (RING - 1)) == 0 && it > 0) {
        rows_start(job, s, p, chunk_of(it + RING + lane), end);
      }
      const int k = pw + NPROD * it, stage = k % STAGES;
      bool ok = true;
      if (k >= STAGES) ok = mbar_wait_bounded(&s.empty[stage], (uint32_t)((k / STAGES - 1) & 1));
      if (!__all_sync(0xffffffffu, ok)) {
        record_error(p.err, kErrWaitTimeout);
        if (lane == 0) {
          atomicExch(&s.abort_, 1);
          // no copy of this producer may still be in flight when the CTA exits
          for (int c = k - NPROD; c >= 0 && c >= k - STAGES; c -= NPROD)
            mbar_wait_bounded(&s.full[c % STAGES], (uint32_t)((c / STAGES) & 1));
        }
        return;
      }
      if (lane == 0) {
        const int32_t* e = rows[(it / RING) & 1][it & (RING - 1)];
        uint32_t bytes = 0;
        int mask = 0;
#pragma unroll
        for (int pg = 0; pg < 4; ++pg)
          if (e[pg] >= 0) {
            bytes += PAGE_BYTES;
            mask |= 1 << pg;
          }
        s.vmask[stage] = mask;
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
  const int grp = warp >> 3, kvh = warp & 3, th = (warp >> 2) & 1;
  const int g = lane >> 2, tig = lane & 3;
  const int woff = th * 2 * PAGE_BYTES + kvh * PAGE_KV;   // the warp's 2 pages, its KV head
  // K B-fragments: word tig of block 0 of token g (n-tile 0)
  const int loff_k = g * ROWB + 4 + 4 * tig;
  // V B-fragments: word g / 2 of block 0 of token 2 tig (k-step 0); the lane
  // takes half g % 2 of that word from two tokens at once
  const int loff_v = PAGE * ROWB + 2 * tig * ROWB + 4 + 4 * (g >> 1);
  const uint32_t vsel = (g & 1) ? 0x7632u : 0x5410u;    // [A.b(2h), A.b(2h+1), B.b(2h), B.b(2h+1)]
  const uint32_t vsel2 = (g & 1) ? 0x0703u : 0x0501u;   // [A.b(2h+1), -, B.b(2h+1), -]
  // factor table: lane L fills pair L % 16 (tokens 2 (L % 16), + 1) with K
  // (L < 16) or V factors, from the two tokens' header words
  const int fj = lane & 15, fpart = lane >> 4;
  const int loff_f = (fj >> 3) * PAGE_BYTES + ((2 * fj) & 15) * ROWB + fpart * PAGE * ROWB;
  uint8_t* const ftw = s.wk[warp] + fj * PAIR_STRIDE + fpart * 32;
  // the lane's token pairs in the fix-up: pair 4 nt + tig
  const uint8_t* const ftr = s.wk[warp] + tig * PAIR_STRIDE;
  // merge mapping: thread -> query head r of the sequence, dims d4 .. d4 + 3
  const int mr = t >> 4, md4 = (t & 15) * 4;
  const float2 neg1 = make_float2(-1.f, -1.f);

  int i = begin;
  while (i < end) {
    const int b = seek_seq(s, p.batch, i);
    const int pb = s.prefix[b];
    const int seg_hi = min(end, s.prefix[b + 1]);
    const int sb = s.beg[b], se = s.end[b], c0b = s.c0[b];
    // q fragments, dims permuted: k-step (blk, ks) pairs dims 32blk + 8tig + {ks*2 + (0,4)} in
    // a0/a1 and {ks*2 + (1,5)} in a2/a3, hi rows 0-7 and lo rows 8-15
    uint32_t qa[2][2][4];
    float2 qs0, qs1;   // sum of the (hi + lo) q values of head g over each block, twice
    {
      const float* qp = p.q + ((int64_t)b * H + kvh * GROUP + g) * HD;
      float qsum[2];
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
          // even elements meet low nibbles (n 2^-24): q 2^8; odd ones high nibbles (n 2^-20): q 2^4
          const float se = p.qscale * 256.0f, so = p.qscale * 16.0f;
          split_f16x2(x[2 * ks] * se, x[2 * ks + 4] * se, h0, l0);
          split_f16x2(x[2 * ks + 1] * so, x[2 * ks + 5] * so, h1, l1);
          qa[blk][ks][0] = h0; qa[blk][ks][1] = l0; qa[blk][ks][2] = h1; qa[blk][ks][3] = l1;
          const float2 fh0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
          const float2 fl0 = __half22float2(*reinterpret_cast<const __half2*>(&l0));
          const float2 fh1 = __half22float2(*reinterpret_cast<const __half2*>(&h1));
          const float2 fl1 = __half22float2(*reinterpret_cast<const __half2*>(&l1));
          // sum of the q values the tensor cores see, back at scale (exact powers of two)
          sum += ((fh0.x + fl0.x) + (fh0.y + fl0.y)) * (1.0f / 256.0f) +
                 ((fh1.x + fl1.x) + (fh1.y + fl1.y)) * (1.0f / 16.0f);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        qsum[blk] = sum;
      }
      qs0 = make_float2(qsum[0], qsum[0]);
      qs1 = make_float2(qsum[1], qsum[1]);
    }
    // O accumulators: n-tile (blk, j) column c = dim 32 blk + 4 c + j; rows g (P' hi)
    // and g + 8 (P' lo) of head g
    float o[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) o[nt][j] = 0.f;
    // per V block: sum_t p_t dmin, and sum_t p_t, for this lane's even / odd tokens
    float2 cb0 = make_float2(0.f, 0.f), cb1 = make_float2(0.f, 0.f), l2 = make_float2(0.f, 0.f);
    float m = -INFINITY;   // reference max (log2 units) of head g

    int k = i - begin;
    k += (grp - k % GROUPS + GROUPS) % GROUPS;   // this group's chunks: k = grp (mod GROUPS)
    for (; k < seg_hi - begin; k += GROUPS) {
      const int stage = k % STAGES;
      if (!s.abort_) {
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(&s.full[stage], (uint32_t)((k / STAGES) & 1)))) {
          record_error(p.err, kErrWaitTimeout);
          if (lane == 0) atomicExch(&s.abort_, 1);
        }
      }
      const int chunk = c0b + (begin + k - pb);
      const int pos0 = chunk * CHUNK + 32 * th;         // absolute position of this warp's token 0
      const int vm = (s.vmask[stage] >> (2 * th)) & 3;  // this warp's two pages were copied
      // the body runs whenever the range meets the warp's tokens; missing pages
      // (rare: bad page ids) go through the masking path like range ends
      const bool any = (pos0 < se) && (pos0 + 32 > sb);
      const bool inner = vm == 3 && (pos0 >= sb) && (pos0 + 32 <= se);   // no token of this warp is masked
      if (any) {
        const uint8_t* const kb = s.kv[stage] + woff;
        // ---- factor table: pair fj's K (or V) block factors ----
        {
          const uint8_t* const hr = kb + loff_f;
          const uint32_t wa0 = *reinterpret_cast<const uint32_t*>(hr);            // token 2 fj, block 0
          const uint32_t wa1 = *reinterpret_cast<const uint32_t*>(hr + BLK);      // token 2 fj, block 1
          const uint32_t wb0 = *reinterpret_cast<const uint32_t*>(hr + ROWB);     // token 2 fj + 1
          const uint32_t wb1 = *reinterpret_cast<const uint32_t*>(hr + ROWB + BLK);
          const float2 fa0 = hdr2f(wa0), fa1 = hdr2f(wa1), fb0 = hdr2f(wb0), fb1 = hdr2f(wb1);
          float2 d0 = make_float2(fa0.x, fb0.x), dm0 = make_float2(fa0.y, fb0.y);
          float2 d1 = make_float2(fa1.x, fb1.x), dm1 = make_float2(fa1.y, fb1.y);
          if (!inner) {   // zero factors for masked tokens (their stage bytes may be stale)
            const int p0 = pos0 + 2 * fj;
            const bool pv = (vm >> (fj >> 3)) & 1;
            const bool l0 = pv && p0 >= sb && p0 < se, l1 = pv && p0 + 1 >= sb && p0 + 1 < se;
            if (!l0) d0.x = dm0.x = d1.x = dm1.x = 0.f;
            if (!l1) d0.y = dm0.y = d1.y = dm1.y = 0.f;
          }
          // K: {2^16 d, dmin} (the scores' nibble products carry 2^-16); V: {d, dmin};
          // each value for both tokens of the pair
          const float2 sc = fpart ? make_float2(1.f, 1.f) : make_float2(65536.f, 65536.f);
          const float2 a0 = __fmul2_rn(d0, sc), a1 = __fmul2_rn(d1, sc);
          *reinterpret_cast<float4*>(ftw) = make_float4(a0.x, a0.y, dm0.x, dm0.y);
          *reinterpret_cast<float4*>(ftw + 16) = make_float4(a1.x, a1.y, dm1.x, dm1.y);
        }
        __syncwarp();   // the factor table is complete
        // ---- S = Q K^T per n-tile of 8 tokens, fixed up at once into
        //      d = score - mref for the lane's tokens 8 nt + 2 tig + (0, 1) ----
        const float mref = m == -INFINITY ? 0.f : m;    // nothing attended yet: scores as they are
        const float2 negm = make_float2(-mref, -mref);
        float2 dv[4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          float sc[2][4];
#pragma unroll
          for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[blk][j] = 0.f;
            const uint32_t w = *reinterpret_cast<const uint32_t*>(kb + loff_k + nt_off(nt) + blk * BLK), w8 = w >> 8;
            mma_f16(sc[blk], qa[blk][0], w & 0x000F000Fu, w & 0x00F000F0u);
            mma_f16(sc[blk], qa[blk][1], w8 & 0x000F000Fu, w8 & 0x00F000F0u);
          }
          // sum q' n' per block, hi + lo rows, both tokens
          const float2 t0 = __fadd2_rn(make_float2(sc[0][0], sc[0][1]), make_float2(sc[0][2], sc[0][3]));
          const float2 t1 = __fadd2_rn(make_float2(sc[1][0], sc[1][1]), make_float2(sc[1][2], sc[1][3]));
          const float4 fk0 = *reinterpret_cast<const float4*>(ftr + nt * 4 * PAIR_STRIDE);        // a0 | c0
          const float4 fk1 = *reinterpret_cast<const float4*>(ftr + nt * 4 * PAIR_STRIDE + 16);   // a1 | c1
          float2 x = __ffma2_rn(make_float2(fk1.z, fk1.w), qs1, negm);
          x = __ffma2_rn(make_float2(fk0.z, fk0.w), qs0, x);
          x = __ffma2_rn(make_float2(fk1.x, fk1.y), t1, x);
          dv[nt] = __ffma2_rn(make_float2(fk0.x, fk0.y), t0, x);
        }
        if (!inner) {   // the range starts or ends, or a page is missing, inside this warp's 32 tokens
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            const int pos = pos0 + 8 * nt + 2 * tig;
            const bool pv = (vm >> (nt >> 1)) & 1;
            if (!(pv && pos >= sb && pos < se)) dv[nt].x = -INFINITY;
            if (!(pv && pos + 1 >= sb && pos + 1 < se)) dv[nt].y = -INFINITY;
          }
        }
        // ---- online softmax.  p = 2^d is taken at once against the current
        //      reference max (d <= 2 in almost every chunk); the chunk max,
        //      reduced over the lanes meanwhile, only decides whether the
        //      reference moves (when d passes 2, so that p <= 4), in which case
        //      the state is rescaled and p recomputed.  The branch is taken by
        //      the whole warp when any of its heads moves (heads that do not
        //      move scale by 1), so that it never diverges ----
        float2 pp[4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) pp[nt] = make_float2(ex2_ftz(dv[nt].x), ex2_ftz(dv[nt].y));
        float mx = fmaxf(dv[0].x, dv[0].y);
#pragma unroll
        for (int nt = 1; nt < 4; ++nt) mx = fmaxf(mx, fmaxf(dv[nt].x, dv[nt].y));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const bool moves = mx > 2.0f || (m == -INFINITY && mx > -INFINITY);
        if (__any_sync(0xffffffffu, moves)) {
          const float sh = moves ? mx : 0.f;
          const float al = moves ? (m == -INFINITY ? 0.f : ex2_ftz(-mx)) : 1.f;
          const float2 al2 = make_float2(al, al);
          l2 = __fmul2_rn(l2, al2);
          cb0 = __fmul2_rn(cb0, al2);
          cb1 = __fmul2_rn(cb1, al2);
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) {
            const float2 a = __fmul2_rn(make_float2(o[nt][0], o[nt][1]), al2);
            const float2 c = __fmul2_rn(make_float2(o[nt][2], o[nt][3]), al2);
            o[nt][0] = a.x; o[nt][1] = a.y; o[nt][2] = c.x; o[nt][3] = c.y;
          }
          if (moves) m = mref + mx;
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) pp[nt] = make_float2(ex2_ftz(dv[nt].x - sh), ex2_ftz(dv[nt].y - sh));
        }
        // ---- per V block: P'_blk = p d_V (the A operand, hi + lo) and the dmin
        //      term, then O += P'_blk V'_blk with the B fragments built straight
        //      from two tokens' nibble words (one block at a time keeps fewer
        //      registers live) ----
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) l2 = __fadd2_rn(l2, pp[nt]);
        const uint8_t* const vq = kb + loff_v;
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          uint32_t pa[2][4];   // [kt]
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            const float4 fv = *reinterpret_cast<const float4*>(ftr + nt * 4 * PAIR_STRIDE + 32 + 16 * blk);   // d | dmin
            const float2 x = __fmul2_rn(pp[nt], make_float2(fv.x, fv.y));
            if (blk == 0) cb0 = __ffma2_rn(pp[nt], make_float2(fv.z, fv.w), cb0);
            else cb1 = __ffma2_rn(pp[nt], make_float2(fv.z, fv.w), cb1);
            // n-tile nt: k-step nt / 2, tokens 2 tig (+1) -> a0 / a1 (even nt) or a2 / a3 (odd nt)
            const int kt = nt >> 1, r = (nt & 1) * 2;
            const __half2 hi = __float22half2_rn(x);
            const float2 res = __ffma2_rn(__half22float2(hi), neg1, x);
            const __half2 lo = __float22half2_rn(res);
            pa[kt][r] = *reinterpret_cast<const uint32_t*>(&hi);
            pa[kt][r + 1] = *reinterpret_cast<const uint32_t*>(&lo);
          }
#pragma unroll
          for (int kt = 0; kt < 2; ++kt) {
            const uint8_t* const vw = vq + kt * PAGE_BYTES + blk * BLK;
            const uint32_t w00 = *reinterpret_cast<const uint32_t*>(vw);              // token 2 tig
            const uint32_t w01 = *reinterpret_cast<const uint32_t*>(vw + ROWB);       // token 2 tig + 1
            const uint32_t w10 = *reinterpret_cast<const uint32_t*>(vw + 8 * ROWB);   // token 2 tig + 8
            const uint32_t w11 = *reinterpret_cast<const uint32_t*>(vw + 9 * ROWB);   // token 2 tig + 9
            // byte 2h (dims 4g, 4g + 1) and byte 2h + 1 (dims 4g + 2, 4g + 3) of each
            // token's halfword, the first token in the low half of the register
            const uint32_t u0 = __byte_perm(w00, w01, vsel), u1 = __byte_perm(w10, w11, vsel);
            const uint32_t v0 = __byte_perm(w00, w01, vsel2), v1 = __byte_perm(w10, w11, vsel2);
            mma_f16(o[4 * blk + 0], pa[kt], u0 & 0x000F000Fu, u1 & 0x000F000Fu);
            mma_f16(o[4 * blk + 1], pa[kt], u0 & 0x00F000F0u, u1 & 0x00F000F0u);
            mma_f16(o[4 * blk + 2], pa[kt], v0 & 0x000F000Fu, v1 & 0x000F000Fu);
            mma_f16(o[4 * blk + 3], pa[kt], v0 & 0x00F000F0u, v1 & 0x00F000F0u);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[stage]);
    }

    // ---- segment end: the 2 GROUPS warps of each KV head (groups x token
    //      halves) fold their partials in shared memory into the CTA's partial ----
    float l = l2.x + l2.y;
    float cbs[2] = {cb0.x + cb0.y, cb1.x + cb1.y};
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      cbs[blk] += __shfl_xor_sync(0xffffffffu, cbs[blk], 1);
      cbs[blk] += __shfl_xor_sync(0xffffffffu, cbs[blk], 2);
    }
    consumer_sync();                    // every warp is done with its factor table
    {
      float* mine = reinterpret_cast<float*>(s.wk[warp]);   // [GROUP][CP]
#pragma unroll
      for (int blk = 0; blk < 2; ++blk)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e)
            // j even: low nibbles (n 2^-24), j odd: high nibbles (n 2^-20)
            mine[g * CP + 32 * blk + 8 * tig + 4 * e + j] =
                fmaf(o[4 * blk + j][e] + o[4 * blk + j][2 + e], (j & 1) ? 1048576.0f : 16777216.0f, cbs[blk]);
      if (tig == 0) {
        mine[g * CP + HD] = m;
        mine[g * CP + HD + 1] = l;
      }
    }
    consumer_sync();
    segment_end(p, s, b, pb, W, total, seg_hi, end);
    i = seg_hi;
  }
  // sequences with nothing to attend: CTA 0 writes their (empty) results
  if (blockIdx.x == 0 && p.mode != kModeRing) {
    for (int b = 0; b < p.batch; ++b)
      if (s.prefix[b + 1] == s.prefix[b])
        finish_block(p, b, t < MT, mr, md4, make_float4(0.f, 0.f, 0.f, 0.f), -INFINITY, 0.f,
                     t < MT ? row_epoch(p, b, mr) : 0u);
  }
}

// ============================================================================
// config 3: the fp32 ring tokens and the reduce of the decode's CTA partials
// ============================================================================
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

constexpr int RU = 20;   // CTA partials loaded per round trip in the ring reduce

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
        const float* src = cta_part + ((((int64_t)c + b) * NKV + kvh) * GROUP + hh) * CP;
        ml[u] = __ldcg(reinterpret_cast<const float2*>(src + HD));
        ov[u] = __ldcg(reinterpret_cast<const float2*>(src) + lane);
      } else {
        ml[u] = make_float2(-INFINITY, 0.f);
        ov[u] = make_float2(0.f, 0.f);
      }
    }
    // the batch's maximum first: its weights are independent exponentials
    float Mn = M;
#pragma unroll
    for (int u = 0; u < RU; ++u)
      if (ml[u].y > 0.f) Mn = fmaxf(Mn, ml[u].x);
    if (Mn == -INFINITY) continue;
    const float sa = L > 0.f ? ex2_ftz(M - Mn) : 0.f;
    L *= sa;
    o0 *= sa;
    o1 *= sa;
#pragma unroll
    for (int u = 0; u < RU; ++u) {
      if (!(ml[u].y > 0.f)) continue;
      const float w = ex2_ftz(ml[u].x - Mn);
      L = fmaf(w, ml[u].y, L);
      o0 = fmaf(w, ov[u].x, o0);
      o1 = fmaf(w, ov[u].y, o1);
    }
    M = Mn;
  }
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  float* dst = final_out + ((int64_t)b * NKV * GROUP + kvh * GROUP + hh) * HD;
  *reinterpret_cast<float2*>(dst + 2 * lane) = make_float2(o0 * inv, o1 * inv);
}

// ============================================================================
// log-sum-exp combine: parts [G][rows][HD+2] -> out [rows][HD]
// ============================================================================
template <int D>
__global__ void lse_combine_kernel(const float* __restrict__ parts, int G, int64_t rows,
                                   float* __restrict__ out) {
  // 16 threads per row, D / 16 dims each
  constexpr int PER = D / 16;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 16) + (threadIdx.x >> 4);
  const int d0 = (threadIdx.x & 15) * PER;
  if (r >= rows) return;
  float M = -INFINITY;
  for (int gi = 0; gi < G; ++gi) {
    const float* pp = parts + ((int64_t)gi * rows + r) * (D + 2);
    if (pp[D + 1] > 0.f) M = fmaxf(M, pp[D]);
  }
  float den = 0.f;
  float acc[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) acc[j] = 0.f;
  if (M != -INFINITY) {
    for (int gi = 0; gi < G; ++gi) {
      const float* pp = parts + ((int64_t)gi * rows + r) * (D + 2);
      const float lg = pp[D + 1];
      if (!(lg > 0.f)) continue;
      const float w = lg * expf(pp[D] - M);
      den += w;
#pragma unroll
      for (int j = 0; j < PER; ++j) acc[j] = fmaf(w, pp[d0 + j], acc[j]);
    }
  }
  const float inv = den > 0.f ? 1.0f / den : 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) out[r * D + d0 + j] = acc[j] * inv;
}

// ============================================================================
// split-KV exchange: the ranks' merged rows combined (one CTA per row)
// ============================================================================
// Launched with programmatic dependent launch after decode_q4_kernel in
// exchange mode, whose merging CTAs wrote this rank's row r into slot [rank] of
// every rank's mailbox as (epoch, value) words and advanced row r's epoch
// counter.  Thread (rank rk = t / 16, dims 4 (t % 16)) polls slot [rk] of this
// rank's mailbox (bounded) until its six words carry the step's epoch; the
// ranks' rows meet in shared memory and 16 threads combine them.  All ranks'
// words are in flight at once (one round trip when they have arrived); this
// kernel's registers are its own, so the decode's chunk loop keeps its
// allocation.
__global__ void __launch_bounds__(16 * MAX_RANKS) q4_exchange_kernel(const Exchange ex, float* __restrict__ out,
                                                                     int32_t* err) {
  __shared__ float4 xo[MAX_RANKS][16];
  __shared__ float2 xml[MAX_RANKS][16];
  asm volatile("griddepcontrol.wait;" ::: "memory");   // the decode's words and epoch counters are written
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int t = threadIdx.x, rk = t >> 4, d4 = (t & 15) * 4;
  const int64_t row = blockIdx.x;
  const uint32_t epoch = (uint32_t)(*reinterpret_cast<const volatile int*>(
      reinterpret_cast<const int*>(ex.mbox[ex.rank]) + row));
  const int buf = epoch & 1;
  if (rk < ex.world) {
    const uint64_t* src = reinterpret_cast<const uint64_t*>(ex.mbox[ex.rank] + mbox_data_off(ex.rows)) +
                          ((size_t)(buf * MAX_RANKS + rk) * ex.rows + row) * (HD + 2);
    const unsigned long long t0 = global_ns();
    uint32_t spins = 0;
    float4 ov = make_float4(0.f, 0.f, 0.f, 0.f);
    float2 ml = make_float2(-INFINITY, 0.f);
    while (true) {
      uint64_t w[6];
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = ld_word(src + d4 + i);
      w[4] = ld_word(src + HD);
      w[5] = ld_word(src + HD + 1);
      bool here = true;
#pragma unroll
      for (int i = 0; i < 6; ++i) here &= (uint32_t)(w[i] >> 32) == epoch;
      if (here) {
        ov = make_float4(__uint_as_float((uint32_t)w[0]), __uint_as_float((uint32_t)w[1]),
                         __uint_as_float((uint32_t)w[2]), __uint_as_float((uint32_t)w[3]));
        ml = make_float2(__uint_as_float((uint32_t)w[4]), __uint_as_float((uint32_t)w[5]));
        break;
      }
      if (++spins > 32) __nanosleep(64);
      if ((long long)(global_ns() - t0) > ex.timeout_ns) {
        record_error(err, kErrWaitTimeout);   // this rank's row is left out
        break;
      }
    }
    xo[rk][t & 15] = ov;
    xml[rk][t & 15] = ml;
  }
  __syncthreads();
  if (t < 16) {
    float Mr = -INFINITY, den = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < ex.world; ++k) {
      const float2 ml = xml[k][t];
      if (!(ml.y > 0.f)) continue;
      const float4 ov = xo[k][t];
      const float Mn = fmaxf(Mr, ml.x);
      const float sa = expf(Mr - Mn), sb = ml.y * expf(ml.x - Mn);
      den = den * sa + sb;
      acc.x = acc.x * sa + ov.x * sb;
      acc.y = acc.y * sa + ov.y * sb;
      acc.z = acc.z * sa + ov.z * sb;
      acc.w = acc.w * sa + ov.w * sb;
      Mr = Mn;
    }
    const float ir = den > 0.f ? 1.0f / den : 0.f;
    *reinterpret_cast<float4*>(out + row * HD + d4) = make_float4(acc.x * ir, acc.y * ir, acc.z * ir, acc.w * ir);
  }
}

size_t smem_bytes() { return sizeof(Smem); }
static_assert(sizeof(Smem) <= 227 * 1024, "decode_q4 shared memory must fit one CTA per SM");

// Workspace: [counters: group (MAX_GRID + MAX_SEQS) | sequence (MAX_SEQS)]
// [meta: batch x 2][CTA partials: (MAX_GRID + batch) x ROWS x CP floats].
// The counter block has a fixed size and must be zero before the first call;
// the kernel leaves it at zero.
struct WsLayout {
  size_t gcnt, scnt, meta, cta_part, total;
};

WsLayout ws_layout(int batch) {
  const int b = batch < MAX_SEQS ? batch : MAX_SEQS;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  WsLayout w;
  w.gcnt = 0;
  w.scnt = al((size_t)(MAX_GRID + MAX_SEQS) * sizeof(int32_t));
  w.meta = w.scnt + al((size_t)MAX_SEQS * sizeof(int32_t));
  w.cta_part = w.meta + al((size_t)b * 2 * sizeof(int32_t));
  w.total = w.cta_part + al((size_t)(MAX_GRID + b) * ROWS * CP * sizeof(float));
  return w;
}

size_t counter_bytes() { return ws_layout(1).meta; }

bool specialised(int32_t n_heads, int32_t n_kv_heads, int32_t head_dim) {
  return n_kv_heads == NKV && n_heads == NKV * GROUP && head_dim == HD;
}

int32_t check_shape(int32_t n_heads, int32_t n_kv_heads, int32_t head_dim) {
  if (n_kv_heads != NKV || n_heads != NKV * GROUP || head_dim != HD)
    return fail(NYION_ERR_UNSUPPORTED,
                "the 4-bit kernels of this build take 32 query heads, 4 KV heads, head_dim 64 "
                "(got %d/%d/%d)", n_heads, n_kv_heads, head_dim);
  return NYION_OK;
}

// The library-owned workspace (when `ws` is null) or a check of the caller's.
int32_t resolve_workspace(void** ws, size_t ws_bytes, size_t need, cudaStream_t stream, const char* who) {
  if (!*ws) return internal_workspace(need, ws, kWsCounters, counter_bytes(), stream);
  if (ws_bytes < need) return fail(NYION_ERR_WORKSPACE, "%s: workspace %zu < %zu", who, ws_bytes, need);
  return NYION_OK;
}

// One decode launch per MAX_SEQS sequences (mode Part / Final / Exchange), or,
// in ring mode, the decode then the ring + reduce kernel.
int32_t launch_partial(Params base, int batch, const int32_t* tok_begin, const int32_t* tok_end,
                       const float* q, void* ws, cudaStream_t stream, RingArgs ra = RingArgs{}) {
  DeviceInfo* dev = nullptr;
  int32_t st = device_info(&dev);
  if (st) return st;
  const size_t smem = smem_bytes();
  int occ = 1;
  st = kernel_setup(reinterpret_cast<const void*>(decode_q4_kernel), smem, THREADS, &occ);
  if (st) return st;
  const int grid = dev->num_sms * occ < MAX_GRID ? dev->num_sms * occ : MAX_GRID;
  const WsLayout w = ws_layout(batch);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  for (int b0 = 0; b0 < batch; b0 += MAX_SEQS) {
    Params p = base;
    const int nb = batch - b0 < MAX_SEQS ? batch - b0 : MAX_SEQS;
    p.batch = nb;
    p.tok_begin = tok_begin ? tok_begin + b0 : nullptr;
    p.tok_end = tok_end ? tok_end + b0 : nullptr;
    p.q = q + (int64_t)b0 * ROWS * HD;
    if (base.part) p.part = base.part + (int64_t)b0 * ROWS * (HD + 2);
    if (base.out) p.out = base.out + (int64_t)b0 * ROWS * HD;
    p.table = base.table + (int64_t)b0 * base.max_pages;
    p.seq_lens = base.seq_lens ? base.seq_lens + b0 : nullptr;
    p.gcnt = reinterpret_cast<int32_t*>(wsb + w.gcnt);
    p.scnt = reinterpret_cast<int32_t*>(wsb + w.scnt);
    p.meta = reinterpret_cast<int32_t*>(wsb + w.meta);
    p.cta_part = reinterpret_cast<float*>(wsb + w.cta_part);
    p.err = dev->err_word;
    st = check_cuda(launch_pdl(decode_q4_kernel, dim3(grid), dim3(THREADS), smem, stream, p), "decode_q4 launch");
    if (st) return st;
    if (p.mode == kModeRing) {   // config 3: ring partial + reduce in one launch (final output)
      RingArgs r = ra;
      r.q = q + (int64_t)b0 * ROWS * HD;
      r.ring = ra.ring + (int64_t)b0 * NKV * 2 * ra.ring_tokens * HD;
      r.seq_lens = ra.seq_lens + b0;
      st = check_cuda(launch_pdl(q4_reduce_ring_kernel, dim3(nb * NKV), dim3(256), 0, stream,
                                 (const float*)p.cta_part, (const int32_t*)p.meta, p.out, r),
                      "q4_reduce_ring launch");
      if (st) return st;
    }
  }
  return NYION_OK;
}

}  // namespace q4

size_t q4_counter_bytes() { return q4::counter_bytes(); }

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
  if (!specialised(n_heads, n_kv_heads, head_dim) && generic_shape_ok(n_heads, n_kv_heads, head_dim)) {
    // other shapes: the generic kernel over the 4-bit pool [pages][n_kv][K|V][16][head_dim / 32 * 20]
    if (!q || !kv_pool || !page_table || !part)
      return fail(NYION_ERR_INVALID, "decode_q4_partial: null pointer argument");
    if (page_tokens != PAGE) return fail(NYION_ERR_UNSUPPORTED, "decode_q4_partial: page_tokens must be 16");
    if (batch <= 0 || max_pages <= 0 || n_pool_pages <= 0)
      return fail(NYION_ERR_INVALID, "decode_q4_partial: batch, max_pages, n_pool_pages must be > 0");
    GenericCall c;
    c.who = "decode_q4_partial";
    c.q = q;
    c.k = kv_pool;
    c.table = page_table;
    c.max_pages = max_pages;
    c.n_pool_pages = n_pool_pages;
    c.n_heads = n_heads;
    c.n_kv = n_kv_heads;
    c.head_dim = head_dim;
    c.rows = batch;
    c.tok_begin = tok_begin;
    c.tok_end = tok_end;
    c.u_begin = u_begin;
    c.u_end = u_end;
    c.scale = scale;
    c.part_mode = 1;
    c.out = part;
    c.max_tokens = (int64_t)max_pages * PAGE;
    c.fmt = kGenQ4;
    c.layout = kGenPaged;
    return generic_decode(c, static_cast<cudaStream_t>(stream));
  }
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = resolve_workspace(&workspace, workspace_bytes, ws_layout(batch).total, s, "decode_q4_partial");
  if (st) return st;
  Params p{};
  p.pool = kv_pool;
  p.table = page_table;
  p.u_begin = u_begin;
  p.u_end = u_end;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  p.mode = kModePart;
  p.part = part;
  return launch_partial(p, batch, tok_begin, tok_end, q, workspace, s);
}

extern "C" int32_t nyion_attn_lse_combine(const float* parts, int32_t n_parts, int64_t rows,
                                          int32_t head_dim, float* out, void* stream) {
  if (!parts || !out || n_parts <= 0 || rows <= 0)
    return fail(NYION_ERR_INVALID, "lse_combine: bad arguments");
  if (head_dim != 64 && head_dim != 128) return fail(NYION_ERR_UNSUPPORTED, "lse_combine: head_dim must be 64 or 128");
  const unsigned grid = (unsigned)((rows + 15) / 16);
  if (head_dim == 64)
    lse_combine_kernel<64><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(parts, n_parts, rows, out);
  else
    lse_combine_kernel<128><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(parts, n_parts, rows, out);
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
  if (ring_tokens > RING_MAX)
    return fail(NYION_ERR_UNSUPPORTED, "decode_q4_window_ring: ring_tokens %d > %d", ring_tokens, RING_MAX);
  // workspace: [q4 decode workspace][2 partial arrays of batch*H*(HD+2) floats][tok ranges]
  // (the documented size; the fused ring reduce writes `out` directly and leaves the
  // partial arrays unused)
  const size_t q4ws = ws_layout(batch).total;
  const size_t rows = (size_t)batch * n_heads;
  const size_t parts_bytes = 2 * rows * (HD + 2) * sizeof(float);
  const size_t range_bytes = 2 * (size_t)batch * sizeof(int32_t);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = resolve_workspace(&workspace, workspace_bytes, q4ws + parts_bytes + range_bytes, s, "decode_q4_window_ring");
  if (st) return st;
  Params p{};
  p.pool = kv_pool;
  p.table = page_table;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.seq_lens = seq_lens;
  p.window = window;
  p.ring_tokens = ring_tokens;
  p.qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  p.mode = kModeRing;
  p.out = out;
  RingArgs ra{};
  ra.q = q;
  ra.ring = ring;
  ra.seq_lens = seq_lens;
  ra.ring_tokens = ring_tokens;
  ra.window = window;
  ra.qscale = p.qscale;
  return launch_partial(p, batch, nullptr, nullptr, q, workspace, s, ra);
}


// ---- split-KV decode: rows sent by the decode, combined by the exchange kernel ----

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
  if (!specialised(n_heads, n_kv_heads, head_dim) && generic_shape_ok(n_heads, n_kv_heads, head_dim) && world == 1) {
    // other shapes on one rank: the generic kernel's merged rows are the output
    if (!q || !kv_pool || !page_table || !out)
      return fail(NYION_ERR_INVALID, "decode_q4_splitkv: null pointer argument");
    if (page_tokens != PAGE) return fail(NYION_ERR_UNSUPPORTED, "decode_q4_splitkv: page_tokens must be 16");
    if (batch <= 0 || max_pages <= 0 || n_pool_pages <= 0 || rank != 0)
      return fail(NYION_ERR_INVALID, "decode_q4_splitkv: bad sizes or rank");
    GenericCall c;
    c.who = "decode_q4_splitkv";
    c.q = q;
    c.k = kv_pool;
    c.table = page_table;
    c.max_pages = max_pages;
    c.n_pool_pages = n_pool_pages;
    c.n_heads = n_heads;
    c.n_kv = n_kv_heads;
    c.head_dim = head_dim;
    c.rows = batch;
    c.u_begin = u_begin;
    c.u_end = u_end;
    c.scale = scale;
    c.out = out;
    c.max_tokens = (int64_t)max_pages * PAGE;
    c.fmt = kGenQ4;
    c.layout = kGenPaged;
    return generic_decode(c, static_cast<cudaStream_t>(stream));
  }
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
  Params p{};
  for (int r = 0; r < world; ++r) {
    if (!mailboxes[r]) return fail(NYION_ERR_INVALID, "decode_q4_splitkv: mailbox of rank %d is null", r);
    p.ex.mbox[r] = static_cast<uint8_t*>(mailboxes[r]);
  }
  p.ex.world = world;
  p.ex.rank = rank;
  p.ex.rows = batch * n_heads;
  p.ex.timeout_ns = (long long)(timeout_ms > 0 ? timeout_ms : 2000) * 1000000LL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = resolve_workspace(&workspace, workspace_bytes, ws_layout(batch).total, s, "decode_q4_splitkv");
  if (st) return st;
  p.pool = kv_pool;
  p.table = page_table;
  p.u_begin = u_begin;
  p.u_end = u_end;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.qscale = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  // one rank: the merged rows are the output (no exchange needed)
  p.mode = world > 1 ? kModeExchange : kModeFinal;
  p.out = out;
  st = launch_partial(p, batch, nullptr, nullptr, q, workspace, s);
  if (st || world == 1) return st;
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st) return st;
  return check_cuda(launch_pdl(q4_exchange_kernel, dim3((unsigned)(batch * n_heads)), dim3(16 * MAX_RANKS), 0, s,
                               p.ex, out, dev->err_word),
                    "q4_exchange launch");
}
