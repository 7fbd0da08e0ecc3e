// prefill_bf16.cu — causal chunked prefill over the bf16 paged KV cache on
// the 5th-generation tensor cores (tcgen05.mma, TMEM accumulators).
//
// The reference prefills one query at a time: for each prompt token t of a
// chunk it calls ops::attention with seq_len = pos_offset + t + 1
// (swamp-engine/src/executor.rs:106-138, chunks of 4096 at :185).  Here one
// launch computes a whole chunk of queries against the cache (causal mask
// t <= position) as tiles:
//
//   * M tile = 128 rows = 16 query positions x the 8 query heads of one GQA
//     group (row r = position r/8, head r%8), so one K/V tile serves 8 heads;
//   * N tile = 128 cached tokens (8 pages of 16), K = head_dim 64;
//   * S = Q K^T: 4 x tcgen05.mma (M128 N128 K16, bf16 -> fp32, both operands
//     in shared memory) into TMEM; P = softmax numerators, written by the
//     row-owning thread into TMEM as bf16 pairs; O += P V: 8 x tcgen05.mma
//     (M128 N64 K16, A = P from TMEM, B = V as an MN-major shared operand)
//     accumulating in TMEM;
//   * two softmax groups of 4 warps take alternate KV tiles (even / odd),
//     each with its own S, P and O TMEM columns and running (m, l); a row's
//     reference max only moves when a tile's max exceeds it by 2^8, and then
//     O (in TMEM) and l are rescaled; the two groups' rows are merged through
//     shared memory at the end;
//   * warps 8 and 10 copy K and V pages (TMA, 6-stage ring; page ids read a
//     block of 32 ahead), warp 9 allocates TMEM and one of its threads issues
//     the MMAs: S(j+2) as soon as group j%2 has read S(j) out of TMEM, PV(j)
//     as soon as P(j) is written, polling both so the two groups overlap;
//     the softmax group that consumed a tile releases its ring stage.
//     Every wait is bounded; TMEM is released on every path.
#include <cuda_bf16.h>
#include <math.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace prefill {

constexpr int HD = 64;
constexpr int GROUP = 8;
constexpr int PAGE = 16;
constexpr int BM = 128;                    // rows per tile
constexpr int POS = BM / GROUP;            // 16 positions per tile
constexpr int BN = 128;                    // cached tokens per KV tile
constexpr int THREADS = 352;                // 8 softmax warps, K producer, MMA, V producer
constexpr uint32_t TMEM_COLS = 512;
// TMEM columns of softmax group g: S at 128 g (fp32), O_tile at 256 + 64 g
// (fp32), P at 384 + 64 g (bf16 pairs: token 2c in the low half of column c)
constexpr uint32_t S_COL = 0, O_COL = 256, P_COL = 384;
constexpr int ROWB = HD * 2;               // 128 bytes per bf16 row
constexpr int STAGES = 6;                  // K/V ring depth (tiles in flight)

struct Smem {
  uint8_t q[BM * ROWB];          // Q tile, 16 KB
  uint8_t k[STAGES][BN * ROWB];  // K tiles, 16 KB each
  uint8_t v[STAGES][BN * ROWB];  // V tiles, 16 KB each
  uint64_t q_full, kv_full[STAGES], kv_empty[STAGES], done;
  // per softmax group: S(j) written | S(j) read out | P(j) written | PV(j) retired
  uint64_t s_ready[2], s_free[2], p_full[2], pv_done[2];
  uint32_t tmem_base;
  int32_t abort_;
};

struct Params {
  const int32_t* table;          // [max_pages] page ids of the sequence
  int32_t max_pages;
  int64_t n_pool_pages;
  int32_t n_kv;
  int64_t q_start, n_q;          // query positions [q_start, q_start + n_q)
  float sl2;                     // scale * log2(e)
  float* out;                    // [n_q][n_kv * GROUP][HD] fp32
  int32_t* err;
};

// ---- tcgen05 / descriptor helpers ------------------------------------------

// Shared-memory matrix descriptor (sm_100): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version 1 [46,48), base offset 0, layout [61,64).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;    // 128-byte swizzle
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (0u << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// A operand from TMEM (K-major rows in lanes), B from shared memory
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 8 consecutive 32-bit columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&w)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
      "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t u[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]),
        "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]),
        "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]),
        "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __uint_as_float(u[i]);
}

// 16 consecutive fp32 columns of this thread's TMEM lane (undefined until
// tmem_wait_ld16 on the same registers)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]),
        "=f"(r[7]), "=f"(r[8]), "=f"(r[9]), "=f"(r[10]), "=f"(r[11]), "=f"(r[12]), "=f"(r[13]),
        "=f"(r[14]), "=f"(r[15])
      : "r"(taddr));
}

// waits for every outstanding tcgen05.ld; the registers are tied to the wait
// so no use of them can be scheduled before it
__device__ __forceinline__ void tmem_wait_ld16(float (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+f"(r[0]), "+f"(r[1]), "+f"(r[2]), "+f"(r[3]), "+f"(r[4]), "+f"(r[5]), "+f"(r[6]),
                 "+f"(r[7]), "+f"(r[8]), "+f"(r[9]), "+f"(r[10]), "+f"(r[11]), "+f"(r[12]),
                 "+f"(r[13]), "+f"(r[14]), "+f"(r[15])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld32(float (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+f"(r[0]), "+f"(r[1]), "+f"(r[2]), "+f"(r[3]), "+f"(r[4]), "+f"(r[5]), "+f"(r[6]),
                 "+f"(r[7]), "+f"(r[8]), "+f"(r[9]), "+f"(r[10]), "+f"(r[11]), "+f"(r[12]),
                 "+f"(r[13]), "+f"(r[14]), "+f"(r[15]), "+f"(r[16]), "+f"(r[17]), "+f"(r[18]),
                 "+f"(r[19]), "+f"(r[20]), "+f"(r[21]), "+f"(r[22]), "+f"(r[23]), "+f"(r[24]),
                 "+f"(r[25]), "+f"(r[26]), "+f"(r[27]), "+f"(r[28]), "+f"(r[29]), "+f"(r[30]),
                 "+f"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// o = o * alpha + (64 fp32 columns of this thread's TMEM lane at taddr)
__device__ __forceinline__ void fold_o(float2 (&o)[HD / 2], uint32_t taddr, float alpha) {
  const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float ot[32];
    tmem_ld32(taddr + 32 * half, ot);
    tmem_wait_ld();
#pragma unroll
    for (int d = 0; d < 16; ++d)
      o[16 * half + d] = __ffma2_rn(o[16 * half + d], a2, make_float2(ot[2 * d], ot[2 * d + 1]));
  }
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
prefill_kernel(const Params p, const __grid_constant__ CUtensorMap map_q,
               const __grid_constant__ CUtensorMap map_kv) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int H = p.n_kv * GROUP;
  const int n_mt = (int)((p.n_q + POS - 1) / POS);
  // longest tiles (latest positions) first
  const int kvh = blockIdx.x % p.n_kv;
  const int mt = n_mt - 1 - blockIdx.x / p.n_kv;
  const int64_t pos0 = p.q_start + (int64_t)mt * POS;        // first absolute position of the tile
  const int64_t ctx_end = p.q_start + p.n_q;
  const int64_t kv_len = pos0 + POS < ctx_end ? pos0 + POS : ctx_end;   // tokens [0, kv_len) visible
  const int nt = (int)((kv_len + BN - 1) / BN);

  if (t == 0) {
    prefetch_tensormap(&map_q);
    prefetch_tensormap(&map_kv);
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.kv_full[i], 2);
      mbar_init(&s.kv_empty[i], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s.s_ready[g], 1);
      mbar_init(&s.s_free[g], 4);
      mbar_init(&s.p_full[g], 128);
      mbar_init(&s.pv_done[g], 1);
    }
    mbar_init(&s.done, 1);
    s.abort_ = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s.tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  // programmatic dependent launch: the next grid in the stream may start its
  // prologue now; this grid reads nothing from global memory before the
  // previous grid has completed and flushed
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*reinterpret_cast<volatile int32_t*>(&s.abort_)) return;
    if (!mbar_wait_bounded(bar, parity)) {
      record_error(p.err, kErrWaitTimeout);
      atomicExch(&s.abort_, 1);
    }
  };

  if (warp == 8 || warp == 10) {
    // ================= TMA producers: warp 8 copies K pages, warp 10 V pages =====
    const bool is_v = warp == 10;
    if (!is_v && lane == 0) {
      mbar_arrive_expect_tx(&s.q_full, BM * ROWB);
      // (x: 64 dims, head, position) box (64, 8, 16): rows = position * 8 + head
      tma_load_3d(s.q, &map_q, 0, kvh * GROUP, (int32_t)(pos0 - p.q_start), &s.q_full);
    }
    // page ids come in blocks of 32 (4 tiles), one per lane, the next block
    // loaded while the current one is in use; tile j takes lanes 8(j%4)..+7
    const int n_pages = (int)((kv_len + PAGE - 1) / PAGE);
    auto page_row = [&](int pidx) -> int32_t {         // first K row of page pidx, or -64
      if (pidx >= n_pages) return -4 * PAGE;
      const int64_t page = (pidx < p.max_pages) ? p.table[pidx] : -1;
      if (page < 0 || page >= p.n_pool_pages) {
        record_error(p.err, kErrPageRange);
        return -4 * PAGE;
      }
      return (int32_t)(((page * p.n_kv + kvh) * 2) * PAGE);
    };
    int32_t blk = page_row(lane);
    int32_t nxt = page_row(32 + lane);
    for (int j = 0; j < nt; ++j) {
      const int st = j % STAGES;
      if ((j & 3) == 0 && j > 0) {
        blk = nxt;
        nxt = page_row(32 * ((j >> 2) + 1) + lane);
      }
      const int32_t row = __shfl_sync(0xffffffffu, blk, 8 * (j & 3) + (lane & 7));
      if (j >= STAGES) wait(&s.kv_empty[st], (uint32_t)((j / STAGES - 1) & 1));
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&s.kv_full[st], BN * ROWB);
      __syncwarp();
      if (lane < BN / PAGE) {
        // rows outside the pool (negative) are zero-filled by the copy
        tma_load_2d((is_v ? s.v[st] : s.k[st]) + lane * PAGE * ROWB, &map_kv, 0, row + (is_v ? PAGE : 0),
                    &s.kv_full[st]);
      }
    }
    // no copy may still be writing shared memory when the CTA exits (matters
    // only after an aborted wait; otherwise these phases completed long ago)
    if (lane == 0) {
      if (!is_v) mbar_wait_bounded(&s.q_full, 0);
      for (int j = nt - STAGES < 0 ? 0 : nt - STAGES; j < nt; ++j)
        mbar_wait_bounded(&s.kv_full[j % STAGES], (uint32_t)((j / STAGES) & 1));
    }
  } else if (warp == 9) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t IQK = instr_desc(BM, BN, false);
      constexpr uint32_t IPV = instr_desc(BM, HD, true);
      const uint32_t qa = smem_u32(s.q);
      auto issue_qk = [&](int j) {
        const uint32_t kb = smem_u32(s.k[j % STAGES]);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          umma(tmem + S_COL + 128 * (j & 1), smem_desc(qa + ks * 32, 16, 1024), smem_desc(kb + ks * 32, 16, 1024),
               IQK, ks > 0);
      };
      // S(j+2) is computed as soon as group g has read S(j) out of TMEM, and
      // PV(j) as soon as P(j) is written, whichever comes first: the issuer
      // polls both (QK in tile order, PV in tile order), so the two softmax
      // groups work at the same time.  Two commits per tile: s_ready[g] (S
      // written) and pv_done[g] (PV retired).  A group is never more than one
      // phase ahead of a poll here.  The poll is bounded like every wait.
      wait(&s.q_full, 0);
      for (int j = 0; j < 2 && j < nt; ++j) {
        wait(&s.kv_full[j], 0);
        tc_fence_after();
        issue_qk(j);
        umma_commit(&s.s_ready[j]);
      }
      int qn = 2, pn = 0;                                // next tile for QK / for PV
      uint32_t idle = 0;
      while (pn < nt && !*reinterpret_cast<volatile int32_t*>(&s.abort_)) {
        bool progress = false;
        if (qn < nt) {
          const int g = qn & 1;
          if (mbar_try_wait(&s.s_free[g], (uint32_t)(((qn - 2) >> 1) & 1)) &&
              mbar_try_wait(&s.kv_full[qn % STAGES], (uint32_t)((qn / STAGES) & 1))) {
            tc_fence_after();
            issue_qk(qn);
            umma_commit(&s.s_ready[g]);
            ++qn;
            progress = true;
          }
        }
        {
          const int g = pn & 1;
          if (mbar_try_wait(&s.p_full[g], (uint32_t)((pn >> 1) & 1))) {
            tc_fence_after();
            const uint32_t vb = smem_u32(s.v[pn % STAGES]);
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk)
              umma_ts(tmem + O_COL + 64 * g, tmem + P_COL + 64 * g + 8 * kk,
                      smem_desc(vb + kk * 2048, 8192, 1024), IPV, (kk > 0 || pn >= 2) ? 1u : 0u);
            umma_commit(&s.pv_done[g]);
            ++pn;
            progress = true;
          }
        }
        if (progress) {
          idle = 0;
        } else if (++idle > kSpinLimit) {
          record_error(p.err, kErrWaitTimeout);
          atomicExch(&s.abort_, 1);
        } else if (idle > 64) {
          __nanosleep(32);
        }
      }
      umma_commit(&s.done);
      mbar_wait_bounded(&s.done, 0);   // every MMA has retired before TMEM is released
    }
    __syncwarp();
  } else {
    // ================= softmax groups: thread = row =================
    // O accumulates in TMEM (PV with accumulate after the group's first
    // tile); the row's reference max m only moves when a tile's max exceeds
    // it by more than 2^8, and then O and l are rescaled, so P <= 256.
    const int g = warp >> 2;                          // group: tiles j with j % 2 == g
    const int r = t & 127;                            // row = TMEM lane
    const int64_t pos = pos0 + (r >> 3);              // this row's absolute position
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    const uint32_t s_addr = lane_base + S_COL + 128 * g;
    const uint32_t o_addr = lane_base + O_COL + 64 * g;
    const uint32_t p_addr = lane_base + P_COL + 64 * g;
    float m = -INFINITY, l = 0.f;
    int i = 0;
    for (int j = g; j < nt; j += 2, ++i) {
      wait(&s.s_ready[g], (uint32_t)(i & 1));         // S(j) written
      __syncwarp();                                   // tcgen05.ld is warp-collective
      tc_fence_after();
      float sv[BN];
#pragma unroll
      for (int q = 0; q < BN / 32; ++q) tmem_ld32(s_addr + 32 * q, *reinterpret_cast<float(*)[32]>(&sv[32 * q]));
#pragma unroll
      for (int q = 0; q < BN / 32; ++q) tmem_wait_ld32(*reinterpret_cast<float(*)[32]>(&sv[32 * q]));
      // S(j) is in registers: its TMEM columns may take S(j+2) now
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.s_free[g]);
      // causal mask (token <= position) on tiles that cross this M tile's diagonal
      const int64_t t0 = (int64_t)j * BN;
      if (t0 + BN - 1 > pos0) {
        const int lim = (int)(pos - t0);
#pragma unroll
        for (int c = 0; c < BN; ++c) sv[c] = (c <= lim) ? sv[c] : -INFINITY;
      }
      float ma = max3(sv[0], sv[1], sv[2]), mb = max3(sv[3], sv[4], sv[5]);
#pragma unroll
      for (int c = 6; c < BN - 2; c += 4) {
        ma = max3(ma, sv[c], sv[c + 1]);
        mb = max3(mb, sv[c + 2], sv[c + 3]);
      }
      // scores enter the log2 domain through one FMA: p = 2^(s * scale * log2e - m)
      const float mxs = max3(ma, mb, fmaxf(sv[BN - 2], sv[BN - 1])) * p.sl2;
      float alpha = 1.f;
      const bool need = mxs > m + 8.f;                // also when m is still -inf
      if (need) {
        alpha = ex2(m - mxs);                         // 0 while nothing was visible
        m = mxs;
        l *= alpha;
      }
      const float mref = (m == -INFINITY) ? 0.f : m;  // a row with nothing visible yet: P = 0
      // P row r as bf16 pairs (token 2c in the low half of column c).  The first
      // half is computed before waiting for PV(j-2) (whose P columns it
      // overwrites), so the exponentials overlap that MMA.
      const float2 sl2v = make_float2(p.sl2, p.sl2), negm = make_float2(-mref, -mref);
      float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      auto p_words = [&](int c16, uint32_t (&w)[8]) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float2 x = __ffma2_rn(make_float2(sv[16 * c16 + 2 * e], sv[16 * c16 + 2 * e + 1]), sl2v, negm);
          x.x = ex2(x.x);
          x.y = ex2(x.y);
          acc[e & 1] = __fadd2_rn(acc[e & 1], x);
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(x.x, x.y);
          w[e] = *reinterpret_cast<const uint32_t*>(&h2);
        }
      };
      uint32_t first[4][8];
#pragma unroll
      for (int c16 = 0; c16 < 4; ++c16) p_words(c16, first[c16]);
      if (i > 0) {
        // PV of this group's previous tile has retired: its P and O columns are
        // free, O may be rescaled, and that tile's K/V stage goes back
        wait(&s.pv_done[g], (uint32_t)((i - 1) & 1));
        __syncwarp();
        tc_fence_after();
        if (r == 0) mbar_arrive(&s.kv_empty[(j - 2) % STAGES]);
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int q = 0; q < HD / 16; ++q) {
            float v[16];
            tmem_ld16(o_addr + 16 * q, v);
            tmem_wait_ld16(v);
#pragma unroll
            for (int c = 0; c < 16; ++c) v[c] *= alpha;
            tmem_st16(o_addr + 16 * q, v);
          }
        }
      }
#pragma unroll
      for (int c16 = 0; c16 < 4; ++c16) tmem_st8(p_addr + 8 * c16, first[c16]);
#pragma unroll
      for (int c16 = 4; c16 < BN / 16; ++c16) {
        uint32_t w[8];
        p_words(c16, w);
        tmem_st8(p_addr + 8 * c16, w);
      }
      l += (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
      tmem_wait_st();
      // V rows past the visible tokens may hold anything: zero them (P is 0 there)
      if (t0 + BN > kv_len && t0 + r >= kv_len) {
        wait(&s.kv_full[j % STAGES], (uint32_t)((j / STAGES) & 1));
        const uint32_t vr = smem_u32(s.v[j % STAGES]) + r * ROWB;
#pragma unroll
        for (int c = 0; c < 8; ++c) sts128(vr + (c << 4), 0u, 0u, 0u, 0u);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&s.p_full[g]);
    }
    if (i > 0) {
      wait(&s.pv_done[g], (uint32_t)((i - 1) & 1));   // the group's last PV has retired
      __syncwarp();
      tc_fence_after();
    }
    // merge the two groups' rows: once both groups are here every MMA has
    // retired and every copy has landed, so the K stages hold the exchange;
    // group g writes output dims [32 g, 32 g + 32) of row r
    tc_fence_before();
    asm volatile("bar.sync 1, 256;" ::: "memory");
    float* xch = reinterpret_cast<float*>(s.k[0]);     // m0 | l0 | m1 | l1, 128 floats each
    xch[(2 * g) * BM + r] = m;
    xch[(2 * g + 1) * BM + r] = l;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    tc_fence_after();                                  // the other group's O columns are read too
    {
      const float m0 = xch[r], l0 = xch[BM + r], m1 = xch[2 * BM + r], l1 = xch[3 * BM + r];
      const float mm = fmaxf(m0, m1);                 // finite: token 0 is visible to every row
      const float a0 = ex2(m0 - mm);
      const bool use1 = m1 != -INFINITY;              // group 1 saw a visible token (or any tile)
      const float a1 = use1 ? ex2(m1 - mm) : 0.f;
      const float inv = 1.0f / (l0 * a0 + l1 * a1);
      float v0[32], v1[32];
      tmem_ld32(lane_base + O_COL + 32 * g, v0);
      tmem_ld32(lane_base + O_COL + 64 + 32 * g, v1);
      tmem_wait_ld32(v0);
      tmem_wait_ld32(v1);
      const int64_t qi = pos - p.q_start;
      if (qi < p.n_q) {
        float* dst = p.out + (qi * H + kvh * GROUP + (r & 7)) * HD + 32 * g;
#pragma unroll
        for (int d = 0; d < 32; d += 4) {
          float4 o4;
          o4.x = (use1 ? fmaf(v1[d], a1, v0[d] * a0) : v0[d] * a0) * inv;
          o4.y = (use1 ? fmaf(v1[d + 1], a1, v0[d + 1] * a0) : v0[d + 1] * a0) * inv;
          o4.z = (use1 ? fmaf(v1[d + 2], a1, v0[d + 2] * a0) : v0[d + 2] * a0) * inv;
          o4.w = (use1 ? fmaf(v1[d + 3], a1, v0[d + 3] * a0) : v0[d + 3] * a0) * inv;
          *reinterpret_cast<float4*>(dst + d) = o4;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

size_t smem_bytes() { return sizeof(Smem) + 1024; }

}  // namespace prefill
}  // namespace nyion

using namespace nyion;
using namespace nyion::prefill;

extern "C" int32_t nyion_attn_prefill_paged_bf16(const void* q, const void* kv_pool,
                                                 int64_t n_pool_pages, const int32_t* page_table,
                                                 int32_t max_pages, int64_t q_start, int64_t n_q,
                                                 float* out, int32_t n_heads, int32_t n_kv_heads,
                                                 int32_t head_dim, int32_t page_tokens, float scale,
                                                 void* stream) {
  if (!q || !kv_pool || !page_table || !out)
    return fail(NYION_ERR_INVALID, "prefill_paged_bf16: null pointer argument");
  if (!(head_dim == HD && n_kv_heads > 0 && n_heads == n_kv_heads * GROUP) &&
      generic_shape_ok(n_heads, n_kv_heads, head_dim)) {
    // other shapes: the reference's loop (executor.rs:106-138) as one launch of the
    // generic decode, query position i attending the q_start + i + 1 tokens before it
    if (page_tokens != PAGE) return fail(NYION_ERR_UNSUPPORTED, "prefill_paged_bf16: page_tokens must be 16");
    if (n_q <= 0 || q_start < 0 || max_pages <= 0 || n_pool_pages <= 0 || n_q > (1ll << 30))
      return fail(NYION_ERR_INVALID, "prefill_paged_bf16: bad sizes");
    if ((q_start + n_q + PAGE - 1) / PAGE > max_pages)
      return fail(NYION_ERR_INVALID, "prefill_paged_bf16: page table shorter than the context");
    GenericCall c;
    c.who = "prefill_paged_bf16";
    c.q = q;
    c.q_bf16 = 1;
    c.k = kv_pool;
    c.table = page_table;
    c.table_shared = 1;
    c.max_pages = max_pages;
    c.n_pool_pages = n_pool_pages;
    c.n_heads = n_heads;
    c.n_kv = n_kv_heads;
    c.head_dim = head_dim;
    c.rows = (int32_t)n_q;
    c.causal_base = q_start;
    c.scale = scale;
    c.out = out;
    c.max_tokens = q_start + n_q;
    c.fmt = kGenBF16;
    c.layout = kGenPaged;
    return generic_decode(c, static_cast<cudaStream_t>(stream));
  }
  if (head_dim != HD || n_kv_heads <= 0 || n_heads != n_kv_heads * GROUP)
    return fail(NYION_ERR_UNSUPPORTED,
                "prefill_paged_bf16: this build takes head_dim 64 and GQA group 8 (got %d, %d/%d)",
                head_dim, n_heads, n_kv_heads);
  if (page_tokens != PAGE) return fail(NYION_ERR_UNSUPPORTED, "prefill_paged_bf16: page_tokens must be 16");
  if (n_q <= 0 || q_start < 0 || max_pages <= 0 || n_pool_pages <= 0)
    return fail(NYION_ERR_INVALID, "prefill_paged_bf16: bad sizes");
  if ((q_start + n_q + PAGE - 1) / PAGE > max_pages)
    return fail(NYION_ERR_INVALID, "prefill_paged_bf16: page table shorter than the context");
  DeviceInfo* dev = nullptr;
  int32_t st = device_info(&dev);
  if (st) return st;
  CUtensorMap mq, mkv;
  {
    const uint64_t dims[3] = {(uint64_t)HD, (uint64_t)n_heads, (uint64_t)n_q};
    const uint64_t strides[2] = {(uint64_t)HD * 2, (uint64_t)n_heads * HD * 2};
    const uint32_t box[3] = {(uint32_t)HD, (uint32_t)GROUP, (uint32_t)POS};
    st = encode_tmap(&mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  {
    const uint64_t rows = (uint64_t)n_pool_pages * n_kv_heads * 2 * PAGE;
    if (rows > (1ull << 31)) return fail(NYION_ERR_INVALID, "prefill_paged_bf16: pool too large");
    const uint64_t dims[2] = {(uint64_t)HD, rows};
    const uint64_t strides[1] = {(uint64_t)HD * 2};
    const uint32_t box[2] = {(uint32_t)HD, (uint32_t)PAGE};
    st = encode_tmap(&mkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv_pool, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
  }
  const size_t smem = smem_bytes();
  st = kernel_setup(reinterpret_cast<const void*>(prefill_kernel), smem, THREADS, nullptr);
  if (st) return st;
  Params p{};
  p.table = page_table;
  p.max_pages = max_pages;
  p.n_pool_pages = n_pool_pages;
  p.n_kv = n_kv_heads;
  p.q_start = q_start;
  p.n_q = n_q;
  p.sl2 = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  p.out = out;
  p.err = dev->err_word;
  const int n_mt = (int)((n_q + POS - 1) / POS);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_mt * n_kv_heads));
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, prefill_kernel, p, mq, mkv), "prefill launch");
}
