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
//   * S = Q K^T: 4 x tcgen05.mma (M128 N128 K16, bf16 -> fp32) into TMEM
//     columns [0, 128); P = softmax numerators in bf16 (shared memory, 128B
//     swizzle); O_tile = P V: 8 x tcgen05.mma (M128 N64 K16, V as an MN-major
//     operand) into TMEM columns [128, 192);
//   * warp roles: warps 0-3 own one row each (tcgen05.ld of the row's S and
//     O_tile, online softmax and the running O in registers, causal mask),
//     warp 4 issues the TMA copies (Q tile once, K/V pages into a 2-stage
//     ring), warp 5 allocates TMEM and one of its threads issues the MMAs —
//     S of the next tile is issued as soon as the softmax warps have read the
//     current one.  Every wait is bounded; TMEM is released on every path.
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
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t S_COL = 0, O_COL = 128;
constexpr int ROWB = HD * 2;               // 128 bytes per bf16 row

struct Smem {
  uint8_t q[BM * ROWB];          // Q tile, 16 KB
  uint8_t k[2][BN * ROWB];       // K tiles, 2 x 16 KB
  uint8_t v[2][BN * ROWB];       // V tiles, 2 x 16 KB
  uint8_t p[2][2][BM * ROWB];    // P per stage: tokens 0-63 | 64-127 (K-major, two 128-B atoms)
  uint64_t q_full, kv_full[2], kv_empty[2], s_full, s_empty, p_full, o_full, done;
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

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_empty, 128);
    mbar_init(&s.p_full, 128);
    mbar_init(&s.o_full, 1);
    mbar_init(&s.done, 1);
    s.abort_ = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
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

  auto wait = [&](uint64_t* bar, uint32_t parity) {
    if (*reinterpret_cast<volatile int32_t*>(&s.abort_)) return;
    if (!mbar_wait_bounded(bar, parity)) {
      record_error(p.err, kErrWaitTimeout);
      atomicExch(&s.abort_, 1);
    }
  };

  if (warp == 4) {
    // ================= TMA producer =================
    if (lane == 0) {
      mbar_arrive_expect_tx(&s.q_full, BM * ROWB);
      // (x: 64 dims, head, position) box (64, 8, 16): rows = position * 8 + head
      tma_load_3d(s.q, &map_q, 0, kvh * GROUP, (int32_t)(pos0 - p.q_start), &s.q_full);
    }
    for (int j = 0; j < nt; ++j) {
      const int st = j & 1;
      if (j >= 2) wait(&s.kv_empty[st], (uint32_t)(((j >> 1) - 1) & 1));
      // page ids of the tile's 8 pages, one per lane
      int32_t row = -4 * PAGE;
      if (lane < BN / PAGE) {
        const int64_t pidx = ((int64_t)j * BN) / PAGE + lane;
        if (pidx * PAGE < kv_len) {
          int64_t page = (pidx < p.max_pages) ? p.table[pidx] : -1;
          if (page < 0 || page >= p.n_pool_pages) {
            record_error(p.err, kErrPageRange);
          } else {
            row = (int32_t)(((page * p.n_kv + kvh) * 2) * PAGE);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&s.kv_full[st], 2 * BN * ROWB);
      __syncwarp();
      if (lane < BN / PAGE) {
        // rows outside the pool (negative) are zero-filled by the copy
        tma_load_2d(s.k[st] + lane * PAGE * ROWB, &map_kv, 0, row, &s.kv_full[st]);
        tma_load_2d(s.v[st] + lane * PAGE * ROWB, &map_kv, 0, row + PAGE, &s.kv_full[st]);
      }
    }
    // no copy may still be writing shared memory when the CTA exits (matters
    // only after an aborted wait; otherwise these phases completed long ago)
    if (lane == 0) {
      mbar_wait_bounded(&s.q_full, 0);
      for (int j = nt - 2 < 0 ? 0 : nt - 2; j < nt; ++j) mbar_wait_bounded(&s.kv_full[j & 1], (uint32_t)((j >> 1) & 1));
    }
  } else if (warp == 5) {
    // ================= MMA issuer =================
    if (lane == 0) {
      constexpr uint32_t IQK = instr_desc(BM, BN, false);
      constexpr uint32_t IPV = instr_desc(BM, HD, true);
      const uint32_t qa = smem_u32(s.q);
      auto issue_qk = [&](int j) {
        const int st = j & 1;
        const uint32_t kb = smem_u32(s.k[st]);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          umma(tmem + S_COL, smem_desc(qa + ks * 32, 16, 1024), smem_desc(kb + ks * 32, 16, 1024), IQK,
               ks > 0);
        umma_commit(&s.s_full);
      };
      wait(&s.q_full, 0);
      wait(&s.kv_full[0], 0);
      tc_fence_after();
      issue_qk(0);
      for (int j = 0; j < nt; ++j) {
        if (j + 1 < nt) {
          wait(&s.kv_full[(j + 1) & 1], (uint32_t)(((j + 1) >> 1) & 1));
          wait(&s.s_empty, (uint32_t)(j & 1));        // S_j has been read
          tc_fence_after();
          issue_qk(j + 1);
        }
        wait(&s.p_full, (uint32_t)(j & 1));
        tc_fence_after();
        const uint32_t vb = smem_u32(s.v[j & 1]);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma(tmem + O_COL, smem_desc(smem_u32(s.p[j & 1][kk >> 2]) + (kk & 3) * 32, 16, 1024),
               smem_desc(vb + kk * 2048, 8192, 1024), IPV, kk > 0);
        umma_commit(&s.o_full);
        umma_commit(&s.kv_empty[j & 1]);
      }
      umma_commit(&s.done);
      mbar_wait_bounded(&s.done, 0);   // every MMA has retired before TMEM is released
    }
    __syncwarp();
  } else {
    // ================= softmax warps: thread = row =================
    const int r = t;                                  // 0..127 = TMEM lane
    const int64_t pos = pos0 + (r >> 3);              // this row's absolute position
    const uint32_t lane_addr = (uint32_t)(32 * warp) << 16;
    float o[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    for (int j = 0; j < nt; ++j) {
      wait(&s.s_full, (uint32_t)(j & 1));
      __syncwarp();                                   // tcgen05.ld is warp-collective
      tc_fence_after();
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        float tmp[32];
        tmem_ld32(tmem + lane_addr + S_COL + c, tmp);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c + i] = tmp[i];
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s.s_empty);
      // causal mask (token <= position) and scale into the log2 domain
      const int64_t t0 = (int64_t)j * BN;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        const float v = (t0 + c <= pos) ? sv[c] * p.sl2 : -INFINITY;
        sv[c] = v;
        mx = fmaxf(mx, v);
      }
      const float mn = fmaxf(m, mx);
      const float alpha = exp2f(m - mn);
      m = mn;
      // P row r -> shared memory (stage j&1, free since PV(j-2) retired),
      // K-major with the 128-byte swizzle, two 64-token atoms; the row sum
      // is taken over the bf16-rounded numerators the tensor cores see
      float ps = 0.f;
      {
        const uint32_t pr0 = smem_u32(s.p[j & 1][0]) + r * ROWB;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(exp2f(sv[8 * c + 2 * e] - mn),
                                                            exp2f(sv[8 * c + 2 * e + 1] - mn));
            const float2 f2 = __bfloat1622float2(h2);
            ps += f2.x + f2.y;
            w[e] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          sts128(pr0 + (c >> 3) * (BM * ROWB) + ((((c & 7) ^ r) & 7) << 4), w[0], w[1], w[2], w[3]);
        }
      }
      l = fmaf(l, alpha, ps);
      // V rows past the visible tokens may hold anything: zero them (P is 0 there)
      if (t0 + BN > kv_len && t0 + r >= kv_len) {
        wait(&s.kv_full[j & 1], (uint32_t)((j >> 1) & 1));
        const uint32_t vr = smem_u32(s.v[j & 1]) + r * ROWB;
#pragma unroll
        for (int c = 0; c < 8; ++c) sts128(vr + (c << 4), 0u, 0u, 0u, 0u);
      }
      if (j > 0) {
        // fold the previous tile's P V into o before PV(j) reuses its TMEM columns
        wait(&s.o_full, (uint32_t)((j - 1) & 1));
        __syncwarp();
        tc_fence_after();
        float ot[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tmem_ld32(tmem + lane_addr + O_COL + 32 * half, ot);
          tmem_wait_ld();
#pragma unroll
          for (int d = 0; d < 32; ++d) o[32 * half + d] = fmaf(o[32 * half + d], alpha_prev, ot[d]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&s.p_full);
      alpha_prev = alpha;
    }
    wait(&s.o_full, (uint32_t)((nt - 1) & 1));
    __syncwarp();
    tc_fence_after();
    {
      float ot[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(tmem + lane_addr + O_COL + 32 * half, ot);
        tmem_wait_ld();
#pragma unroll
        for (int d = 0; d < 32; ++d) o[32 * half + d] = fmaf(o[32 * half + d], alpha_prev, ot[d]);
      }
    }
    const int64_t qi = pos - p.q_start;
    if (qi < p.n_q) {
      const float inv = 1.0f / l;
      float* dst = p.out + (qi * H + kvh * GROUP + (r & 7)) * HD;
#pragma unroll
      for (int d = 0; d < HD; d += 4)
        *reinterpret_cast<float4*>(dst + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
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
  static bool attr_done[64] = {false};
  const size_t smem = smem_bytes();
  if (!attr_done[dev->device < 64 ? dev->device : 0]) {
    st = check_cuda(cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                    "cudaFuncSetAttribute(prefill)");
    if (st) return st;
    attr_done[dev->device < 64 ? dev->device : 0] = true;
  }
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
  prefill_kernel<<<n_mt * n_kv_heads, THREADS, smem, static_cast<cudaStream_t>(stream)>>>(p, mq, mkv);
  return check_cuda(cudaGetLastError(), "prefill launch");
}
