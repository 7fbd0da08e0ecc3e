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
//     positions go through this kernel, whose CTA folds the window's
//     log-sum-exp partial into its own and writes the output.  Nibbles are read in the writer's order (element i in byte i/2,
//     low nibble for even i, cache.rs:637-663).
//
// Scattered positions cannot use page-granular copies, so rows are gathered:
// CTA = (sequence, KV head, 128-position split), warp = 32 positions.  Lane l
// resolves position l of its warp's tile to a pool row and brings that row's
// K and V into the warp's shared tiles (fp32 rows by sixteen 16-byte async
// copies each, 4-bit rows dequantized on the way with the reference's
// separate multiply and add), written in the 128-byte swizzled layout the
// tensor copies of the row-cache kernel produce; each scattered row crosses
// from memory once for all 8 query heads.  The warp then computes its tile
// alone: S = Q K^T and O = P V on mma.sync with every fp32 operand split into
// bf16 hi + lo (the A operand stacks the 8 heads' hi parts over their lo
// parts), softmax over the tile in the log2 domain.  The 4 warps' partials
// are folded in shared memory into one (o/l, m, l) partial per head and
// split; the last CTA of each (sequence, KV head) to finish merges the
// splits' partials and writes the output.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "host.h"

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
constexpr int WARPS = 4;               // one 32-position tile per warp
constexpr int THREADS = 32 * WARPS;
constexpr int SPLIT = 32 * WARPS;      // positions per CTA
constexpr int TILE_BYTES = 32 * HD * 4;   // 32 fp32 rows as two 128-byte column halves, swizzled
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
  float* out;                    // [batch][H][64]: merged here, or null: partials only
  int32_t* cnt;                  // [batch * n_kv] merge counters (start at 0, left at 0), n_splits > 1
  int32_t n_splits;              // with `out`
  const float* extra_part;       // with `out`: one more partial row set [batch * H][66] folded in, or null
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
  uint8_t kv[WARPS][2][TILE_BYTES];   // per warp: K tile | V tile (1024-byte aligned)
  float2 wml[WARPS][GROUP];           // per warp and head: (m log2, l)
  int32_t last;
};

// With `out`: the CTA counts in for (b, kvh) after its partial is stored (one
// acq_rel atomic after the CTA barrier; a single split is its own last CTA),
// and the last of the n_splits CTAs merges the partials of the 8 heads, plus
// `extra_part`'s row when given: w_s = l_s exp(m_s - M), o = sum w_s o_s /
// sum w_s (the log-sum-exp identity of nyion_attn_lse_combine).
__device__ __forceinline__ void count_in_and_merge(const Params& p, GatherSmem& sm, int b, int kvh) {
  const int tid = threadIdx.x;
  __syncthreads();   // this CTA's partial stores are ordered before thread 0's atomic
  if (p.n_splits > 1) {
    if (tid == 0) {
      int old;
      asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + b * p.n_kv + kvh) : "memory");
      const int last = old == p.n_splits - 1;
      if (last) atomicExch(p.cnt + b * p.n_kv + kvh, 0);
      sm.last = last;
    }
    __syncthreads();
    if (!sm.last) return;
  }
  const int H = p.n_kv * GROUP;
  const int h = tid >> 4, d0 = 4 * (tid & 15);   // head of the group, 4 dims
  const int64_t row0 = (int64_t)b * H + kvh * GROUP;
  const int64_t row = row0 + h;
  const int64_t sstride = (int64_t)p.batch * H * PART;
  const int n_all = p.n_splits + (p.extra_part ? 1 : 0);
  // partial row of split sp (the extra set last) for head row r
  auto prow = [&](int sp, int64_t r) {
    return sp < p.n_splits ? p.part + (int64_t)sp * sstride + r * PART : p.extra_part + r * PART;
  };
  // splits in chunks of MCH: their (m, l) pairs for the 8 heads go to shared
  // memory in one parallel pass (the tiles are free), then every thread sums
  // its 4 dims with 8 partial rows in flight; chunks fold online
  constexpr int MCH = 256;
  float2* mls = reinterpret_cast<float2*>(sm.kv);   // [MCH][8]
  float M = -INFINITY, den = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c0 = 0; c0 < n_all; c0 += MCH) {
    const int cn = min(MCH, n_all - c0);
    __syncthreads();   // the previous chunk's pairs have been read
    for (int i = tid; i < cn * GROUP; i += THREADS) {
      const float* pp = prow(c0 + i / GROUP, row0 + i % GROUP);
      mls[i] = make_float2(__ldcg(pp + HD), __ldcg(pp + HD + 1));
    }
    __syncthreads();
    float mc = -INFINITY;
    for (int k = 0; k < cn; ++k) {
      const float2 x = mls[k * GROUP + h];
      if (x.y > 0.f) mc = fmaxf(mc, x.x);
    }
    const float Mn = fmaxf(M, mc);
    if (Mn == -INFINITY) continue;                  // nothing attended so far
    const float sc = M > -INFINITY ? expf(M - Mn) : 0.f;
    den *= sc;
    acc.x *= sc; acc.y *= sc; acc.z *= sc; acc.w *= sc;
    M = Mn;
    for (int k = 0; k < cn; k += 8) {
      float4 ov[8];
      float wv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int kk = k + u;
        const float2 x = kk < cn ? mls[kk * GROUP + h] : make_float2(-INFINITY, 0.f);
        wv[u] = x.y > 0.f ? x.y * expf(x.x - M) : 0.f;
        ov[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (wv[u] > 0.f) {
          const float* src = prow(c0 + kk, row) + d0;
          const float2 a = __ldcg(reinterpret_cast<const float2*>(src));
          const float2 c = __ldcg(reinterpret_cast<const float2*>(src + 2));
          ov[u] = make_float4(a.x, a.y, c.x, c.y);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        den += wv[u];
        acc.x = fmaf(wv[u], ov[u].x, acc.x);
        acc.y = fmaf(wv[u], ov[u].y, acc.y);
        acc.z = fmaf(wv[u], ov[u].z, acc.z);
        acc.w = fmaf(wv[u], ov[u].w, acc.w);
      }
    }
  }
  const float inv = den > 0.f ? 1.0f / den : 0.f;
  *reinterpret_cast<float4*>(p.out + row * HD + d0) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

// byte offset of 16-byte chunk c16 (0..15) of row rr (0..31) in a tile
__device__ __forceinline__ uint32_t tile_off(int rr, int c16) {
  return (uint32_t)((c16 >> 3) * 4096 + rr * 128 + (((c16 & 7) ^ (rr & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <bool Q4, bool RULE>
__global__ void __launch_bounds__(THREADS, 3) positions_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  GatherSmem& sm =
      *reinterpret_cast<GatherSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
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
    if (p.out) count_in_and_merge(p, sm, b, kvh);
    return;
  }
  const int cnt = j1 - j0;
  // ---- lane -> position 32 w + lane of the split -> pool row ----
  int64_t row = -1;
  if (32 * w + lane < cnt) {
    const int pos = position_of<RULE>(p, b, j0 + 32 * w + lane);
    const int pidx = pos / PAGE;
    int64_t page = -1;
    if (pos >= 0 && pidx < p.max_pages) page = p.table[(int64_t)b * p.max_pages + pidx];
    if (page < 0 || page >= p.n_pool_pages) record_error(p.err, kErrPageRange);
    else row = ((page * p.n_kv + kvh) * 2) * PAGE + pos % PAGE;
  }
  const uint32_t vmask = __ballot_sync(0xffffffffu, row >= 0);   // tokens of this tile that exist
  // ---- gather this lane's K and V rows into the warp's tiles ----
  const uint32_t kb = smem_u32(sm.kv[w][0]), vb = smem_u32(sm.kv[w][1]);
  if (row >= 0) {
    if (!Q4) {
      const float* ks = static_cast<const float*>(p.pool) + row * HD;
      const float* vs = ks + PAGE * HD;
#pragma unroll
      for (int c16 = 0; c16 < 16; ++c16) {
        cp_async16(kb + tile_off(lane, c16), ks + 4 * c16);
        cp_async16(vb + tile_off(lane, c16), vs + 4 * c16);
      }
      asm volatile("cp.async.commit_group;\ncp.async.wait_all;" ::: "memory");
    } else {
#pragma unroll
      for (int kv = 0; kv < 2; ++kv) {
        float x[HD];
        load_row_q4(p, row + kv * PAGE, x);
        const uint32_t base = kv ? vb : kb;
#pragma unroll
        for (int c16 = 0; c16 < 16; ++c16)
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(base + tile_off(lane, c16)),
                       "f"(x[4 * c16]), "f"(x[4 * c16 + 1]), "f"(x[4 * c16 + 2]), "f"(x[4 * c16 + 3])
                       : "memory");
      }
    }
  } else {   // a missing row reads as zeros (its score is masked; V must be finite)
#pragma unroll
    for (int c16 = 0; c16 < 16; ++c16) {
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(kb + tile_off(lane, c16)), "r"(0u) : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(vb + tile_off(lane, c16)), "r"(0u) : "memory");
    }
  }
  __syncwarp();
  // ---- S = Q K^T for the tile: head g, tokens 8nt + 2tg + {0, 1} ----
  const int g = lane >> 2, tg = lane & 3, r8 = lane & 7, j4 = lane >> 3;
  uint32_t qa[4][4];   // k-step ks: kappa 2t, 2t+1, 2t+8, 2t+9 -> dims 16ks + t, +4, +8, +12
  {
    const float* qh = p.q + ((int64_t)b * H + kvh * GROUP + g) * HD;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const float* bq = qh + 16 * ks;
      split_bf16x2(bq[tg] * p.sl2, bq[4 + tg] * p.sl2, qa[ks][0], qa[ks][1]);
      split_bf16x2(bq[8 + tg] * p.sl2, bq[12 + tg] * p.sl2, qa[ks][2], qa[ks][3]);
    }
  }
  float sc[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int tok = 8 * nt + r8, chunk = 4 * (ks & 1) + j4;
      uint32_t a0, a1, a2, a3;
      ldsm_x4(kb + (ks >> 1) * 4096 + tok * 128 + ((chunk ^ r8) << 4), a0, a1, a2, a3);
      uint32_t bh0, bl0, bh1, bl1;
      split_bf16x2(__uint_as_float(a0), __uint_as_float(a1), bh0, bl0);
      split_bf16x2(__uint_as_float(a2), __uint_as_float(a3), bh1, bl1);
      mma_bf16(sc[nt], qa[ks], bh0, bh1);
      mma_bf16(sc[nt], qa[ks], bl0, bl1);
    }
  float sv[4][2];
  float mx = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int tok = 8 * nt + 2 * tg + e;
      sv[nt][e] = ((vmask >> tok) & 1u) ? sc[nt][e] + sc[nt][e + 2] : -INFINITY;
      mx = fmaxf(mx, sv[nt][e]);
    }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  float l = 0.f;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    sv[nt][0] = mx > -INFINITY ? exp2f(sv[nt][0] - mx) : 0.f;
    sv[nt][1] = mx > -INFINITY ? exp2f(sv[nt][1] - mx) : 0.f;
    l += sv[nt][0] + sv[nt][1];
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  // ---- O = P V: k = tokens (2 steps of 16), n = dims (8 tiles of 8) ----
  float o[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    uint32_t pa[4];
    split_bf16x2(sv[2 * kk][0], sv[2 * kk][1], pa[0], pa[1]);
    split_bf16x2(sv[2 * kk + 1][0], sv[2 * kk + 1][1], pa[2], pa[3]);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int f = 8 * nt + g, chunk = (f & 31) >> 2;
      const uint32_t col = vb + (f >> 5) * 4096 + 4 * (f & 3);
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = 16 * kk + 2 * tg + (e & 1) + 8 * (e >> 1);
        v[e] = lds32(col + tok * 128 + ((chunk ^ (tok & 7)) << 4));
      }
      uint32_t bh0, bl0, bh1, bl1;
      split_bf16x2(v[0], v[1], bh0, bl0);
      split_bf16x2(v[2], v[3], bh1, bl1);
      mma_bf16(o[nt], pa, bh0, bh1);
      mma_bf16(o[nt], pa, bl0, bl1);
    }
  }
  // ---- fold the 4 warps: head h's (m, l) and o rows through shared memory ----
  __syncthreads();   // every warp is done with its tiles
  float* fo = reinterpret_cast<float*>(sm.kv);   // [warp][head][64]
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
    *reinterpret_cast<float2*>(fo + (w * GROUP + g) * HD + 8 * nt + 2 * tg) =
        make_float2(o[nt][0] + o[nt][2], o[nt][1] + o[nt][3]);
  if (tg == 0) sm.wml[w][g] = make_float2(mx, l);
  __syncthreads();
  // thread -> head tid / 16, dims 4 (tid % 16) .. + 3
  const int h = tid >> 4, d0 = 4 * (tid & 15);
  float M = -INFINITY;
#pragma unroll
  for (int ww = 0; ww < WARPS; ++ww) M = fmaxf(M, sm.wml[ww][h].x);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int ww = 0; ww < WARPS; ++ww) {
    const float2 x = sm.wml[ww][h];
    const float sw = (M > -INFINITY && x.x > -INFINITY) ? exp2f(x.x - M) : 0.f;
    const float4 ov = *reinterpret_cast<const float4*>(fo + (ww * GROUP + h) * HD + d0);
    L = fmaf(sw, x.y, L);
    acc.x = fmaf(sw, ov.x, acc.x);
    acc.y = fmaf(sw, ov.y, acc.y);
    acc.z = fmaf(sw, ov.z, acc.z);
    acc.w = fmaf(sw, ov.w, acc.w);
  }
  float* dst = p.part + ((int64_t)split * p.batch * H + (int64_t)b * H + kvh * GROUP + h) * PART;
  const float inv = L > 0.f ? 1.0f / L : 0.f;
  // partial rows are 66 floats (264 bytes): 8-byte stores keep every address aligned
  *reinterpret_cast<float2*>(dst + d0) = make_float2(acc.x * inv, acc.y * inv);
  *reinterpret_cast<float2*>(dst + d0 + 2) = make_float2(acc.z * inv, acc.w * inv);
  if ((tid & 15) == 0) {
    dst[HD] = L > 0.f ? M * 0.69314718055994531f : -INFINITY;
    dst[HD + 1] = L;
  }
  if (p.out) count_in_and_merge(p, sm, b, kvh);
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

constexpr size_t kSmem = sizeof(GatherSmem) + 1024;

template <bool Q4, bool RULE>
int32_t launch_positions(dim3 grid, const Params& p, cudaStream_t stream) {
  const int32_t st = kernel_setup(reinterpret_cast<const void*>(positions_kernel<Q4, RULE>), kSmem, THREADS, nullptr);
  if (st) return st;
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

// [merge counters: batch * n_kv ints, 256-byte aligned][split partials]
static size_t positions_counter_bytes(int32_t batch, int32_t n_heads) {
  return ((size_t)batch * (n_heads / GROUP > 0 ? n_heads / GROUP : 1) * sizeof(int32_t) + 255) & ~size_t(255);
}

extern "C" size_t nyion_attn_positions_workspace_size(int32_t batch, int32_t n_heads, int32_t max_positions) {
  const int ns = max_positions <= 0 ? 1 : (max_positions + SPLIT - 1) / SPLIT;
  return positions_counter_bytes(batch, n_heads) + part_bytes(ns, batch, n_heads);
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
  const size_t cb = positions_counter_bytes(batch, n_heads);
  const size_t need = cb + part_bytes(ns, batch, n_heads);
  if (!workspace) {
    st = internal_workspace(need, &workspace, kWsCounters, cb, static_cast<cudaStream_t>(stream));
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
  p.cnt = static_cast<int32_t*>(workspace);
  p.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + cb);
  p.out = out;
  p.n_splits = ns;
  p.err = dev->err_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)(batch * n_kv_heads), (unsigned)ns);
  // the last CTA of each (sequence, KV head) merges the splits: one launch
  return kv_format == 0 ? launch_positions<false, false>(grid, p, s) : launch_positions<true, false>(grid, p, s);
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
    // the Q4 decode keeps its merge counters at the start of this buffer
    st = internal_workspace(need, &workspace, kWsCounters, q4_counter_bytes(), static_cast<cudaStream_t>(stream));
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
  // <= 128 globals: one split per (sequence, KV head), whose CTA folds the
  // window's partial in and writes the output
  p.out = out;
  p.n_splits = 1;
  p.extra_part = parts;
  p.err = dev->err_word;
  return launch_positions<true, true>(dim3((unsigned)(batch * n_kv_heads), 1), p, s);
}
