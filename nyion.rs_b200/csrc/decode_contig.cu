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
// One call reads a few MB to a few hundred MB once:
//
//   * grid = (KV head, split), one CTA per SM: each CTA owns a contiguous
//     range of tiles of one KV head (f32: 32 tokens; f16: 64 tokens, so each
//     copy is 8 KB: 4 KB pieces stream at about half the rate);
//   * a producer warp streams the tiles with tensor copies (128-byte swizzle)
//     into a ring of stages (f32: 8 x 16 KB; f16: 12 x 16 KB); 8 consumer
//     warps take them round-robin, every 32 tokens computed by ONE warp for
//     all 8 query heads of the GQA group (an f16 tile by a pair of warps), so
//     no barrier spans the consumer warps;
//   * programmatic dependent launch: barrier set-up overlaps the previous grid,
//     nothing global is read before it has completed;
//   * S = Q K^T and O += P V run on mma.sync m16n8k16 with fp32 accumulation.
//     The A operand stacks the hi parts of the 8 heads (rows 0-7) over their
//     lo parts (rows 8-15), so one mma covers both halves of a split operand:
//       - f16 caches: K and V are exact f16 B operands, q and P are split into
//         f16 hi + lo (q pre-scaled by 2^8, P by 2^7, so their lo halves
//         stay clear of f16's subnormal range);
//       - f32 caches: K and V are split into bf16 hi + lo as well and every
//         product is issued twice (B hi, B lo), so all four cross products
//         accumulate (~2^-17 relative residual per operand);
//     K fragments come from ldmatrix on the tile, V fragments from
//     ldmatrix.trans (f16) or 32-bit shared loads (f32);
//   * online softmax per warp in the log2 domain, the reference maximum moved
//     only when a tile's maximum passes it by 8 (most tiles skip the rescale);
//   * the 8 warps fold their partials in shared memory; every CTA leaves one
//     (m, l, o[8][64]) partial per KV head and counts in with one acq_rel
//     atomic per KV head; the last CTA merges them (warp = head, the weights
//     computed once per split, the first 32 splits' rows loaded together with
//     the (m, l) pairs).  A single split writes the output directly.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace contig {

constexpr int HD = 64;
constexpr int GROUP = 8;
constexpr int SUB = 32;                // tokens one warp computes at a time
constexpr int NCW = 8;                 // consumer warps
constexpr int THREADS = (NCW + 1) * 32;
constexpr int TARGET_CTAS = 148;       // one CTA per SM
constexpr int MAX_SPLITS = 296;
constexpr float Q_PRE = 256.0f;        // f16 path: q * 2^8 before the split
constexpr float P_PRE = 128.0f;        // f16 path: P * 2^7 before the split (P < 2^8: below f16 max)
constexpr float RESCALE_AT = 8.0f;     // log2 units

enum Layout { kRows = 0, kZoned = 1 };

struct Params {
  const float* q;            // [n_kv * 8][64]
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

// One stage = the K tile then the V tile.  Copies of 8 KB or more keep HBM
// near its copy rate where 4 KB pieces reach about half of it, so an f16 tile
// is 64 tokens (64 x 128 B swizzled rows, 8 KB), computed by a pair of warps
// (32 tokens each); an f32 tile is 32 tokens (two 128-byte column halves of
// 32 swizzled rows, 8 KB) computed by one warp.
template <typename T>
struct Geo {
  static constexpr int WPT = sizeof(T) == 2 ? 2 : 1;         // warps per tile
  static constexpr int GROUPS = NCW / WPT;                   // tiles in flight on the consumers
  static constexpr int TILE = SUB * WPT;                     // tokens per tile
  static constexpr int TILE_BYTES = TILE * HD * (int)sizeof(T);
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int RING_BYTES = sizeof(T) == 2 ? 192 * 1024 : 128 * 1024;
  static constexpr int STAGES = RING_BYTES / STAGE_BYTES;   // 12 (f16) or 8 (f32)
  // tile k uses stage k % STAGES and warp group k % GROUPS: with STAGES a
  // multiple of GROUPS a stage is always read by the same warps, which take
  // their tiles in order, so none can wait on a barrier phase two
  // completions ahead of the stage's last copy
  static_assert(STAGES % GROUPS == 0, "a stage must always belong to one group of consumer warps");
  static_assert(STAGES <= 16, "Tail holds 16 stages");
};

struct Tail {                       // after the stage ring
  uint64_t full[16];
  uint64_t empty[16];               // WPT arrivals: the group's warps are done with the stage
  int32_t rows[16];                 // valid rows of the tile in the stage (0: none)
  int32_t abort_;
  int32_t last;
};

template <typename T>
size_t smem_bytes() { return Geo<T>::RING_BYTES + sizeof(Tail) + 1024; }

// first row of the tile starting at t0 for KV head kvh, or -1 when its zone
// page is not in the arena (zone-arena tiles are 32 tokens: page-aligned)
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

// tensor copies of one tile (K then V): f16 maps are (x 64 halves, row),
// f32 maps (x 32 floats, row, 128-byte half)
template <typename T>
__device__ __forceinline__ void copy_tile(uint8_t* dst, const CUtensorMap* mk, const CUtensorMap* mv, int32_t row,
                                          uint64_t* bar) {
  using G = Geo<T>;
  if (sizeof(T) == 2) {
    tma_load_2d(dst, mk, 0, row, bar);
    tma_load_2d(dst + G::TILE_BYTES, mv, 0, row, bar);
  } else {
    tma_load_3d(dst, mk, 0, row, 0, bar);
    tma_load_3d(dst + G::TILE_BYTES, mv, 0, row, 0, bar);
  }
}

// bounded wait that also gives up as soon as another warp has aborted
__device__ __forceinline__ bool wait_stage(uint64_t* bar, uint32_t parity, const volatile int32_t* abort_) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_) return false;
    if (i > 64) __nanosleep(64);
  }
  return false;
}

// Q as the A operand of S = Q K^T for k-step ks (dims 16ks..16ks+15): rows
// 0-7 = hi parts of heads 0-7, rows 8-15 = lo parts.  The k index kappa maps
// to dims identically for f16; for f32 it follows the ldmatrix word order of
// the fp32 tile: kappa 2t, 2t+1, 2t+8, 2t+9 -> dims t, 4+t, 8+t, 12+t.
template <typename T>
__device__ __forceinline__ void load_q(const float* qh, float pre, int t, uint32_t (&qa)[4][4]) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const float* b = qh + 16 * ks;
    float x0, x1, x2, x3;
    if (sizeof(T) == 2) {
      x0 = b[2 * t]; x1 = b[2 * t + 1]; x2 = b[2 * t + 8]; x3 = b[2 * t + 9];
    } else {
      x0 = b[t]; x1 = b[4 + t]; x2 = b[8 + t]; x3 = b[12 + t];
    }
    if (sizeof(T) == 2) {
      split_f16x2(x0 * pre, x1 * pre, qa[ks][0], qa[ks][1]);
      split_f16x2(x2 * pre, x3 * pre, qa[ks][2], qa[ks][3]);
    } else {
      split_bf16x2(x0 * pre, x1 * pre, qa[ks][0], qa[ks][1]);
      split_bf16x2(x2 * pre, x3 * pre, qa[ks][2], qa[ks][3]);
    }
  }
}

template <typename T, int LAYOUT>
__global__ void __launch_bounds__(THREADS, 1)
contig_kernel(const Params p, const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v) {
  using G = Geo<T>;
  constexpr bool F16 = sizeof(T) == 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Tail& t = *reinterpret_cast<Tail*>(ring + G::RING_BYTES);
  static_assert(LAYOUT == kRows || G::TILE == 32, "zone-arena tiles must be page-aligned (32 tokens)");
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    prefetch_tensormap(&map_k);
    prefetch_tensormap(&map_v);
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&t.full[s], 1);
      mbar_init(&t.empty[s], G::WPT);
    }
    t.abort_ = 0;
    fence_barrier_init();
  }
  // programmatic dependent launch: the set-up above overlaps the previous
  // grid; nothing global is read before that grid has completed and flushed
  // (the K/V rows, q and the device length may be its outputs), and the next
  // grid may start its own set-up now (our kernels wait the same way before
  // reading anything)
  pdl_wait();

  int n = p.n;
  if (p.d_len) {
    n = __ldg(p.d_len);
    n = n < 0 ? 0 : (n > p.window ? p.window : n);
  }
  const int n_tiles = (n + G::TILE - 1) / G::TILE;
  const int tb = split * p.tiles_per_split;
  const int my_tiles = max(0, min(n_tiles, tb + p.tiles_per_split) - tb);

  __syncthreads();

  const int g = lane >> 2, tg = lane & 3;
  float o[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m = -INFINITY, l = 0.f;   // head g: reference max (log2 units), this lane's share of the sum

  if (warp == NCW) {
    // ================= producer =================
    if (lane == 0) {
      int issued = 0;
      for (int k = 0; k < my_tiles; ++k) {
        const int st = k % G::STAGES;
        if (k >= G::STAGES && !wait_stage(&t.empty[st], (uint32_t)((k / G::STAGES) - 1) & 1u, &t.abort_)) {
          record_error(p.err, kErrWaitTimeout);
          atomicExch(&t.abort_, 1);
          break;
        }
        const int t0 = (tb + k) * G::TILE;
        int rows = min(G::TILE, n - t0);
        const int64_t r0 = tile_row<LAYOUT>(p, kvh, t0);
        if (r0 < 0) {
          record_error(p.err, kErrPageRange);
          rows = 0;
        }
        t.rows[st] = rows;
        if (rows > 0) {
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(&t.full[st], (uint32_t)G::STAGE_BYTES);
          copy_tile<T>(ring + st * G::STAGE_BYTES, &map_k, &map_v, (int32_t)r0, &t.full[st]);
        } else {
          mbar_arrive(&t.full[st]);
        }
        issued = k + 1;
      }
      if (t.abort_) {   // the copies in flight must land before the CTA leaves
        for (int k = max(0, issued - G::STAGES); k < issued; ++k)
          mbar_wait_bounded(&t.full[k % G::STAGES], (uint32_t)(k / G::STAGES) & 1u);
      }
    }
  } else {
    // ====== consumers: tile k -> warp group k % GROUPS, warp sub of the group takes
    // ====== tokens [32 sub, 32 sub + 32) of the tile
    uint32_t qa[4][4];
    load_q<T>(p.q + ((int64_t)kvh * GROUP + g) * HD, p.sl2 * (F16 ? Q_PRE : 1.0f), tg, qa);
    const float s_post = F16 ? 1.0f / Q_PRE : 1.0f;
    const float p_pre = F16 ? P_PRE : 1.0f;
    const int r8 = lane & 7, j4 = lane >> 3;
    const int grp = warp / G::WPT, sub = warp % G::WPT;
    for (int k = grp; k < my_tiles; k += G::GROUPS) {
      const int st = k % G::STAGES;
      const bool ok = wait_stage(&t.full[st], (uint32_t)(k / G::STAGES) & 1u, &t.abort_);
      if (!__all_sync(0xffffffffu, ok)) {
        record_error(p.err, kErrWaitTimeout);
        if (lane == 0) atomicExch(&t.abort_, 1);
        break;
      }
      const int nv = min(SUB, max(0, t.rows[st] - SUB * sub));   // valid rows of this warp's 32
      // this warp's 32 rows start 4 KB (f16) into the tile: a multiple of the
      // 1024-byte swizzle period, so the in-tile row index keeps its phase
      const uint32_t kb = smem_u32(ring + st * G::STAGE_BYTES) + sub * SUB * 128, vb = kb + G::TILE_BYTES;
      if (nv == 0) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&t.empty[st]);
        continue;
      }
      // ---- K fragments ----
      uint32_t kf[4][4][2];   // [nt][ks] f16: B fragments of K
      float kx[4][4][4];      // [nt][ks] f32: K[8nt+g][16ks + 4j + tg], j = 0..3
      if (F16) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int kp = 0; kp < 2; ++kp) {
            const int tok = 8 * nt + r8, chunk = 4 * kp + j4;
            ldsm_x4(kb + tok * 128 + ((chunk ^ r8) << 4), kf[nt][2 * kp][0], kf[nt][2 * kp][1],
                    kf[nt][2 * kp + 1][0], kf[nt][2 * kp + 1][1]);
          }
      } else {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const int tok = 8 * nt + r8, chunk = 4 * (ks & 1) + j4;
            uint32_t a, b, c, d;
            ldsm_x4(kb + (ks >> 1) * (SUB * 128) + tok * 128 + ((chunk ^ r8) << 4), a, b, c, d);
            kx[nt][ks][0] = __uint_as_float(a);
            kx[nt][ks][1] = __uint_as_float(b);
            kx[nt][ks][2] = __uint_as_float(c);
            kx[nt][ks][3] = __uint_as_float(d);
          }
      }
      // ---- S = Q K^T: head g, tokens 8nt + 2tg + {0, 1} ----
      float sc[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          if (F16) {
            mma_f16(sc[nt], qa[ks], kf[nt][ks][0], kf[nt][ks][1]);
          } else {
            uint32_t bh0, bl0, bh1, bl1;
            split_bf16x2(kx[nt][ks][0], kx[nt][ks][1], bh0, bl0);
            split_bf16x2(kx[nt][ks][2], kx[nt][ks][3], bh1, bl1);
            mma_bf16(sc[nt], qa[ks], bh0, bh1);
            mma_bf16(sc[nt], qa[ks], bl0, bl1);
          }
        }
      // ---- V fragments, then hand the stage back ----
      uint32_t vf16[2][8][2]; // [kk][nt] f16: B fragments of V
      float vx[2][8][4];      // [kk][nt] f32: V[16kk + 2tg + {0,1,8,9}][8nt + g]
      if (F16) {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            const int tok = 16 * kk + 8 * (j4 & 1) + r8, chunk = 2 * np + (j4 >> 1);
            ldsm_x4_t(vb + tok * 128 + ((chunk ^ r8) << 4), vf16[kk][2 * np][0], vf16[kk][2 * np][1],
                      vf16[kk][2 * np + 1][0], vf16[kk][2 * np + 1][1]);
          }
      } else {
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) {
            const int f = 8 * nt + g, chunk = (f & 31) >> 2;
            const uint32_t col = vb + (f >> 5) * (SUB * 128) + 4 * (f & 3);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int tok = 16 * kk + 2 * tg + (e & 1) + 8 * (e >> 1);
              vx[kk][nt][e] = lds32(col + tok * 128 + ((chunk ^ (tok & 7)) << 4));
            }
          }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&t.empty[st]);
      float sv[4][2];
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = (sc[nt][e] + sc[nt][e + 2]) * s_post;
          sv[nt][e] = (8 * nt + 2 * tg + e < nv) ? v : -INFINITY;
          mx = fmaxf(mx, sv[nt][e]);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      // ---- online softmax: the reference max moves only when passed by RESCALE_AT ----
      if (mx > m + RESCALE_AT) {
        const float al = exp2f(m - mx);   // 0 on the first tile (m = -inf)
        l *= al;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          o[nt][0] *= al; o[nt][1] *= al; o[nt][2] *= al; o[nt][3] *= al;
        }
        m = mx;
      }
      const bool live = m > -INFINITY;   // false only while every score of head g is -inf
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        sv[nt][0] = live ? exp2f(sv[nt][0] - m) : 0.f;
        sv[nt][1] = live ? exp2f(sv[nt][1] - m) : 0.f;
        l += sv[nt][0] + sv[nt][1];
      }
      // ---- O += P V: k = tokens (2 steps of 16), n = dims (8 tiles of 8) ----
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        if (16 * kk >= nv) break;
        uint32_t pa[4];
        if (F16) {
          split_f16x2(sv[2 * kk][0] * p_pre, sv[2 * kk][1] * p_pre, pa[0], pa[1]);
          split_f16x2(sv[2 * kk + 1][0] * p_pre, sv[2 * kk + 1][1] * p_pre, pa[2], pa[3]);
        } else {
          split_bf16x2(sv[2 * kk][0], sv[2 * kk][1], pa[0], pa[1]);
          split_bf16x2(sv[2 * kk + 1][0], sv[2 * kk + 1][1], pa[2], pa[3]);
        }
        // rows past the sequence end may hold anything: P is 0 there, V must be finite
        const int r = 16 * kk + 2 * tg;
        const bool ragged = nv < 16 * kk + 16;
        if (F16) {
          const uint32_t m0 = (r < nv ? 0x0000ffffu : 0u) | (r + 1 < nv ? 0xffff0000u : 0u);
          const uint32_t m1 = (r + 8 < nv ? 0x0000ffffu : 0u) | (r + 9 < nv ? 0xffff0000u : 0u);
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) {
            uint32_t b0 = vf16[kk][nt][0], b1 = vf16[kk][nt][1];
            if (ragged) {
              b0 &= m0;
              b1 &= m1;
            }
            mma_f16(o[nt], pa, b0, b1);
          }
        } else {
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) {
            float v0 = vx[kk][nt][0], v1 = vx[kk][nt][1], v2 = vx[kk][nt][2], v3 = vx[kk][nt][3];
            if (ragged) {
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
    }
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
  }
  __syncthreads();   // every copy has landed and been read: the ring is free

  // ---- fold the 8 warps: [warp][head][64] partials and (m, l) in the ring ----
  float* wo = reinterpret_cast<float*>(ring);                              // 16 KB
  float2* wml = reinterpret_cast<float2*>(ring + NCW * GROUP * HD * 4);    // 512 B
  if (warp < NCW) {
    const float post = F16 ? 1.0f / P_PRE : 1.0f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
      *reinterpret_cast<float2*>(wo + (warp * GROUP + g) * HD + 8 * nt + 2 * tg) =
          make_float2((o[nt][0] + o[nt][2]) * post, (o[nt][1] + o[nt][3]) * post);
    if (tg == 0) wml[warp * GROUP + g] = make_float2(m, l);
  }
  __syncthreads();
  const int h = warp;   // fold, publish and merge: warp = head (consumer warps only)
  float M = -INFINITY, L = 0.f;
  float2 acc = make_float2(0.f, 0.f);
  if (warp < NCW) {
#pragma unroll
    for (int w = 0; w < NCW; ++w) M = fmaxf(M, wml[w * GROUP + h].x);
#pragma unroll
    for (int w = 0; w < NCW; ++w) {
      const float2 x = wml[w * GROUP + h];
      const float sw = (M > -INFINITY && x.x > -INFINITY) ? exp2f(x.x - M) : 0.f;
      const float2 ov = *reinterpret_cast<const float2*>(wo + (w * GROUP + h) * HD + 2 * lane);
      L = fmaf(sw, x.y, L);
      acc.x = fmaf(sw, ov.x, acc.x);
      acc.y = fmaf(sw, ov.y, acc.y);
    }
  }
  float* dst = p.out + ((int64_t)kvh * GROUP + h) * HD + 2 * lane;
  if (p.n_splits == 1) {
    if (warp < NCW) {
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      *reinterpret_cast<float2*>(dst) = make_float2(acc.x * inv, acc.y * inv);
    }
    return;
  }
  const int64_t slot = (int64_t)kvh * p.n_splits + split;
  if (warp < NCW) {
    __stcg(reinterpret_cast<float2*>(p.part_o + (slot * GROUP + h) * HD + 2 * lane), acc);
    if (lane == 0) __stcg(&p.part_ml[slot * GROUP + h], make_float2(M, L));
  }
  // count in: the barrier makes the CTA's partial stores visible to thread 0,
  // whose acq_rel atomic releases them at gpu scope (and, for the last CTA,
  // acquires every other CTA's); the second barrier extends that to the CTA
  __syncthreads();
  if (tid == 0) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + kvh) : "memory");
    const int last = old == p.n_splits - 1;
    if (last) atomicExch(&p.cnt[kvh], 0);
    t.last = last;
  }
  __syncthreads();
  if (!t.last || warp >= NCW) return;
  // ---- last CTA of this KV head: merge the splits, warp = head ----
  // The first 32 splits' o rows are loaded before the weights are known, so
  // their loads and the (m, l) loads share one L2 round trip.
  float* wgt = reinterpret_cast<float*>(ring + 32 * 1024) + h * MAX_SPLITS;
  const int S = p.n_splits;
  const float2* ml = p.part_ml + (int64_t)kvh * S * GROUP + h;
  const float* po = p.part_o + ((int64_t)kvh * S * GROUP + h) * HD + 2 * lane;
  float2 x[32];
#pragma unroll
  for (int u = 0; u < 32; ++u)
    x[u] = u < S ? __ldcg(reinterpret_cast<const float2*>(po + (int64_t)u * GROUP * HD)) : make_float2(0.f, 0.f);
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
  float2 r = make_float2(0.f, 0.f);
#pragma unroll
  for (int u = 0; u < 32; ++u) {
    if (u < S) {
      const float wv = wgt[u];
      r.x = fmaf(wv, x[u].x, r.x);
      r.y = fmaf(wv, x[u].y, r.y);
    }
  }
  int s = 32;
  for (; s + 8 <= S; s += 8) {
    float2 y[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) y[u] = __ldcg(reinterpret_cast<const float2*>(po + (int64_t)(s + u) * GROUP * HD));
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float wv = wgt[s + u];
      r.x = fmaf(wv, y[u].x, r.x);
      r.y = fmaf(wv, y[u].y, r.y);
    }
  }
  for (; s < S; ++s) {
    const float2 y = __ldcg(reinterpret_cast<const float2*>(po + (int64_t)s * GROUP * HD));
    const float wv = wgt[s];
    r.x = fmaf(wv, y.x, r.x);
    r.y = fmaf(wv, y.y, r.y);
  }
  const float inv = den > 0.f ? 1.0f / den : 0.f;
  *reinterpret_cast<float2*>(dst) = make_float2(r.x * inv, r.y * inv);
}

struct Plan {
  int n_splits, tiles_per_split;
};

// Splits per KV head: one CTA per SM over all heads, as long as every split
// has a tile.  Short contexts gain from the widest spread (a single SM pulls
// a few hundred KB at well under its share of HBM bandwidth) more than they
// lose to the longer merge.
Plan plan(int n_kv, int max_tokens, int tile) {
  const int tiles = max_tokens > 0 ? (max_tokens + tile - 1) / tile : 1;
  int per_head = TARGET_CTAS / n_kv;
  if (per_head < 1) per_head = 1;
  int s = tiles < per_head ? tiles : per_head;
  const int tps = (tiles + s - 1) / s;
  s = (tiles + tps - 1) / tps;   // no trailing split without tiles
  return {s, tps};
}

size_t al(size_t x) { return (x + 255) & ~size_t(255); }

size_t counters_bytes(int n_kv) { return al((size_t)n_kv * sizeof(int32_t)); }

// sized for the most splits any element type plans, so one size serves f16 and f32
size_t workspace_bytes(int n_kv, int max_tokens) {
  const Plan pl = plan(n_kv, max_tokens, SUB);
  const size_t slots = (size_t)n_kv * pl.n_splits * GROUP;
  return counters_bytes(n_kv) + al(slots * sizeof(float2)) + al(slots * HD * sizeof(float));
}

// Tensor maps over `rows` rows of 64 elements: f16 (x 64, row), box 64 x 64;
// f32 (x 32, row, 128-byte half), box 32 x 32 x 2; 128-byte swizzle.
template <typename T>
int32_t row_map(CUtensorMap* m, const void* base, uint64_t rows) {
  if (sizeof(T) == 2)
    return encode_rows_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, HD, rows, HD, Geo<T>::TILE,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  const uint64_t dims[3] = {32, rows, 2};
  const uint64_t strides[2] = {HD * 4, 128};
  const uint32_t box[3] = {32, (uint32_t)Geo<T>::TILE, 2};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, int LAYOUT>
int32_t launch(Params p, const void* k, const void* v, uint64_t rows, int max_tokens, void* ws, size_t ws_bytes,
               cudaStream_t stream) {
  if (p.n_kv <= 0 || p.n_kv > 65535) return fail(NYION_ERR_INVALID, "row decode: bad n_kv_heads %d", p.n_kv);
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
    return fail(NYION_ERR_INVALID, "row decode: K/V must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(p.out) & 7) return fail(NYION_ERR_INVALID, "row decode: out must be 8-byte aligned");
  if (rows == 0 || rows >= (1ull << 31)) return fail(NYION_ERR_INVALID, "row decode: %llu rows (limit 2^31)",
                                                     (unsigned long long)rows);
  DeviceInfo* dev = nullptr;
  int32_t st = device_info(&dev);
  if (st) return st;
  CUtensorMap mk, mv;
  st = row_map<T>(&mk, k, rows);
  if (st) return st;
  st = row_map<T>(&mv, v, rows);
  if (st) return st;
  const Plan pl = plan(p.n_kv, max_tokens, Geo<T>::TILE);
  const size_t need = workspace_bytes(p.n_kv, max_tokens);
  if (!ws) {
    st = internal_workspace(need, &ws, kWsCounters, counters_bytes(p.n_kv), stream);
    if (st) return st;
  } else if (ws_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "row decode: workspace %zu B < %zu B", ws_bytes, need);
  }
  st = kernel_setup(reinterpret_cast<const void*>(contig_kernel<T, LAYOUT>), smem_bytes<T>(), THREADS, nullptr);
  if (st) return st;
  p.n_splits = pl.n_splits;
  p.tiles_per_split = pl.tiles_per_split;
  uint8_t* base = static_cast<uint8_t*>(ws);
  const size_t slots = (size_t)p.n_kv * pl.n_splits * GROUP;
  p.cnt = reinterpret_cast<int32_t*>(base);
  p.part_ml = reinterpret_cast<float2*>(base + counters_bytes(p.n_kv));
  p.part_o = reinterpret_cast<float*>(base + counters_bytes(p.n_kv) + al(slots * sizeof(float2)));
  p.err = dev->err_word;
  return check_cuda(launch_pdl(contig_kernel<T, LAYOUT>, dim3((unsigned)p.n_kv, (unsigned)pl.n_splits),
                              dim3(THREADS), smem_bytes<T>(), stream, p, mk, mv),
                    "row decode launch");
}

}  // namespace contig

size_t contig_workspace_bytes(int n_kv, int max_tokens) { return contig::workspace_bytes(n_kv, max_tokens); }

int32_t contig_rows_f32(const float* q, const float* k, const float* v, float* out, int n_kv, int64_t stride, int n,
                        float sl2, void* ws, size_t ws_bytes, cudaStream_t stream) {
  contig::Params p{};
  p.q = q;
  p.out = out;
  p.stride = stride;
  p.n_kv = n_kv;
  p.n = n;
  p.sl2 = sl2;
  return contig::launch<float, contig::kRows>(p, k, v, (uint64_t)n_kv * (uint64_t)stride, n, ws, ws_bytes, stream);
}

int32_t contig_rows_f16(const float* q, const void* k, const void* v, float* out, int n_kv, int64_t stride, int n,
                        const int32_t* d_len, int window, float sl2, void* ws, size_t ws_bytes,
                        cudaStream_t stream) {
  contig::Params p{};
  p.q = q;
  p.out = out;
  p.stride = stride;
  p.n_kv = n_kv;
  p.n = n;
  p.d_len = d_len;
  p.window = window;
  p.sl2 = sl2;
  return contig::launch<__half, contig::kRows>(p, k, v, (uint64_t)n_kv * (uint64_t)stride, d_len ? window : n, ws,
                                               ws_bytes, stream);
}

int32_t contig_zoned_f32(const float* q, const float* k_arena, const float* v_arena, float* out, int n_kv,
                         int n_layers, int layer, int64_t n_pages, int n, float sl2, void* ws, size_t ws_bytes,
                         cudaStream_t stream) {
  contig::Params p{};
  p.q = q;
  p.out = out;
  p.n_kv = n_kv;
  p.n = n;
  p.n_layers = n_layers;
  p.layer = layer;
  p.n_pages = n_pages;
  p.sl2 = sl2;
  // rows in the arena: zone pages [0, n_pages) of 32 / 128 / 1024 slots
  const int64_t lp = (int64_t)n_layers * n_kv;
  const int64_t z0 = n_pages < 128 ? n_pages : 128;
  const int64_t z1 = n_pages - z0 < 992 ? n_pages - z0 : 992;
  const int64_t z2 = n_pages - z0 - z1;
  const uint64_t rows = (uint64_t)(z0 * 32 + z1 * 128 + z2 * 1024) * (uint64_t)lp;
  return contig::launch<float, contig::kZoned>(p, k_arena, v_arena, rows, n, ws, ws_bytes, stream);
}

}  // namespace nyion
