// decode_generic.cu — decode attention for the shapes the specialised kernels
// of this library do not take: head_dim 64 or 128, any GQA group from 1 to 8,
// any number of KV heads (ops::attention takes any n_heads / n_kv_heads /
// head_dim, swamp-engine/src/ops.rs:170-191, and so does the reference's CUDA
// decode, swamp-gpu/kernels/fused_attention.cu:20-68, 194-243).  The entry
// points route every call whose shape is not head_dim 64 with group 8 here:
//
//   * paged fp32 pools (nyion_attn_decode_paged_f32), 4-bit pools
//     (nyion_attn_decode_q4_partial, ..._splitkv on one rank) and bf16 pools
//     (nyion_attn_prefill_paged_bf16: query position i of a chunk attends the
//     q_start + i + 1 tokens before it, the reference's prefill loop,
//     swamp-engine/src/executor.rs:106-138);
//   * contiguous fp32 / f16 caches [n_kv][stride][head_dim]
//     (gpu_attention_*, gpu_graph_create_attention[_half],
//     nyion_attn_decode_contig_f16, the layer-graph f16 ring with its length
//     read on the device);
//   * the reference's zone-page arena (nyion_attn_decode_zoned_f32).
//
// Work item = (query row, KV head, split of the token range); 128 threads.
// Tiles of 32 tokens are staged in shared memory as fp32 rows padded by 16
// bytes (16-byte reads of consecutive rows hit distinct banks); f16 / bf16 are
// widened on the way, 4-bit rows dequantized with the reference's separate
// multiply and add (cache.rs:375-394, bit-exact).  Scores: thread = (head,
// token), dot of the staged row against q in shared memory; softmax: warp =
// head, lane = token, online across tiles in the log2 domain; P.V: thread =
// (dim, head group), the group's heads accumulated in registers.  These are
// CUDA-core FMAs: with at most 8 query heads per KV row the arithmetic stays
// below the HBM rate.  A row split over several CTAs is merged by the last
// CTA to finish (per-(row, KV head) counter, acq_rel), in the same launch.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace gen {

constexpr int THREADS = 128;
constexpr int TILE = 32;          // tokens per staged tile
constexpr int MAXG = 8;           // query heads per KV head
constexpr int MAXSPLIT = 64;      // work items per (row, KV head)
constexpr int PAGE = 16;

struct Params {
  const void* q;               // [rows][n_heads][hd] f32, or bf16 when q_bf16
  int32_t q_bf16;
  const uint8_t* k;            // paged: the pool; rows / zoned: the K base
  const uint8_t* v;            // rows / zoned: the V base
  const int32_t* table;        // paged: [rows][max_pages] or one shared row
  int32_t table_shared, max_pages;
  int64_t n_pool_pages;
  int32_t n_kv, group, rows;   // rows = query rows of this launch
  // attended tokens [lo, hi) of row b: lens -> [0, lens[b]); tok arrays; u range;
  // causal_base >= 0 -> [0, causal_base + b + 1); d_len -> [0, min(*d_len, window))
  const int32_t* lens;
  const int32_t* tok_begin;
  const int32_t* tok_end;
  int32_t u_begin, u_end;
  int64_t causal_base;
  const int32_t* d_len;
  int32_t window;
  int64_t stride;              // rows layout: tokens per KV head
  int32_t n_layers, layer;     // zoned layout
  int64_t n_pages;             // zoned: arena pages
  float qscale;                // scale * log2(e)
  int32_t n_splits, split_len;
  int32_t part_mode;           // 0: out [rows][H][hd]; 1: part [rows][H][hd + 2] (o / l, m natural, l)
  float* out;
  float* ws_part;              // [rows * n_kv * n_splits][MAXG][hd + 2]
  int32_t* cnt;                // [rows * n_kv], zero between calls
  int32_t* err;
};

constexpr int32_t kF32 = kGenF32, kF16 = kGenF16, kBF16 = kGenBF16, kQ4 = kGenQ4;
constexpr int32_t kPaged = kGenPaged, kRows = kGenRows, kZoned = kGenZoned;

template <int HD, int FMT>
__host__ __device__ constexpr int row_bytes() {
  return FMT == kQ4 ? HD / 32 * 20 : HD * (FMT == kF32 ? 4 : 2);
}

__device__ __forceinline__ void row_range(const Params& p, int b, int64_t& lo, int64_t& hi) {
  if (p.causal_base >= 0) {
    lo = 0;
    hi = p.causal_base + b + 1;
  } else if (p.d_len) {
    lo = 0;
    const int32_t n = *p.d_len;
    hi = n < p.window ? n : p.window;
  } else if (p.lens) {
    lo = 0;
    hi = p.lens[b];
  } else {
    lo = p.tok_begin ? p.tok_begin[b] : p.u_begin;
    hi = p.tok_end ? p.tok_end[b] : p.u_end;
  }
  if (lo < 0) lo = 0;
  if (hi < lo) hi = lo;
}

// K (which = 0) or V row of token t for (row b, KV head kv), or null when its
// page is missing (then the token is masked; a page id out of range is reported)
template <int HD, int FMT, int LAY>
__device__ __forceinline__ const uint8_t* kv_row(const Params& p, int b, int kv, int64_t t, int which) {
  constexpr int RB = row_bytes<HD, FMT>();
  if (LAY == kPaged) {
    const int64_t pidx = t / PAGE;
    if (pidx >= p.max_pages) {
      record_error(p.err, kErrPageRange);
      return nullptr;
    }
    const int32_t page = p.table[(p.table_shared ? 0 : (int64_t)b * p.max_pages) + pidx];
    if (page < 0 || page >= p.n_pool_pages) {
      record_error(p.err, kErrPageRange);
      return nullptr;
    }
    return p.k + ((((int64_t)page * p.n_kv + kv) * 2 + which) * PAGE + t % PAGE) * RB;
  } else if (LAY == kRows) {
    return (which ? p.v : p.k) + ((int64_t)kv * p.stride + t) * RB;
  } else {
    // cache.rs:185-237, 681-747: zone z holds pages of bs_z slots laid out
    // [layer][kv head][slot][head_dim]; pages consecutive in the arena
    const int zone = t < 4096 ? 0 : (t < 131072 ? 1 : 2);
    const int64_t bs = zone == 0 ? 32 : (zone == 1 ? 128 : 1024);
    const int64_t zs = zone == 0 ? 0 : (zone == 1 ? 4096 : 131072);
    const int64_t zpage = zone == 0 ? 0 : (zone == 1 ? 128 : 1120);
    const int64_t lp = (int64_t)p.n_layers * p.n_kv;
    const int64_t zrow = zone == 0 ? 0 : (zone == 1 ? 128 * lp * 32 : 128 * lp * 32 + 992 * lp * 128);
    const int64_t local = (t - zs) / bs, slot = (t - zs) % bs;
    if (zpage + local >= p.n_pages) return nullptr;
    return (which ? p.v : p.k) + (zrow + local * lp * bs + ((int64_t)p.layer * p.n_kv + kv) * bs + slot) * RB;
  }
}

// elements 4c .. 4c + 3 of a row as fp32
template <int HD, int FMT>
__device__ __forceinline__ float4 load4(const uint8_t* row, int c) {
  if (FMT == kF32) return __ldg(reinterpret_cast<const float4*>(row) + c);
  if (FMT == kF16) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(row) + c);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  if (FMT == kBF16) {
    const uint2 w = __ldg(reinterpret_cast<const uint2*>(row) + c);
    return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u), __uint_as_float(w.y << 16),
                       __uint_as_float(w.y & 0xffff0000u));
  }
  // 4-bit: block (4c) / 32 = [f16 d][f16 dmin][16 B nibbles], element i in byte i/2,
  // low nibble for even i; x = f32(d) * q + f32(dmin), separate multiply and add
  const int e0 = 4 * c, blk = e0 >> 5, j = e0 & 31;
  const uint8_t* bp = row + blk * 20;
  const uint32_t h = __ldg(reinterpret_cast<const uint32_t*>(bp));
  const float d = __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
  const float dm = __half2float(__ushort_as_half((unsigned short)(h >> 16)));
  const uint32_t nb = __ldg(reinterpret_cast<const unsigned short*>(bp + 4 + j / 2));
  return make_float4(__fadd_rn(__fmul_rn(d, (float)(nb & 0xf)), dm), __fadd_rn(__fmul_rn(d, (float)((nb >> 4) & 0xf)), dm),
                     __fadd_rn(__fmul_rn(d, (float)((nb >> 8) & 0xf)), dm),
                     __fadd_rn(__fmul_rn(d, (float)((nb >> 12) & 0xf)), dm));
}

template <int HD, int FMT, int LAY>
__global__ void __launch_bounds__(THREADS) generic_kernel(const Params p) {
  constexpr int HP = HD + 4;            // padded row, floats
  constexpr int C4 = HD / 4;            // float4 chunks per row
  constexpr int HG = THREADS / HD;      // head groups in P.V (2 for hd 64, 1 for hd 128)
  constexpr int NH = (MAXG + HG - 1) / HG;
  __shared__ __align__(16) float qs[MAXG][HD];
  __shared__ __align__(16) float ks[TILE][HP];
  __shared__ __align__(16) float vs[TILE][HP];
  __shared__ float ps[MAXG][TILE];
  __shared__ float mh[MAXG], lh[MAXG], sch[MAXG];
  __shared__ const uint8_t* rowp[2][TILE];
  __shared__ int last;
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, rk = blockIdx.y, b = rk / p.n_kv, kv = rk % p.n_kv;
  const int G = p.group, H = p.n_kv * G;
  int64_t lo, hi;
  row_range(p, b, lo, hi);
  const int64_t s0 = lo + (int64_t)split * p.split_len;
  const int64_t s1 = s0 + p.split_len < hi ? s0 + p.split_len : hi;
  for (int i = tid; i < G * HD; i += THREADS) {
    const int h = i / HD, d = i % HD;
    const int64_t qi = ((int64_t)b * H + kv * G + h) * HD + d;
    const float x = p.q_bf16 ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(p.q)[qi] << 16)
                             : reinterpret_cast<const float*>(p.q)[qi];
    qs[h][d] = x * p.qscale;
  }
  if (tid < MAXG) {
    mh[tid] = -INFINITY;
    lh[tid] = 0.f;
  }
  const int d = tid % HD, hg = tid / HD;
  float acc[NH];
#pragma unroll
  for (int k = 0; k < NH; ++k) acc[k] = 0.f;
  __syncthreads();

  for (int64_t t0 = s0; t0 < s1; t0 += TILE) {
    if (tid < 2 * TILE) {
      const int i = tid % TILE, which = tid / TILE;
      const int64_t t = t0 + i;
      rowp[which][i] = t < s1 ? kv_row<HD, FMT, LAY>(p, b, kv, t, which) : nullptr;
    }
    __syncthreads();
    for (int idx = tid; idx < TILE * C4; idx += THREADS) {
      const int i = idx / C4, c = idx % C4;
      const uint8_t* kr = rowp[0][i];
      const uint8_t* vr = rowp[1][i];
      const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
      const bool live = kr && vr;
      *reinterpret_cast<float4*>(&ks[i][4 * c]) = live ? load4<HD, FMT>(kr, c) : zero;
      *reinterpret_cast<float4*>(&vs[i][4 * c]) = live ? load4<HD, FMT>(vr, c) : zero;
    }
    __syncthreads();
    // scores (log2 units): thread = (head, token)
    for (int j = tid; j < G * TILE; j += THREADS) {
      const int h = j / TILE, i = j % TILE;
      float s = -INFINITY;
      if (rowp[0][i] && rowp[1][i]) {
        s = 0.f;
#pragma unroll
        for (int c = 0; c < C4; ++c) {
          const float4 kk = *reinterpret_cast<const float4*>(&ks[i][4 * c]);
          const float4 qq = *reinterpret_cast<const float4*>(&qs[h][4 * c]);
          s = fmaf(qq.x, kk.x, fmaf(qq.y, kk.y, fmaf(qq.z, kk.z, fmaf(qq.w, kk.w, s))));
        }
      }
      ps[h][i] = s;
    }
    __syncthreads();
    // online softmax: warp = head, lane = token
    for (int h = warp; h < G; h += THREADS / 32) {
      const float s = ps[h][lane];
      const float mx = warp_max(s);
      const float mo = mh[h];
      const float mn = fmaxf(mo, mx);
      float pe = 0.f, scale = 1.f;
      if (mn > -INFINITY) {
        pe = exp2f(s - mn);
        scale = mo > -INFINITY ? exp2f(mo - mn) : 0.f;
      }
      const float sum = warp_sum(pe);
      ps[h][lane] = pe;
      if (lane == 0) {
        mh[h] = mn;
        lh[h] = lh[h] * scale + sum;
        sch[h] = scale;
      }
    }
    __syncthreads();
    // P.V: thread = (dim d, head group hg): heads hg, hg + HG, ...
#pragma unroll
    for (int k = 0; k < NH; ++k) {
      const int h = hg + k * HG;
      if (h < G) acc[k] *= sch[h];
    }
#pragma unroll 8
    for (int i = 0; i < TILE; ++i) {
      const float vv = vs[i][d];
#pragma unroll
      for (int k = 0; k < NH; ++k) {
        const int h = hg + k * HG;
        if (h < G) acc[k] = fmaf(ps[h][i], vv, acc[k]);
      }
    }
    __syncthreads();   // the tile buffers are rewritten next
  }

  const int64_t orow = (int64_t)b * H + kv * G;   // first query head of this KV head
  if (p.n_splits == 1) {
#pragma unroll
    for (int k = 0; k < NH; ++k) {
      const int h = hg + k * HG;
      if (h >= G) continue;
      const float L = lh[h];
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      if (p.part_mode) {
        float* dst = p.out + (orow + h) * (HD + 2);
        dst[d] = acc[k] * inv;
        if (d == 0) {
          dst[HD] = L > 0.f ? mh[h] * 0.6931471805599453f : -INFINITY;
          dst[HD + 1] = L;
        }
      } else {
        p.out[(orow + h) * HD + d] = acc[k] * inv;
      }
    }
    return;
  }
  // split partial, then the last CTA of (row, KV head) merges
  {
    float* mine = p.ws_part + ((int64_t)rk * p.n_splits + split) * MAXG * (HD + 2);
#pragma unroll
    for (int k = 0; k < NH; ++k) {
      const int h = hg + k * HG;
      if (h >= G) continue;
      __stcg(mine + h * (HD + 2) + d, acc[k]);
      if (d == 0) {
        __stcg(mine + h * (HD + 2) + HD, mh[h]);
        __stcg(mine + h * (HD + 2) + HD + 1, lh[h]);
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(p.cnt + rk) : "memory");
    last = old == p.n_splits - 1;
    if (last) atomicExch(p.cnt + rk, 0);
  }
  __syncthreads();
  if (!last) return;
  const float* base = p.ws_part + (int64_t)rk * p.n_splits * MAXG * (HD + 2);
#pragma unroll
  for (int k = 0; k < NH; ++k) {
    const int h = hg + k * HG;
    if (h >= G) continue;
    float M = -INFINITY;
    for (int sp = 0; sp < p.n_splits; ++sp) {
      const float* src = base + ((int64_t)sp * MAXG + h) * (HD + 2);
      if (__ldcg(src + HD + 1) > 0.f) M = fmaxf(M, __ldcg(src + HD));
    }
    float L = 0.f, o = 0.f;
    if (M > -INFINITY) {
      for (int sp = 0; sp < p.n_splits; ++sp) {
        const float* src = base + ((int64_t)sp * MAXG + h) * (HD + 2);
        const float l = __ldcg(src + HD + 1);
        if (!(l > 0.f)) continue;
        const float w = exp2f(__ldcg(src + HD) - M);
        L = fmaf(w, l, L);
        o = fmaf(w, __ldcg(src + d), o);
      }
    }
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    if (p.part_mode) {
      float* dst = p.out + (orow + h) * (HD + 2);
      dst[d] = o * inv;
      if (d == 0) {
        dst[HD] = L > 0.f ? M * 0.6931471805599453f : -INFINITY;
        dst[HD + 1] = L;
      }
    } else {
      p.out[(orow + h) * HD + d] = o * inv;
    }
  }
}

template <int HD>
int32_t launch_hd(const Params& p, int fmt, int lay, dim3 grid, cudaStream_t stream) {
#define NYION_GEN_CASE(F, L)                                                                                   \
  if (fmt == F && lay == L)                                                                                    \
    return check_cuda(launch_pdl(generic_kernel<HD, F, L>, grid, dim3(THREADS), 0, stream, p), "generic decode launch");
  NYION_GEN_CASE(kF32, kPaged)
  NYION_GEN_CASE(kQ4, kPaged)
  NYION_GEN_CASE(kBF16, kPaged)
  NYION_GEN_CASE(kF32, kRows)
  NYION_GEN_CASE(kF16, kRows)
  NYION_GEN_CASE(kF32, kZoned)
#undef NYION_GEN_CASE
  return fail(NYION_ERR_UNSUPPORTED, "generic decode: no kernel for format %d, layout %d", fmt, lay);
}

}  // namespace gen

bool generic_shape_ok(int n_heads, int n_kv_heads, int head_dim) {
  return n_kv_heads > 0 && n_heads > 0 && n_heads % n_kv_heads == 0 && n_heads / n_kv_heads <= gen::MAXG &&
         (head_dim == 64 || head_dim == 128);
}

int32_t generic_decode(const GenericCall& c, cudaStream_t stream) {
  using namespace gen;
  if (!generic_shape_ok(c.n_heads, c.n_kv, c.head_dim))
    return fail(NYION_ERR_UNSUPPORTED,
                "%s: shapes take head_dim 64 or 128 and 1 to 8 query heads per KV head (got head_dim %d, %d/%d)",
                c.who, c.head_dim, c.n_heads, c.n_kv);
  if (c.rows <= 0 || c.max_tokens < 0) return fail(NYION_ERR_INVALID, "%s: bad sizes", c.who);
  DeviceInfo* dev = nullptr;
  int32_t st = device_info(&dev);
  if (st) return st;
  const int hd = c.head_dim, G = c.n_heads / c.n_kv;
  const int pairs = c.rows * c.n_kv;
  // splits: about four CTAs per SM over the whole call, tiles of 32 tokens each
  int n_splits = (4 * dev->num_sms + pairs - 1) / pairs;
  const int max_tiles = (int)((c.max_tokens + TILE - 1) / TILE);
  if (n_splits > max_tiles) n_splits = max_tiles;
  if (n_splits > MAXSPLIT) n_splits = MAXSPLIT;
  if (n_splits < 1) n_splits = 1;
  int64_t split_len = (c.max_tokens + n_splits - 1) / n_splits;
  split_len = (split_len + TILE - 1) / TILE * TILE;
  if (split_len < TILE) split_len = TILE;
  if (split_len > (1ll << 30)) return fail(NYION_ERR_INVALID, "%s: context too long", c.who);
  // library-owned workspace: per-(row, KV head) counters first, then the split partials
  const int rows_per_launch = 65535 / c.n_kv > 0 ? 65535 / c.n_kv : 1;
  const int lrows = c.rows < rows_per_launch ? c.rows : rows_per_launch;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t cnt_bytes = al((size_t)lrows * c.n_kv * sizeof(int32_t));
  const size_t part_bytes = n_splits > 1 ? (size_t)lrows * c.n_kv * n_splits * MAXG * (hd + 2) * sizeof(float) : 0;
  void* ws = nullptr;
  st = internal_workspace(cnt_bytes + part_bytes, &ws, kWsCounters, cnt_bytes, stream);
  if (st) return st;
  for (int r0 = 0; r0 < c.rows; r0 += lrows) {
    const int nr = c.rows - r0 < lrows ? c.rows - r0 : lrows;
    Params p{};
    const size_t qelt = c.q_bf16 ? 2 : 4;
    p.q = static_cast<const uint8_t*>(c.q) + (size_t)r0 * c.n_heads * hd * qelt;
    p.q_bf16 = c.q_bf16;
    p.k = static_cast<const uint8_t*>(c.k);
    p.v = static_cast<const uint8_t*>(c.v);
    p.table = c.table ? (c.table_shared ? c.table : c.table + (int64_t)r0 * c.max_pages) : nullptr;
    p.table_shared = c.table_shared;
    p.max_pages = c.max_pages;
    p.n_pool_pages = c.n_pool_pages;
    p.n_kv = c.n_kv;
    p.group = G;
    p.rows = nr;
    p.lens = c.lens ? c.lens + r0 : nullptr;
    p.tok_begin = c.tok_begin ? c.tok_begin + r0 : nullptr;
    p.tok_end = c.tok_end ? c.tok_end + r0 : nullptr;
    p.u_begin = c.u_begin;
    p.u_end = c.u_end;
    p.causal_base = c.causal_base >= 0 ? c.causal_base + r0 : -1;
    p.d_len = c.d_len;
    p.window = c.window;
    p.stride = c.stride;
    p.n_layers = c.n_layers;
    p.layer = c.layer;
    p.n_pages = c.n_pages;
    p.qscale = (c.scale > 0.f ? c.scale : 1.0f / sqrtf((float)hd)) * 1.4426950408889634f;
    p.n_splits = n_splits;
    p.split_len = (int32_t)split_len;
    p.part_mode = c.part_mode;
    p.out = c.out + (size_t)r0 * c.n_heads * (c.part_mode ? hd + 2 : hd);
    p.cnt = static_cast<int32_t*>(ws);
    p.ws_part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + cnt_bytes);
    p.err = dev->err_word;
    const dim3 grid((unsigned)n_splits, (unsigned)(nr * c.n_kv));
    st = hd == 64 ? gen::launch_hd<64>(p, c.fmt, c.layout, grid, stream)
                  : gen::launch_hd<128>(p, c.fmt, c.layout, grid, stream);
    if (st) return st;
  }
  return NYION_OK;
}

}  // namespace nyion
