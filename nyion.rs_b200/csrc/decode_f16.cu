// decode_f16.cu — decode attention over f16 KV caches laid out
// [n_kv_heads][stride][64]:
//
//   * the reference's contiguous half cache behind gpu_attention_streamed_half
//     and gpu_graph_create_attention_half
//     (swamp-gpu/kernels/fused_attention.cu:534-582, :687-717);
//   * the layer-graph attention node over the f16 ring, whose length is read
//     from device memory at run time so one captured graph serves every
//     position (kernel_scores_dptr / kernel_softmax_v_dptr,
//     fused_attention.cu:1505-1556, captured at :1631-1638; the scheduler
//     clamps the length to the ring window, scheduler.rs:103-171).
//
// The work is a few MB per call and launch-latency bound, so the design is
// plain: CTA = (KV head, 256-token split), warp = one query head of the GQA
// group, lane = one token of a 32-token chunk for the scores (f16 row read
// as 8 x 16 B, fp32 dot with the pre-scaled query held in registers) and two
// output dims for P.V; online softmax in the log2 domain; each CTA writes a
// log-sum-exp partial per head that nyion_attn_lse_combine merges.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "host.h"

extern "C" int32_t nyion_attn_lse_combine(const float* parts, int32_t n_parts, int64_t rows,
                                          int32_t head_dim, float* out, void* stream);

namespace nyion {
namespace f16dec {

constexpr int HD = 64;
constexpr int GROUP = 8;
constexpr int SPLIT = 256;                 // tokens per CTA
constexpr int THREADS = 32 * GROUP;
constexpr int PART = HD + 2;               // o / l, m (natural log units), l

struct Params {
  const float* q;                // [n_heads][64]
  const __half* k;               // [n_kv][stride][64]
  const __half* v;
  float* part;                   // [n_split][n_heads][66]
  int n_kv;
  int64_t stride;
  int seq_len;                   // host length (contiguous cache)
  const int32_t* d_seq_len;      // device length (ring), or null
  int window;                    // ring window: the device length is clamped to it
  float sl2;                     // scale * log2(e)
};

__global__ void __launch_bounds__(THREADS) f16_partial_kernel(const Params p) {
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = p.n_kv * GROUP;
  const int h = kvh * GROUP + w;
  int n = p.seq_len;
  if (p.d_seq_len) {
    n = *p.d_seq_len;
    n = n < 0 ? 0 : (n > p.window ? p.window : n);
  }
  const int t_begin = split * SPLIT;
  const int t_end = min(t_begin + SPLIT, n);
  float* dst = p.part + ((int64_t)split * H + h) * PART;
  if (t_begin >= t_end) {                          // nothing to attend in this split
    dst[2 * lane] = 0.f;
    dst[2 * lane + 1] = 0.f;
    if (lane == 0) {
      dst[HD] = -INFINITY;
      dst[HD + 1] = 0.f;
    }
    return;
  }
  float qr[HD];
#pragma unroll
  for (int d = 0; d < HD; d += 4) {
    const float4 v4 = *reinterpret_cast<const float4*>(p.q + (int64_t)h * HD + d);
    qr[d] = v4.x * p.sl2;
    qr[d + 1] = v4.y * p.sl2;
    qr[d + 2] = v4.z * p.sl2;
    qr[d + 3] = v4.w * p.sl2;
  }
  const __half* kb = p.k + (int64_t)kvh * p.stride * HD;
  const __half* vb = p.v + (int64_t)kvh * p.stride * HD;
  float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
  for (int t0 = t_begin; t0 < t_end; t0 += 32) {
    const int t = t0 + lane;
    float s = -INFINITY;
    if (t < t_end) {
      const uint4* row = reinterpret_cast<const uint4*>(kb + (int64_t)t * HD);
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) {
        const uint4 u = __ldg(row + c);
        const __half2* hh = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(hh[e]);
          acc = fmaf(qr[8 * c + 2 * e], f.x, acc);
          acc = fmaf(qr[8 * c + 2 * e + 1], f.y, acc);
        }
      }
      s = acc;
    }
    const float mn = fmaxf(m, warp_max(s));        // finite: token t0 is valid
    const float alpha = exp2f(m - mn);
    const float pt = (t < t_end) ? exp2f(s - mn) : 0.f;
    l = fmaf(l, alpha, warp_sum(pt));
    o0 *= alpha;
    o1 *= alpha;
    const int cnt = min(32, t_end - t0);
    const __half2* vrow = reinterpret_cast<const __half2*>(vb + (int64_t)t0 * HD) + lane;
    for (int j = 0; j < cnt; ++j) {
      const float pj = __shfl_sync(0xffffffffu, pt, j);
      const float2 f = __half22float2(__ldg(vrow + (int64_t)j * (HD / 2)));
      o0 = fmaf(pj, f.x, o0);
      o1 = fmaf(pj, f.y, o1);
    }
    m = mn;
  }
  const float inv = 1.0f / l;
  dst[2 * lane] = o0 * inv;
  dst[2 * lane + 1] = o1 * inv;
  if (lane == 0) {
    dst[HD] = m * 0.69314718055994531f;           // back to natural-log units
    dst[HD + 1] = l;
  }
}

int n_splits(int max_tokens) { return max_tokens <= 0 ? 1 : (max_tokens + SPLIT - 1) / SPLIT; }

size_t workspace_bytes(int n_heads, int max_tokens) {
  return (size_t)n_splits(max_tokens) * n_heads * PART * sizeof(float);
}

int32_t run(const float* q, const void* k, const void* v, int64_t stride, int seq_len,
            const int32_t* d_seq_len, int window, float* out, int n_heads, int n_kv, int head_dim,
            float scale, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (!q || !k || !v || !out) return fail(NYION_ERR_INVALID, "f16 decode: null pointer argument");
  if (head_dim != HD || n_kv <= 0 || n_heads != n_kv * GROUP)
    return fail(NYION_ERR_UNSUPPORTED, "f16 decode: this build takes head_dim 64 and GQA group 8 (got %d, %d/%d)",
                head_dim, n_heads, n_kv);
  const int max_tokens = d_seq_len ? window : seq_len;
  if (max_tokens <= 0 || stride < max_tokens)
    return fail(NYION_ERR_INVALID, "f16 decode: length %d must be in [1, stride=%lld]", max_tokens,
                (long long)stride);
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
    return fail(NYION_ERR_INVALID, "f16 decode: K/V must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(q) & 15) return fail(NYION_ERR_INVALID, "f16 decode: q must be 16-byte aligned");
  const size_t need = workspace_bytes(n_heads, max_tokens);
  if (!ws) {
    int32_t st = internal_workspace(need, &ws);
    if (st) return st;
  } else if (ws_bytes < need) {
    return fail(NYION_ERR_WORKSPACE, "f16 decode: workspace %zu B < %zu B", ws_bytes, need);
  }
  Params p{};
  p.q = q;
  p.k = static_cast<const __half*>(k);
  p.v = static_cast<const __half*>(v);
  p.part = static_cast<float*>(ws);
  p.n_kv = n_kv;
  p.stride = stride;
  p.seq_len = seq_len;
  p.d_seq_len = d_seq_len;
  p.window = window;
  p.sl2 = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  const int ns = n_splits(max_tokens);
  f16_partial_kernel<<<dim3((unsigned)n_kv, (unsigned)ns), THREADS, 0, stream>>>(p);
  int32_t st = check_cuda(cudaGetLastError(), "f16 decode launch");
  if (st) return st;
  return nyion_attn_lse_combine(p.part, ns, n_heads, HD, out, stream);
}

}  // namespace f16dec
}  // namespace nyion

using namespace nyion;

extern "C" size_t nyion_attn_f16_workspace_size(int32_t n_heads, int32_t max_tokens) {
  return f16dec::workspace_bytes(n_heads, max_tokens);
}

extern "C" int32_t nyion_attn_decode_contig_f16(const float* q, const void* k_cache, const void* v_cache,
                                                float* out, int32_t n_heads, int32_t n_kv_heads,
                                                int32_t seq_len, int32_t head_dim, int32_t kv_stride,
                                                float scale, void* workspace, size_t workspace_bytes,
                                                void* stream) {
  return f16dec::run(q, k_cache, v_cache, kv_stride, seq_len, nullptr, 0, out, n_heads, n_kv_heads,
                     head_dim, scale, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int32_t nyion_attn_decode_ring_f16(const float* q, const void* k_ring, const void* v_ring,
                                              const int32_t* d_seq_len, float* out, int32_t n_heads,
                                              int32_t n_kv_heads, int32_t head_dim, int32_t window,
                                              float scale, void* workspace, size_t workspace_bytes,
                                              void* stream) {
  if (!d_seq_len) return fail(NYION_ERR_INVALID, "decode_ring_f16: null device length");
  return f16dec::run(q, k_ring, v_ring, window, 0, d_seq_len, window, out, n_heads, n_kv_heads, head_dim,
                     scale, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int gpu_attention_streamed_half(const float* d_q, const void* d_k_cache, const void* d_v_cache,
                                           float* d_output, int n_heads, int n_kv_heads, int seq_len,
                                           int head_dim, int kv_stride, void* stream) {
  return nyion_attn_decode_contig_f16(d_q, d_k_cache, d_v_cache, d_output, n_heads, n_kv_heads, seq_len,
                                      head_dim, kv_stride, 0.f, nullptr, 0, stream) == NYION_OK
             ? 0
             : -1;
}

extern "C" void* gpu_graph_create_attention_half(const float* d_q, const void* d_k_cache,
                                                 const void* d_v_cache, float* d_scores, float* d_output,
                                                 int n_heads, int n_kv_heads, int seq_len, int head_dim,
                                                 int kv_stride) {
  (void)d_scores;   // scores never leave the SM
  DeviceInfo* dev = nullptr;
  if (device_info(&dev)) return nullptr;
  const size_t wsb = f16dec::workspace_bytes(n_heads > 0 ? n_heads : 1, seq_len);
  void* ws = nullptr;
  if (check_cuda(cudaMalloc(&ws, wsb), "cudaMalloc(graph workspace)")) return nullptr;
  cudaStream_t s;
  if (check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) {
    cudaFree(ws);
    return nullptr;
  }
  cudaGraph_t g = nullptr;
  cudaGraphExec_t exec = nullptr;
  bool ok = check_cuda(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "BeginCapture") == 0;
  if (ok) {
    const int32_t rc = nyion_attn_decode_contig_f16(d_q, d_k_cache, d_v_cache, d_output, n_heads, n_kv_heads,
                                                    seq_len, head_dim, kv_stride, 0.f, ws, wsb, s);
    const cudaError_t e = cudaStreamEndCapture(s, &g);
    ok = rc == NYION_OK && check_cuda(e, "EndCapture") == 0;
  }
  if (ok) ok = check_cuda(cudaGraphInstantiate(&exec, g, 0), "cudaGraphInstantiate") == 0;
  if (g) cudaGraphDestroy(g);
  cudaStreamDestroy(s);
  if (!ok) {
    cudaFree(ws);
    return nullptr;
  }
  return new AttnGraph{exec, ws};
}
