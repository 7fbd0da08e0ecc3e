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
// The kernel is the row-cache decode of decode_contig.cu; this file holds the
// argument checks and the entry points.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace f16dec {

constexpr int HD = 64;
constexpr int GROUP = 8;

size_t workspace_bytes(int n_heads, int max_tokens) {
  return contig_workspace_bytes(n_heads / GROUP > 0 ? n_heads / GROUP : 1, max_tokens);
}

int32_t run(const float* q, const void* k, const void* v, int64_t stride, int seq_len,
            const int32_t* d_seq_len, int window, float* out, int n_heads, int n_kv, int head_dim,
            float scale, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (!q || !k || !v || !out) return fail(NYION_ERR_INVALID, "f16 decode: null pointer argument");
  if (!(head_dim == HD && n_kv > 0 && n_heads == n_kv * GROUP) && generic_shape_ok(n_heads, n_kv, head_dim)) {
    const int max_tokens = d_seq_len ? window : seq_len;
    if (max_tokens <= 0 || stride < max_tokens)
      return fail(NYION_ERR_INVALID, "f16 decode: length %d must be in [1, stride=%lld]", max_tokens,
                  (long long)stride);
    GenericCall c;
    c.who = "f16 decode";
    c.q = q;
    c.k = k;
    c.v = v;
    c.n_heads = n_heads;
    c.n_kv = n_kv;
    c.head_dim = head_dim;
    c.rows = 1;
    c.u_begin = 0;
    c.u_end = seq_len;
    c.d_len = d_seq_len;
    c.window = window;
    c.stride = stride;
    c.scale = scale;
    c.out = out;
    c.max_tokens = max_tokens;
    c.fmt = kGenF16;
    c.layout = kGenRows;
    return generic_decode(c, stream);
  }
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
  const float sl2 = (scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
  return contig_rows_f16(q, k, v, out, n_kv, stride, seq_len, d_seq_len, window, sl2, ws, ws_bytes, stream);
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
  if (check_cuda(cudaMemset(ws, 0, wsb), "cudaMemset(graph workspace)")) {   // merge counters start at 0
    cudaFree(ws);
    return nullptr;
  }
  cudaStream_t s;
  if (check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) {
    cudaFree(ws);
    return nullptr;
  }
  // one eager launch sets the kernel attributes outside capture
  if (nyion_attn_decode_contig_f16(d_q, d_k_cache, d_v_cache, d_output, n_heads, n_kv_heads, seq_len, head_dim,
                                   kv_stride, 0.f, ws, wsb, s) != NYION_OK ||
      check_cuda(cudaStreamSynchronize(s), "warm-up")) {
    cudaStreamDestroy(s);
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
