// mojo_ffi.cu — the reference's Mojo FFI entry point `sparse_attention_q4`
// (swamp-gpu/kernels/attention.mojo:40-152, bound by swamp-gpu/src/mojo.rs:5,
// 65-97), same symbol and the argument list the Rust side declares:
// (u64 q, u64 k_q4, u64 v_q4, u64 positions, u64 out, i32 n_heads,
//  i32 head_dim, i32 n_sparse, i32 window, i32 global_stride), host pointers.
//
// Buffer format of that kernel: a row of head_dim values is ceil(hd/32)
// blocks of 20 f32 elements [d, dmin, 16 "nibble bytes" stored as floats
// 0..255, 2 unused]; element i of a block is ((int)byte[i/2] >> 4(i%2)) & 15,
// value d * nib + dmin.  Row t (a position) starts at element t * blocks * 20.
// One KV row set serves every head (no GQA mapping); window and
// global_stride are unused by the kernel (the Rust caller passes
// n_heads * head_dim * 4 as the last argument).
//
// Semantics kept as written, including its tile quirk: positions are taken
// in tiles of 64; per tile the running (m, d) is updated as
// d = d e^(m - m') + sum_tile e^(s - m_tile) e^(m_tile - m'), then every
// position of that tile adds v * e^(s - m') / d to the output with the
// tile's (m', d) — earlier tiles are never rescaled — and weights below 1e-8
// are skipped.  scale = 1 / sqrt(head_dim).
//
// Host side: the rows named by `positions` are gathered into pinned staging
// (only those rows cross to the device), q is uploaded, one CTA per head
// runs the tiles in order (threads = positions for the scores, then threads =
// output dims, each summing its dim over the tile's positions in order), and
// the output is copied back; the call returns when `out` is written.
#include <math.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace mojo {

constexpr int TILE = 64;
constexpr int BLOCK = 32;
constexpr int BLOCK_F = 20;
constexpr int MAX_HD = 256;
constexpr int THREADS = 256;

__device__ __forceinline__ float dequant(const float* row, int i) {
  const float* blk = row + (i / BLOCK) * BLOCK_F;
  const int j = i % BLOCK;
  const int byte = (int)blk[2 + j / 2];
  const int nib = (byte >> ((j % 2) * 4)) & 0x0F;
  return __fadd_rn(__fmul_rn(blk[0], (float)nib), blk[1]);
}

__global__ void __launch_bounds__(THREADS) mojo_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                       const float* __restrict__ v, int n_sparse, int head_dim,
                                                       float scale, float* __restrict__ out) {
  __shared__ float sc[TILE];
  __shared__ float w[TILE];
  __shared__ float mstate[2];
  const int h = blockIdx.x, t = threadIdx.x;
  const int blocks = (head_dim + BLOCK - 1) / BLOCK;
  const int row_f = blocks * BLOCK_F;
  const float* qh = q + (int64_t)h * head_dim;
  float acc = 0.f;                                  // output dim t (t < head_dim)
  if (t == 0) {
    mstate[0] = -1e10f;
    mstate[1] = 0.f;
  }
  for (int t0 = 0; t0 < n_sparse; t0 += TILE) {
    const int n_tile = min(TILE, n_sparse - t0);
    // scores: thread = position of the tile
    if (t < n_tile) {
      const float* kr = k + (int64_t)(t0 + t) * row_f;
      float dot = 0.f;
      for (int i = 0; i < head_dim; ++i) dot = __fadd_rn(dot, __fmul_rn(dequant(kr, i), qh[i]));
      sc[t] = __fmul_rn(dot, scale);
    }
    __syncthreads();
    // tile max (initial -1e10) and tile sum of exp(s - max), in position order
    if (t == 0) {
      float mx = -1e10f;
      for (int i = 0; i < n_tile; ++i) mx = sc[i] > mx ? sc[i] : mx;
      float td = 0.f;
      for (int i = 0; i < n_tile; ++i) td = __fadd_rn(td, expf(__fsub_rn(sc[i], mx)));
      const float m = mstate[0], d = mstate[1];
      const float nm = fmaxf(m, mx);
      mstate[1] = __fadd_rn(__fmul_rn(d, expf(__fsub_rn(m, nm))), __fmul_rn(td, expf(__fsub_rn(mx, nm))));
      mstate[0] = nm;
    }
    __syncthreads();
    if (t < n_tile) w[t] = __fdiv_rn(expf(__fsub_rn(sc[t], mstate[0])), mstate[1]);
    __syncthreads();
    // weighted sum: thread = output dim, positions in order
    if (t < head_dim) {
      for (int i = 0; i < n_tile; ++i) {
        const float wi = w[i];
        if (wi < 1e-8f) continue;
        acc = __fadd_rn(acc, __fmul_rn(dequant(v + (int64_t)(t0 + i) * row_f, t), wi));
      }
    }
    __syncthreads();
  }
  if (t < head_dim) out[(int64_t)h * head_dim + t] = acc;
}

struct Buffers {
  float* dev = nullptr;       // q | k rows | v rows | out
  size_t dev_bytes = 0;
  float* pinned = nullptr;    // staging of the same
  size_t pinned_bytes = 0;
};
std::mutex g_mu;
std::vector<Buffers> g_buf;

}  // namespace mojo
}  // namespace nyion

using namespace nyion;
using namespace nyion::mojo;

extern "C" void sparse_attention_q4(uint64_t q_ptr, uint64_t k_q4_ptr, uint64_t v_q4_ptr, uint64_t positions_ptr,
                                    uint64_t out_ptr, int32_t n_heads, int32_t head_dim, int32_t n_sparse,
                                    int32_t window, int32_t global_stride) {
  (void)window;
  (void)global_stride;
  const float* q = reinterpret_cast<const float*>(q_ptr);
  const float* kq = reinterpret_cast<const float*>(k_q4_ptr);
  const float* vq = reinterpret_cast<const float*>(v_q4_ptr);
  const int32_t* pos = reinterpret_cast<const int32_t*>(positions_ptr);
  float* out = reinterpret_cast<float*>(out_ptr);
  if (!q || !out || n_heads <= 0 || head_dim <= 0) return;
  if (head_dim > MAX_HD) {
    fail(NYION_ERR_UNSUPPORTED, "sparse_attention_q4: head_dim > %d", MAX_HD);
    return;
  }
  if (n_sparse <= 0) {   // the reference's loops leave zeros
    memset(out, 0, (size_t)n_heads * head_dim * sizeof(float));
    return;
  }
  if (!kq || !vq || !pos) {
    fail(NYION_ERR_INVALID, "sparse_attention_q4: null k_q4 / v_q4 / positions");
    return;
  }
  int dev = -1;
  if (check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return;
  const int row_f = (head_dim + BLOCK - 1) / BLOCK * BLOCK_F;
  const size_t nq = (size_t)n_heads * head_dim, nr = (size_t)n_sparse * row_f;
  const size_t total = (nq + 2 * nr + nq) * sizeof(float);
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_buf.size() <= dev) g_buf.resize(dev + 1);
  Buffers& b = g_buf[dev];
  if (b.dev_bytes < total) {
    cudaFree(b.dev);
    cudaFreeHost(b.pinned);
    b.dev = nullptr;
    b.pinned = nullptr;
    b.dev_bytes = b.pinned_bytes = 0;
    if (check_cuda(cudaMalloc(&b.dev, total), "sparse_attention_q4 device buffers") ||
        check_cuda(cudaMallocHost(&b.pinned, total), "sparse_attention_q4 staging")) {
      cudaFree(b.dev);
      cudaFreeHost(b.pinned);
      b.dev = b.pinned = nullptr;
      return;
    }
    b.dev_bytes = b.pinned_bytes = total;
  }
  // gather q and the rows named by `positions` into the staging buffer
  float* hq = b.pinned;
  float* hk = hq + nq;
  float* hv = hk + nr;
  memcpy(hq, q, nq * sizeof(float));
  for (int i = 0; i < n_sparse; ++i) {
    const int64_t t = pos[i];
    if (t < 0) {
      fail(NYION_ERR_INVALID, "sparse_attention_q4: negative position at %d", i);
      return;
    }
    memcpy(hk + (size_t)i * row_f, kq + t * row_f, row_f * sizeof(float));
    memcpy(hv + (size_t)i * row_f, vq + t * row_f, row_f * sizeof(float));
  }
  cudaStream_t s = nullptr;
  const size_t in_bytes = (nq + 2 * nr) * sizeof(float);
  if (check_cuda(cudaMemcpyAsync(b.dev, b.pinned, in_bytes, cudaMemcpyHostToDevice, s), "sparse_attention_q4 upload"))
    return;
  float* dq = b.dev;
  float* dk = dq + nq;
  float* dv = dk + nr;
  float* dout = dv + nr;
  mojo_kernel<<<n_heads, THREADS, 0, s>>>(dq, dk, dv, n_sparse, head_dim, 1.0f / sqrtf((float)head_dim), dout);
  if (check_cuda(cudaGetLastError(), "sparse_attention_q4 launch")) return;
  if (check_cuda(cudaMemcpyAsync(b.pinned + nq + 2 * nr, dout, nq * sizeof(float), cudaMemcpyDeviceToHost, s),
                 "sparse_attention_q4 download") ||
      check_cuda(cudaStreamSynchronize(s), "sparse_attention_q4"))
    return;
  memcpy(out, b.pinned + nq + 2 * nr, nq * sizeof(float));
}
