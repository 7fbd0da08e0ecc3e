// gemv_q4k.cu — the output projection that follows attention in the layer
// graph (step 6 of gpu_graph_create_layer): the reference CUDA Q4_K GEMV
// (swamp-gpu/kernels/fused_attention.cu:858-925), so the attention output
// stays on the device.
//
// Weight format of that kernel: super-blocks of 256 columns, 144 bytes each
// [f16 d][f16 dmin][12 bytes of 6-bit scales / mins][128 bytes of nibbles],
// stored column-major at super-block level (block b of row r at
// (b * n_rows + r) * 144, gpu_upload_weights_transposed).  Sub-block sb
// (32 columns) has scale_sb / min_sb unpacked as the kernel does
// (j < 4: scale = s[j] & 63, min = s[4 + j] & 63; j >= 4: scale =
// (s[4 + j] & 15) | ((s[j - 4] >> 6) << 4), min = (s[4 + j] >> 4) |
// ((s[j] >> 6) << 4)), nibble k of sub-block sb = qs[16 sb + k/2] >> 4(k%2),
// weight = d (nib - 8) scale_sb + dmin min_sb — the reference kernel's
// formula, kept as written.
//
// B200 layout of the work: CTA = 32 rows x 8 warps; warp w takes super-blocks
// w, w + 8, ... of the CTA's rows, lane = row, so a warp reads 32 consecutive
// 144-byte blocks (4.6 KB contiguous) with 16-byte loads; x (up to 4 rows of
// the batch per pass) sits in shared memory; per-row sums of the super-blocks
// are added in block order through shared memory.
#include <cuda_fp16.h>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace q4k {

constexpr int SB = 144;
constexpr int COLS = 256;
constexpr int ROWS_CTA = 32;
constexpr int WARPS = 8;
constexpr int THREADS = 32 * WARPS;
constexpr int BT = 4;              // batch rows per pass

// dot of one super-block (144 B at `blk`) with x[0..256) for BT batch rows
template <int NB>
__device__ __forceinline__ void block_dot(const uint8_t* __restrict__ blk, const float* __restrict__ xs, int xstride,
                                          float (&dot)[BT]) {
  uint4 raw[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) raw[i] = __ldg(reinterpret_cast<const uint4*>(blk) + i);
  const uint8_t* b = reinterpret_cast<const uint8_t*>(raw);
  const float d = __half2float(__ushort_as_half((unsigned short)(b[0] | (b[1] << 8))));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(b[2] | (b[3] << 8))));
  float sc[8], mn[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sc[j] = (float)(b[4 + j] & 63);
    mn[j] = (float)(b[8 + j] & 63);
  }
#pragma unroll
  for (int j = 4; j < 8; ++j) {
    sc[j] = (float)((b[8 + j] & 0xF) | ((b[4 + j - 4] >> 6) << 4));
    mn[j] = (float)((b[8 + j] >> 4) | ((b[4 + j] >> 6) << 4));
  }
#pragma unroll
  for (int r = 0; r < BT; ++r) dot[r] = 0.f;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const float ds = d * sc[s], mm = dmin * mn[s];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const int nib = (b[16 + s * 16 + k / 2] >> ((k % 2) * 4)) & 0x0F;
      const float wv = fmaf(ds, (float)(nib - 8), mm);
#pragma unroll
      for (int r = 0; r < NB; ++r) dot[r] = fmaf(wv, xs[r * xstride + s * 32 + k], dot[r]);
    }
  }
}

__global__ void __launch_bounds__(THREADS) gemv_kernel(const uint8_t* __restrict__ w, const float* __restrict__ x,
                                                       float* __restrict__ out, int n_rows, int n_blocks,
                                                       int batch) {
  extern __shared__ float smem[];
  float* xs = smem;                                   // [BT][n_blocks * 256]
  float* part = smem + BT * n_blocks * COLS;          // [n_blocks][BT][32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * ROWS_CTA + lane;
  const int n_cols = n_blocks * COLS;
  for (int b0 = 0; b0 < batch; b0 += BT) {
    const int nb = min(BT, batch - b0);
    __syncthreads();
    for (int i = threadIdx.x; i < nb * n_cols; i += THREADS) xs[i] = x[(int64_t)b0 * n_cols + i];
    __syncthreads();
    for (int blk = warp; blk < n_blocks; blk += WARPS) {
      float dot[BT] = {0.f, 0.f, 0.f, 0.f};
      if (row < n_rows) {
        const uint8_t* bp = w + ((int64_t)blk * n_rows + row) * SB;
        if (nb == BT) block_dot<BT>(bp, xs + blk * COLS, n_cols, dot);
        else if (nb == 3) block_dot<3>(bp, xs + blk * COLS, n_cols, dot);
        else if (nb == 2) block_dot<2>(bp, xs + blk * COLS, n_cols, dot);
        else block_dot<1>(bp, xs + blk * COLS, n_cols, dot);
      }
#pragma unroll
      for (int r = 0; r < BT; ++r) part[(blk * BT + r) * 32 + lane] = dot[r];
    }
    __syncthreads();
    // per (batch row, output row): super-block sums added in block order
    if (threadIdx.x < nb * 32) {
      const int r = threadIdx.x >> 5;
      float total = 0.f;
      for (int blk = 0; blk < n_blocks; ++blk) total += part[(blk * BT + r) * 32 + lane];
      if (row < n_rows) out[(int64_t)(b0 + r) * n_rows + row] = total;
    }
  }
}

size_t smem_bytes(int n_blocks) { return (size_t)BT * n_blocks * COLS * 4 + (size_t)n_blocks * BT * 32 * 4; }

}  // namespace q4k
}  // namespace nyion

using namespace nyion;
using namespace nyion::q4k;

extern "C" int32_t nyion_attn_gemv_q4k(const uint8_t* w, const float* x, float* out, int32_t n_rows, int32_t n_blocks,
                                       int32_t batch, void* stream) {
  if (!w || !x || !out) return fail(NYION_ERR_INVALID, "gemv_q4k: null pointer argument");
  if (n_rows <= 0 || n_blocks <= 0 || batch <= 0) return fail(NYION_ERR_INVALID, "gemv_q4k: sizes must be > 0");
  if (reinterpret_cast<uintptr_t>(w) & 15) return fail(NYION_ERR_INVALID, "gemv_q4k: weights must be 16-byte aligned");
  const size_t sm = smem_bytes(n_blocks);
  if (sm > 227 * 1024) return fail(NYION_ERR_UNSUPPORTED, "gemv_q4k: n_blocks %d too large for one pass", n_blocks);
  if (sm > 48 * 1024) {   // the limit is raised once per device to the largest size any call may use
    const int32_t st = kernel_setup(reinterpret_cast<const void*>(gemv_kernel), 227 * 1024, THREADS, nullptr);
    if (st) return st;
  }
  gemv_kernel<<<(n_rows + ROWS_CTA - 1) / ROWS_CTA, THREADS, sm, static_cast<cudaStream_t>(stream)>>>(
      w, x, out, n_rows, n_blocks, batch);
  return check_cuda(cudaGetLastError(), "gemv_q4k launch");
}

// fused_attention.cu:916-925: same name and arguments (void, device pointers)
extern "C" void gpu_gemv_q4k(const uint8_t* d_w, const float* d_x, float* d_out, int n_rows, int n_blocks,
                             void* stream) {
  nyion_attn_gemv_q4k(d_w, d_x, d_out, n_rows, n_blocks, 1, stream);
}
