// softmax_stokes.cu — the two small C ABIs of swamp-kernels that sit on the
// attention path: the Q16.16 "p-adic" softmax (mojo_softmax_padic,
// swamp-kernels/src/lib.rs:97-223) and the Stokes KV store
// (mojo_stokes_init / append / free, lib.rs:27-85), with the same names and
// argument meaning, device-resident on B200.
//
// Softmax, bit-exact with the reference's AVX-512 path (the path it takes on
// an AVX-512 host):
//   fixed_i = (i32, saturating) (logit_i * (1 / max(T, 1e-6)) * 65536)
//   e_i     = exp_q16_16(fixed_i - max)        (wrapping i32 difference)
//             = 0 below -655360, 65536 at >= 0, else round(exp(x/65536)*65536)
//   inv     = 2^32 / sum e  (u64 division, kept as i32)
//   16-wide blocks: (u32)(e * inv) >> 16 (low 32 bits, logical shift);
//   tail: (i64)e * inv >> 16;  probs = fixed / 65536.
// exp is taken in double and rounded to float (the correctly rounded expf
// value).  glibc's expf, which Rust's f32::exp calls on Linux, is not always
// correctly rounded (glibc 2.39: 437 of the 655,360 inputs of exp_q16_16 get
// the other neighbour), but on none of those inputs does the difference
// survive round(e * 65536): the Q16.16 results agree on the whole domain.
// nyion_attn_exp_q16_16 exposes this function over an array so that a test
// compares every input with the CPU oracle bit for bit.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "host.h"

namespace nyion {
namespace smx {

constexpr int THREADS = 1024;

__device__ __forceinline__ int32_t sat_i32(float x) {   // Rust `as i32`
  if (x != x) return 0;
  if (x >= 2147483648.0f) return 2147483647;
  if (x <= -2147483648.0f) return (int32_t)0x80000000u;
  return __float2int_rz(x);
}

__device__ __forceinline__ int32_t exp_q16_16(int32_t x_fixed) {
  if (x_fixed < -655360) return 0;
  if (x_fixed >= 0) return 65536;
  const float x = __fdiv_rn(__int2float_rn(x_fixed), 65536.0f);
  const float e = __double2float_rn(exp((double)x));
  const float r = fmaxf(roundf(__fmul_rn(e, 65536.0f)), 0.0f);
  return (int32_t)r;
}

// One CTA: pass 1 fixed-point logits + max, pass 2 exponentials + sum, pass 3
// normalisation.  `probs` holds the integer e_i between passes.
__global__ void __launch_bounds__(THREADS) softmax_padic_kernel(const float* __restrict__ logits,
                                                               float* __restrict__ probs, int n,
                                                               float temperature) {
  __shared__ int32_t smax[THREADS / 32];
  __shared__ unsigned long long ssum[THREADS / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float inv_tmp = __fdiv_rn(1.0f, fmaxf(temperature, 1e-6f));
  int32_t* fo = reinterpret_cast<int32_t*>(probs);
  int32_t mx = (int32_t)0x80000000u;
  for (int i = t; i < n; i += THREADS) {
    const int32_t f = sat_i32(__fmul_rn(__fmul_rn(logits[i], inv_tmp), 65536.0f));
    fo[i] = f;
    mx = max(mx, f);
  }
  for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) smax[warp] = mx;
  __syncthreads();
  mx = smax[0];
  for (int w = 1; w < THREADS / 32; ++w) mx = max(mx, smax[w]);
  unsigned long long sum = 0;
  for (int i = t; i < n; i += THREADS) {
    const int32_t diff = (int32_t)((uint32_t)fo[i] - (uint32_t)mx);
    const int32_t e = exp_q16_16(diff);
    fo[i] = e;
    sum += (unsigned long long)e;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) ssum[warp] = sum;
  __syncthreads();
  sum = 0;
  for (int w = 0; w < THREADS / 32; ++w) sum += ssum[w];
  const int simd_end = (n / 16) * 16;
  const int32_t inv = sum > 0 ? (int32_t)(uint32_t)((1ull << 32) / sum) : 0;
  for (int i = t; i < n; i += THREADS) {
    int32_t v = fo[i];
    if (sum > 0) {
      if (i < simd_end) v = (int32_t)(((uint32_t)v * (uint32_t)inv) >> 16);
      else v = (int32_t)(((int64_t)v * (int64_t)inv) >> 16);
    }
    probs[i] = __fmul_rn(__int2float_rn(v), 1.0f / 65536.0f);
  }
}

// exp_q16_16 over an array (the test of the whole domain).
__global__ void exp_q16_16_kernel(const int32_t* __restrict__ x, int32_t* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = exp_q16_16(x[i]);
}

}  // namespace smx

// ---- Stokes KV store: device rows, host scores ------------------------------
// The reference keeps K, V and scores in Vecs and, above 4096 tokens, drains
// the first minimum-score token (order of the rest kept).  Here K and V rows
// live in HBM ([n][head_dim] each, capacity 4097 rows), scores on the host
// (they arrive from the host); eviction moves the rows after the evicted one
// down by one with two device copies through a scratch buffer.
struct StokesStore {
  int hd = 0;
  int n = 0;
  float* keys = nullptr;      // device [kCap][hd]
  float* values = nullptr;
  float* scratch = nullptr;   // device [kCap][hd]
  std::vector<float> scores;
  static constexpr int kKeep = 4096;
  static constexpr int kCap = kKeep + 1;
};

}  // namespace nyion

using namespace nyion;

extern "C" int32_t nyion_attn_softmax_padic(const float* logits, float* probs, int32_t n, float temperature,
                                            void* stream) {
  if (!logits || !probs || n <= 0) return NYION_OK;   // the reference returns silently
  smx::softmax_padic_kernel<<<1, smx::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(logits, probs, n,
                                                                                      temperature);
  return check_cuda(cudaGetLastError(), "softmax_padic launch");
}

extern "C" int32_t nyion_attn_exp_q16_16(const int32_t* x_fixed, int32_t* out, int64_t n, void* stream) {
  if (!x_fixed || !out || n < 0) return fail(NYION_ERR_INVALID, "exp_q16_16: bad arguments");
  if (n == 0) return NYION_OK;
  const int64_t blocks = (n + 255) / 256;
  smx::exp_q16_16_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x_fixed, out, n);
  return check_cuda(cudaGetLastError(), "exp_q16_16 launch");
}

// Same name, arguments and silence on bad input as the reference
// (host pointers; synchronous).
extern "C" void mojo_softmax_padic(const float* logits, float* probs, int n, float temperature) {
  if (!logits || !probs || n <= 0) return;
  float *dl = nullptr, *dp = nullptr;
  const size_t b = (size_t)n * sizeof(float);
  if (check_cuda(cudaMalloc(&dl, b), "cudaMalloc(logits)") || check_cuda(cudaMalloc(&dp, b), "cudaMalloc(probs)")) {
    cudaFree(dl);
    cudaFree(dp);
    return;
  }
  if (!check_cuda(cudaMemcpy(dl, logits, b, cudaMemcpyHostToDevice), "copy logits") &&
      nyion_attn_softmax_padic(dl, dp, n, temperature, nullptr) == NYION_OK)
    check_cuda(cudaMemcpy(probs, dp, b, cudaMemcpyDeviceToHost), "copy probs");
  cudaFree(dl);
  cudaFree(dp);
}

extern "C" void* mojo_stokes_init(int head_dim) {
  if (head_dim <= 0) {
    fail(NYION_ERR_INVALID, "mojo_stokes_init: head_dim %d", head_dim);
    return nullptr;
  }
  StokesStore* s = new StokesStore();
  s->hd = head_dim;
  const size_t b = (size_t)StokesStore::kCap * head_dim * sizeof(float);
  if (check_cuda(cudaMalloc(&s->keys, b), "cudaMalloc(stokes keys)") ||
      check_cuda(cudaMalloc(&s->values, b), "cudaMalloc(stokes values)") ||
      check_cuda(cudaMalloc(&s->scratch, b), "cudaMalloc(stokes scratch)")) {
    cudaFree(s->keys);
    cudaFree(s->values);
    cudaFree(s->scratch);
    delete s;
    return nullptr;
  }
  s->scores.reserve(StokesStore::kCap);
  return s;
}

extern "C" void mojo_stokes_free(void* cache) {
  if (!cache) return;
  StokesStore* s = static_cast<StokesStore*>(cache);
  cudaFree(s->keys);
  cudaFree(s->values);
  cudaFree(s->scratch);
  delete s;
}

extern "C" void mojo_stokes_append(void* cache, int token_id, const float* key, const float* value, float score) {
  (void)token_id;   // unused by the reference too
  if (!cache || !key || !value) return;
  StokesStore* s = static_cast<StokesStore*>(cache);
  const size_t row = (size_t)s->hd * sizeof(float);
  if (check_cuda(cudaMemcpy(s->keys + (size_t)s->n * s->hd, key, row, cudaMemcpyHostToDevice), "stokes key") ||
      check_cuda(cudaMemcpy(s->values + (size_t)s->n * s->hd, value, row, cudaMemcpyHostToDevice), "stokes value"))
    return;
  s->scores.push_back(score);
  s->n += 1;
  if (s->n <= StokesStore::kKeep) return;
  // first minimum (Iterator::min_by keeps the first of equal minima); the
  // reference panics on a NaN score, here the eviction is skipped with an error
  int mi = 0;
  for (int i = 0; i < s->n; ++i) {
    if (s->scores[i] != s->scores[i]) {
      fail(NYION_ERR_INVALID, "mojo_stokes_append: NaN score at %d", i);
      return;
    }
    if (s->scores[i] < s->scores[mi]) mi = i;
  }
  const size_t tail = (size_t)(s->n - 1 - mi) * row;
  if (tail) {
    for (float* buf : {s->keys, s->values}) {
      float* src = buf + (size_t)(mi + 1) * s->hd;
      if (check_cuda(cudaMemcpy(s->scratch, src, tail, cudaMemcpyDeviceToDevice), "stokes shift") ||
          check_cuda(cudaMemcpy(buf + (size_t)mi * s->hd, s->scratch, tail, cudaMemcpyDeviceToDevice), "stokes shift"))
        return;
    }
  }
  s->scores.erase(s->scores.begin() + mi);
  s->n -= 1;
}

// Device view of a Stokes store: K and V rows [n][head_dim] in HBM, ready for
// the decode entry points (e.g. gpu_attention_device with kv_stride = n).
extern "C" int32_t nyion_attn_stokes_view(void* cache, const float** keys, const float** values, int32_t* n,
                                          int32_t* head_dim) {
  if (!cache || !keys || !values || !n) return fail(NYION_ERR_INVALID, "stokes_view: null pointer");
  StokesStore* s = static_cast<StokesStore*>(cache);
  *keys = s->keys;
  *values = s->values;
  *n = s->n;
  if (head_dim) *head_dim = s->hd;
  return NYION_OK;
}
