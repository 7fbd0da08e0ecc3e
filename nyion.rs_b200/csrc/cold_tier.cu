// cold_tier.cu — the reference's cold-tier page format moved in and out of
// the 16-token 4-bit page pools.
//
// PagedKVCache evicts a page to its NVMe file as one slot
// (swamp-engine/src/cache.rs:251-276, 440-483, 485-529):
//   slot = [K q4 page][V q4 page], each q4 page = [layer][kv head][bs slots]
//          [ceil(head_dim/32) x 20 B] (cache.rs:681-747), bs = 32 / 128 / 1024
//          for zones 0 / 1 / 2, written at file offset slot * 2 * q4_bytes(zone).
// Here one such slot (in HBM, or in mapped pinned host memory the kernel
// reads over the bus) is scattered into per-layer page pools
// [page][n_kv][K|V][16][40] (bs / 16 pool pages per layer, page ids given per
// layer), and gathered back the same way for eviction.  Every pointer is
// checked with cudaPointerGetAttributes before the launch, so the kernel only
// dereferences memory this device can reach.  One thread moves one 40-byte
// row as five 8-byte words; consecutive threads take consecutive rows of the
// slot, so the slot side is read (or written) contiguously.
#include "common.cuh"
#include "host.h"

namespace nyion {
namespace cold {

constexpr int HD = 64;
constexpr int ROW = 40;       // 2 blocks x 20 bytes
constexpr int PAGE = 16;
constexpr int THREADS = 256;
constexpr int MAX_LAYERS = 128;

struct Pools {
  uint8_t* p[MAX_LAYERS];
};

template <bool TO_POOL>
__global__ void __launch_bounds__(THREADS) move_kernel(const uint8_t* __restrict__ slot_in,
                                                       uint8_t* __restrict__ slot_out,
                                                       const __grid_constant__ Pools pools,
                                                       const int32_t* __restrict__ page_ids, int bs,
                                                       int n_layers, int n_kv, int64_t n_pool_pages,
                                                       int32_t* err) {
  const int64_t rows_per_kv = (int64_t)n_layers * n_kv * bs;        // rows in one q4 page (K or V)
  const int64_t i = (int64_t)blockIdx.x * THREADS + threadIdx.x;
  if (i >= 2 * rows_per_kv) return;
  const int kv = (int)(i / rows_per_kv);
  const int64_t r = i % rows_per_kv;                                  // (layer, kv head, slot)
  const int t = (int)(r % bs);
  const int kvh = (int)((r / bs) % n_kv);
  const int layer = (int)(r / ((int64_t)bs * n_kv));
  const int32_t page = page_ids[(int64_t)layer * (bs / PAGE) + t / PAGE];
  if (page < 0 || page >= n_pool_pages) {
    record_error(err, kErrPageRange);
    return;
  }
  uint8_t* prow = pools.p[layer] + (((int64_t)page * n_kv + kvh) * 2 + kv) * PAGE * ROW + (int64_t)(t % PAGE) * ROW;
  if (TO_POOL) {
    const uint2* s = reinterpret_cast<const uint2*>(slot_in + i * ROW);
    uint2* d = reinterpret_cast<uint2*>(prow);
#pragma unroll
    for (int w = 0; w < ROW / 8; ++w) d[w] = s[w];
  } else {
    const uint2* s = reinterpret_cast<const uint2*>(prow);
    uint2* d = reinterpret_cast<uint2*>(slot_out + i * ROW);
#pragma unroll
    for (int w = 0; w < ROW / 8; ++w) d[w] = s[w];
  }
}

// Device address of `ptr` when the GPU can dereference it (device or managed
// memory, or pinned host memory mapped into the device address space).
int32_t device_view(const void* ptr, const void** out, const char* what, const char* who) {
  cudaPointerAttributes a{};
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(NYION_ERR_INVALID, "%s: %s is not memory CUDA knows", who, what);
  }
  int cur = -1;
  cudaGetDevice(&cur);
  if (a.type == cudaMemoryTypeManaged || (a.type == cudaMemoryTypeDevice && a.device == cur)) {
    *out = ptr;
    return NYION_OK;
  }
  if (a.type == cudaMemoryTypeHost && a.devicePointer) {
    *out = a.devicePointer;
    return NYION_OK;
  }
  return fail(NYION_ERR_INVALID, "%s: %s must be memory of this device or mapped pinned host memory", who, what);
}

int32_t prepare(const void* slot, uint8_t* const* layer_pools, const int32_t* page_ids, int32_t block_slots,
                int32_t n_layers, int32_t n_kv, int32_t head_dim, int64_t n_pool_pages, const char* who,
                const void** slot_dev, Pools* pools) {
  if (!slot || !layer_pools || !page_ids) return fail(NYION_ERR_INVALID, "%s: null pointer argument", who);
  if (head_dim != HD) return fail(NYION_ERR_UNSUPPORTED, "%s: this build takes head_dim 64", who);
  if (block_slots != 32 && block_slots != 128 && block_slots != 1024)
    return fail(NYION_ERR_INVALID, "%s: block_slots must be 32, 128 or 1024 (zones 0, 1, 2)", who);
  if (n_layers <= 0 || n_layers > MAX_LAYERS || n_kv <= 0 || n_pool_pages <= 0)
    return fail(NYION_ERR_INVALID, "%s: bad sizes (n_layers in [1, %d])", who, MAX_LAYERS);
  int32_t st = device_view(slot, slot_dev, "slot", who);
  if (st) return st;
  if (reinterpret_cast<uintptr_t>(*slot_dev) & 7) return fail(NYION_ERR_INVALID, "%s: slot must be 8-byte aligned", who);
  const void* ids = nullptr;
  st = device_view(page_ids, &ids, "page_ids", who);
  if (st) return st;
  if (ids != page_ids) return fail(NYION_ERR_INVALID, "%s: page_ids must be device memory", who);
  for (int l = 0; l < n_layers; ++l) {
    const void* pv = nullptr;
    st = device_view(layer_pools[l], &pv, "a layer pool", who);
    if (st) return st;
    if (pv != layer_pools[l] || (reinterpret_cast<uintptr_t>(pv) & 7))
      return fail(NYION_ERR_INVALID, "%s: layer pools must be 8-byte aligned device memory", who);
    pools->p[l] = layer_pools[l];
  }
  return NYION_OK;
}

}  // namespace cold
}  // namespace nyion

using namespace nyion;
using namespace nyion::cold;

extern "C" size_t nyion_attn_cold_q4_page_bytes(int32_t block_slots, int32_t n_layers, int32_t n_kv_heads,
                                                int32_t head_dim) {
  if (block_slots <= 0 || n_layers <= 0 || n_kv_heads <= 0 || head_dim <= 0) return 0;
  return (size_t)n_layers * n_kv_heads * block_slots * ((head_dim + 31) / 32) * 20;
}

extern "C" int64_t nyion_attn_cold_slot_offset(int64_t slot, int32_t block_slots, int32_t n_layers,
                                               int32_t n_kv_heads, int32_t head_dim) {
  return slot * 2 * (int64_t)nyion_attn_cold_q4_page_bytes(block_slots, n_layers, n_kv_heads, head_dim);
}

extern "C" int32_t nyion_attn_cold_to_pool(const uint8_t* slot, int32_t block_slots, int32_t n_layers,
                                           int32_t n_kv_heads, int32_t head_dim, uint8_t* const* layer_pools,
                                           const int32_t* page_ids, int64_t n_pool_pages, void* stream) {
  const void* sd = nullptr;
  Pools pools{};
  int32_t st = prepare(slot, layer_pools, page_ids, block_slots, n_layers, n_kv_heads, head_dim, n_pool_pages,
                       "cold_to_pool", &sd, &pools);
  if (st) return st;
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st) return st;
  const int64_t rows = 2ll * n_layers * n_kv_heads * block_slots;
  move_kernel<true><<<(unsigned)((rows + THREADS - 1) / THREADS), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(sd), nullptr, pools, page_ids, block_slots, n_layers, n_kv_heads, n_pool_pages,
      dev->err_word);
  return check_cuda(cudaGetLastError(), "cold_to_pool launch");
}

extern "C" int32_t nyion_attn_pool_to_cold(uint8_t* const* layer_pools, const int32_t* page_ids,
                                           int32_t block_slots, int32_t n_layers, int32_t n_kv_heads,
                                           int32_t head_dim, int64_t n_pool_pages, uint8_t* slot, void* stream) {
  const void* sd = nullptr;
  Pools pools{};
  int32_t st = prepare(slot, layer_pools, page_ids, block_slots, n_layers, n_kv_heads, head_dim, n_pool_pages,
                       "pool_to_cold", &sd, &pools);
  if (st) return st;
  DeviceInfo* dev = nullptr;
  st = device_info(&dev);
  if (st) return st;
  const int64_t rows = 2ll * n_layers * n_kv_heads * block_slots;
  move_kernel<false><<<(unsigned)((rows + THREADS - 1) / THREADS), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      nullptr, static_cast<uint8_t*>(const_cast<void*>(sd)), pools, page_ids, block_slots, n_layers, n_kv_heads,
      n_pool_pages, dev->err_word);
  return check_cuda(cudaGetLastError(), "pool_to_cold launch");
}
