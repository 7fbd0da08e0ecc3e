// arena.cu — the HBM arena behind the reference's DeviceAllocator
// (swamp-tensors/src/hma.rs:215-221: allocate_device, allocate_unified, free,
// upload, download), which HeterogeneousMemoryAllocator holds as its device
// side and from which the KV page pools, page tables and per-step buffers of
// the attention path are carved (hma.rs:223-265 routes DeviceLocal and
// UnifiedMapped requests to it).
//
// The reference's implementation (swamp-gpu/src/lib.rs:101-150) allocates one
// Vulkan buffer per request.  Here one cudaMalloc reservation of HBM is made
// up front and carved: allocations are 256-byte aligned (every TMA and bulk
// copy of the kernels needs 16), placed best-fit from a free list kept by
// offset, and freed blocks coalesce with their neighbours, so serving loops
// allocate and free KV pages without cudaMalloc / cudaFree (and without the
// device-wide synchronisation cudaFree implies).  UnifiedMapped requests are
// managed-memory allocations (host- and device-addressable) outside the
// reservation.  Every call is thread-safe (one mutex per arena).
#include <stdint.h>
#include <string.h>

#include <map>
#include <mutex>
#include <unordered_map>

#include "host.h"

namespace nyion {
namespace arena {

constexpr size_t kAlign = 256;

struct Block {
  size_t offset = 0;   // within the reservation (device-local blocks)
  size_t size = 0;     // bytes requested
  size_t span = 0;     // bytes taken from the reservation (aligned)
  void* ptr = nullptr; // device pointer (device-local) or managed pointer (unified)
  bool unified = false;
};

struct Arena {
  int device = -1;
  uint8_t* base = nullptr;
  size_t capacity = 0;
  size_t used = 0;                        // bytes of the reservation in live blocks
  std::mutex mu;
  std::map<size_t, size_t> free_;         // offset -> span of each free range
  std::unordered_map<uint64_t, Block> live;
  uint64_t next = 1;
};

size_t round_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

Arena* get(void* a) { return static_cast<Arena*>(a); }

// The arena's device is made current for the CUDA calls of one entry point.
struct DeviceScope {
  int prev = -1;
  bool changed = false;
  explicit DeviceScope(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) changed = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceScope() {
    if (changed) cudaSetDevice(prev);
  }
};

int32_t copy(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return NYION_OK;
  if (!stream) return check_cuda(cudaMemcpy(dst, src, bytes, cudaMemcpyDefault), "arena copy");
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
                    "arena copy");
}

}  // namespace arena
}  // namespace nyion

using namespace nyion;
using namespace nyion::arena;

extern "C" int32_t nyion_attn_arena_create(size_t capacity, void** out) {
  if (!out || capacity == 0) return fail(NYION_ERR_INVALID, "arena_create: bad arguments");
  *out = nullptr;
  Arena* a = new Arena();
  int32_t st = check_cuda(cudaGetDevice(&a->device), "cudaGetDevice");
  if (!st) {
    a->capacity = round_up(capacity);
    void* p = nullptr;
    st = check_cuda(cudaMalloc(&p, a->capacity), "cudaMalloc(arena)");
    a->base = static_cast<uint8_t*>(p);
  }
  if (st) {
    delete a;
    return st;
  }
  a->free_[0] = a->capacity;
  *out = a;
  return NYION_OK;
}

extern "C" int32_t nyion_attn_arena_destroy(void* arena) {
  Arena* a = get(arena);
  if (!a) return fail(NYION_ERR_INVALID, "arena_destroy: null arena");
  int32_t st = NYION_OK;
  {
    DeviceScope ds(a->device);
    std::lock_guard<std::mutex> lk(a->mu);
    for (auto& kv : a->live)
      if (kv.second.unified) cudaFree(kv.second.ptr);
    st = check_cuda(cudaFree(a->base), "cudaFree(arena)");
  }
  delete a;
  return st;
}

extern "C" int32_t nyion_attn_arena_allocate_device(void* arena, size_t size, uint64_t* handle, void** dev_ptr) {
  Arena* a = get(arena);
  if (!a || !handle || !dev_ptr || size == 0) return fail(NYION_ERR_INVALID, "arena_allocate_device: bad arguments");
  const size_t span = round_up(size);
  std::lock_guard<std::mutex> lk(a->mu);
  auto best = a->free_.end();
  for (auto it = a->free_.begin(); it != a->free_.end(); ++it)   // best fit, lowest offset on ties
    if (it->second >= span && (best == a->free_.end() || it->second < best->second)) best = it;
  if (best == a->free_.end())
    return fail(NYION_ERR_WORKSPACE, "arena_allocate_device: no free range of %zu bytes (capacity %zu, in use %zu)",
                span, a->capacity, a->used);
  const size_t off = best->first, rest = best->second - span;
  a->free_.erase(best);
  if (rest) a->free_[off + span] = rest;
  Block blk;
  blk.offset = off;
  blk.size = size;
  blk.span = span;
  blk.ptr = a->base + off;
  const uint64_t h = a->next++;
  a->live[h] = blk;
  a->used += span;
  *handle = h;
  *dev_ptr = blk.ptr;
  return NYION_OK;
}

extern "C" int32_t nyion_attn_arena_allocate_unified(void* arena, size_t size, uint64_t* handle, void** ptr) {
  Arena* a = get(arena);
  if (!a || !handle || !ptr || size == 0) return fail(NYION_ERR_INVALID, "arena_allocate_unified: bad arguments");
  DeviceScope ds(a->device);
  void* p = nullptr;
  int32_t st = check_cuda(cudaMallocManaged(&p, size), "cudaMallocManaged(arena unified)");
  if (st) return st;
  std::lock_guard<std::mutex> lk(a->mu);
  Block blk;
  blk.size = size;
  blk.ptr = p;
  blk.unified = true;
  const uint64_t h = a->next++;
  a->live[h] = blk;
  *handle = h;
  *ptr = p;
  return NYION_OK;
}

extern "C" int32_t nyion_attn_arena_free(void* arena, uint64_t handle) {
  Arena* a = get(arena);
  if (!a) return fail(NYION_ERR_INVALID, "arena_free: null arena");
  Block blk;
  {
    std::lock_guard<std::mutex> lk(a->mu);
    auto it = a->live.find(handle);
    if (it == a->live.end()) return fail(NYION_ERR_INVALID, "arena_free: unknown handle %llu", (unsigned long long)handle);
    blk = it->second;
    a->live.erase(it);
    if (!blk.unified) {
      // coalesce with the free neighbours
      size_t off = blk.offset, span = blk.span;
      auto next = a->free_.lower_bound(off);
      if (next != a->free_.end() && next->first == off + span) {
        span += next->second;
        next = a->free_.erase(next);
      }
      if (next != a->free_.begin()) {
        auto prev = std::prev(next);
        if (prev->first + prev->second == off) {
          off = prev->first;
          span += prev->second;
          a->free_.erase(prev);
        }
      }
      a->free_[off] = span;
      a->used -= blk.span;
      return NYION_OK;
    }
  }
  DeviceScope ds(a->device);
  return check_cuda(cudaFree(blk.ptr), "cudaFree(arena unified)");
}

static int32_t find_block(Arena* a, uint64_t handle, Block* out, const char* who) {
  std::lock_guard<std::mutex> lk(a->mu);
  auto it = a->live.find(handle);
  if (it == a->live.end()) return fail(NYION_ERR_INVALID, "%s: unknown handle %llu", who, (unsigned long long)handle);
  *out = it->second;
  return NYION_OK;
}

extern "C" int32_t nyion_attn_arena_upload(void* arena, uint64_t handle, const void* src, size_t bytes,
                                           void* stream) {
  Arena* a = get(arena);
  if (!a || (!src && bytes)) return fail(NYION_ERR_INVALID, "arena_upload: bad arguments");
  Block blk;
  int32_t st = find_block(a, handle, &blk, "arena_upload");
  if (st) return st;
  DeviceScope ds(a->device);
  return copy(blk.ptr, src, bytes < blk.size ? bytes : blk.size, stream);   // min(src, dst), as the reference
}

extern "C" int32_t nyion_attn_arena_download(void* arena, uint64_t handle, void* dst, size_t bytes, void* stream) {
  Arena* a = get(arena);
  if (!a || (!dst && bytes)) return fail(NYION_ERR_INVALID, "arena_download: bad arguments");
  Block blk;
  int32_t st = find_block(a, handle, &blk, "arena_download");
  if (st) return st;
  DeviceScope ds(a->device);
  return copy(dst, blk.ptr, bytes < blk.size ? bytes : blk.size, stream);
}

extern "C" int32_t nyion_attn_arena_info(void* arena, size_t* capacity, size_t* used, size_t* largest_free) {
  Arena* a = get(arena);
  if (!a) return fail(NYION_ERR_INVALID, "arena_info: null arena");
  std::lock_guard<std::mutex> lk(a->mu);
  size_t lf = 0;
  for (auto& kv : a->free_) lf = kv.second > lf ? kv.second : lf;
  if (capacity) *capacity = a->capacity;
  if (used) *used = a->used;
  if (largest_free) *largest_free = lf;
  return NYION_OK;
}
