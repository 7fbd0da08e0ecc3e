// host.cu — status, device bookkeeping, workspace and tensor-map helpers.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "host.h"

namespace nyion {

static thread_local char g_msg[512] = "";

int32_t fail(int32_t status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

int32_t check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return NYION_OK;
  return fail(NYION_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static std::mutex g_dev_mu;
static std::vector<DeviceInfo> g_devs;

int32_t device_info(DeviceInfo** out) {
  int dev = -1;
  int32_t st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if ((int)g_devs.size() <= dev) g_devs.resize(dev + 1, DeviceInfo{-1, 0, nullptr});
  DeviceInfo& d = g_devs[dev];
  if (d.device < 0) {
    int sms = 0;
    st = check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
                    "cudaDeviceGetAttribute(SM count)");
    if (st) return st;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10)
      return fail(NYION_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                  dev, major, minor);
    int32_t* w = nullptr;
    st = check_cuda(cudaMalloc(&w, 256), "cudaMalloc(error word)");
    if (st) return st;
    st = check_cuda(cudaMemset(w, 0, 256), "cudaMemset(error word)");
    if (st) return st;
    d.device = dev;
    d.num_sms = sms;
    d.err_word = w;
  }
  *out = &d;
  return NYION_OK;
}

int32_t* device_error_word_if_ready() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (dev < 0 || (int)g_devs.size() <= dev || g_devs[dev].device < 0) return nullptr;
  return g_devs[dev].err_word;
}

static std::mutex g_kernel_mu;
static std::map<std::pair<const void*, int>, int> g_kernel_occ;   // (kernel, device) -> blocks per SM

int32_t kernel_setup(const void* func, size_t smem, int threads, int* occ) {
  int dev = -1;
  int32_t st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  std::lock_guard<std::mutex> lk(g_kernel_mu);
  const auto key = std::make_pair(func, dev);
  auto it = g_kernel_occ.find(key);
  if (it == g_kernel_occ.end()) {
    if (smem > 48 * 1024) {
      st = check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                      "cudaFuncSetAttribute(max dynamic shared memory)");
      if (st) return st;
    }
    int n = 0;
    st = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, threads, smem), "occupancy query");
    if (st) return st;
    it = g_kernel_occ.emplace(key, n > 0 ? n : 1).first;
  }
  if (occ) *occ = it->second;
  return NYION_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int32_t encode_rows_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                         const void* base, uint64_t row_elems, uint64_t rows, uint32_t box_x,
                         uint32_t box_y, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(NYION_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16)
    return fail(NYION_ERR_INVALID, "tensor base %p is not 16-byte aligned", base);
  if (rows == 0 || rows > (1ull << 32))
    return fail(NYION_ERR_INVALID, "tensor row count %llu out of range", (unsigned long long)rows);
  cuuint64_t dims[2] = {row_elems, rows};
  cuuint64_t strides[1] = {row_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_x, box_y};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NYION_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NYION_OK;
}

int32_t encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                    const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                    CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(NYION_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16)
    return fail(NYION_ERR_INVALID, "tensor base %p is not 16-byte aligned", base);
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
    if (dims[i] == 0 || dims[i] > (1ull << 32))
      return fail(NYION_ERR_INVALID, "tensor dim %d extent %llu out of range", i,
                  (unsigned long long)dims[i]);
  }
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NYION_ERR_CUDA, "cuTensorMapEncodeTiled(rank %d) failed (%d)", rank, (int)r);
  return NYION_OK;
}

struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  size_t clean = 0;   // leading bytes known to be zero (the last call's counters)
};
static std::vector<Workspace> g_ws;   // [device * kWsKinds + kind]

int32_t internal_workspace(size_t bytes, void** ptr, WsKind kind, size_t zero_prefix, cudaStream_t stream) {
  int dev = -1;
  int32_t st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  const size_t slot = (size_t)dev * kWsKinds + kind;
  if (g_ws.size() <= slot) g_ws.resize(slot + 1);
  Workspace& w = g_ws[slot];
  if (zero_prefix > bytes) bytes = zero_prefix;
  if (w.bytes < bytes) {
    if (w.ptr) {
      cudaDeviceSynchronize();
      cudaFree(w.ptr);
      w.ptr = nullptr;
      w.bytes = 0;
    }
    st = check_cuda(cudaMalloc(&w.ptr, bytes), "cudaMalloc(workspace)");
    if (st) return st;
    st = check_cuda(cudaMemset(w.ptr, 0, bytes), "cudaMemset(workspace)");
    if (st) return st;
    w.bytes = bytes;
    w.clean = bytes;
  }
  if (zero_prefix > w.clean) {
    st = check_cuda(cudaMemsetAsync(w.ptr, 0, zero_prefix, stream), "clear workspace counters");
    if (st) return st;
  }
  w.clean = zero_prefix;
  *ptr = w.ptr;
  return NYION_OK;
}

}  // namespace nyion

using namespace nyion;

extern "C" int32_t nyion_attn_version(void) { return NYION_ATTN_VERSION; }

extern "C" const char* nyion_attn_last_error(void) { return g_msg; }

// Reads and clears the error words of the current device: the one the
// workspace-taking entry points share and the allocation-free decode's own.
// Only words that already exist are read, so a process that has used nothing
// but the allocation-free entry point allocates nothing here either.
extern "C" int32_t nyion_attn_device_error(void* stream, int32_t* bits) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* words[2] = {device_error_word_if_ready(), noalloc_error_word_if_ready()};
  int32_t vals[2] = {0, 0};
  int32_t st = NYION_OK;
  for (int i = 0; i < 2; ++i) {
    if (!words[i]) continue;
    st = check_cuda(cudaMemcpyAsync(&vals[i], words[i], sizeof(int32_t), cudaMemcpyDeviceToHost, s),
                    "read error word");
    if (st) return st;
  }
  st = check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  if (st) return st;
  for (int i = 0; i < 2; ++i) {
    if (!vals[i]) continue;
    st = check_cuda(cudaMemsetAsync(words[i], 0, sizeof(int32_t), s), "clear error word");
    if (st) return st;
  }
  if (vals[0] || vals[1]) cudaStreamSynchronize(s);
  const int32_t h = vals[0] | vals[1];
  if (bits) *bits = h;
  if (h)
    return fail(NYION_ERR_DEVICE, "device error word 0x%x (%s%s%s)", h,
                (h & NYION_DEVERR_PAGE_RANGE) ? "page id out of range " : "",
                (h & NYION_DEVERR_WAIT_TIMEOUT) ? "wait timeout " : "",
                (h & NYION_DEVERR_SHAPE) ? "shape " : "");
  return NYION_OK;
}

extern "C" int32_t nyion_attn_workspace_reset(void* workspace, size_t bytes, void* stream) {
  if (!workspace || !bytes) return fail(NYION_ERR_INVALID, "workspace_reset: null workspace");
  return check_cuda(cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)),
                    "cudaMemsetAsync(workspace)");
}
