// C-ABI plumbing: error strings, the per-device status word, tensor-map encoding.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace asb {

namespace {
thread_local char g_last_error[512] = {0};

// One status word per device; kernels get its address as a parameter.
__device__ int g_device_status;

constexpr int kMaxDevices = 64;
// Per-device caches filled once under g_mu and read without it afterwards: atomics
// (acquire / release) so a reader never sees a half-published value.
std::atomic<int*> g_status_ptr[kMaxDevices];
std::atomic<int> g_sm_count[kMaxDevices];
std::mutex g_mu;

constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;
std::atomic<uint64_t> g_wait_limit_ns{kDefaultWaitLimitNs};
std::atomic<int> g_starve_next{0};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AS_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return AS_OK;
}

int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  int* p = g_status_ptr[dev].load(std::memory_order_acquire);
  if (p) return p;
  std::lock_guard<std::mutex> lock(g_mu);
  p = g_status_ptr[dev].load(std::memory_order_relaxed);
  if (!p) {
    void* a = nullptr;
    if (cudaGetSymbolAddress(&a, g_device_status) != cudaSuccess) return nullptr;
    p = static_cast<int*>(a);
    g_status_ptr[dev].store(p, std::memory_order_release);
  }
  return p;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (!n) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

bool take_starve_flag(int kernel_bit) {
  return (g_starve_next.fetch_and(~kernel_bit) & kernel_bit) != 0;
}

int dtype_size(int dtype) {
  switch (dtype) {
    case AS_DTYPE_F32: return 4;
    case AS_DTYPE_F16: return 2;
    case AS_DTYPE_BF16: return 2;
    default: return 0;
  }
}

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  if (!g_encode) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(AS_ERR_CUDA, "cannot resolve cuTensorMapEncodeTiled");
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5], es[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, dtype, rank, base, d, s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return AS_OK;
}

}  // namespace asb

extern "C" int as_version(void) { return 100; }

extern "C" const char* as_last_error(void) { return asb::g_last_error; }

extern "C" int as_device_status(int clear, int* out_bits, as_stream_t stream) {
  int* p = asb::device_status_ptr();
  if (!p) return asb::fail(AS_ERR_CUDA, "as_device_status: no device status word");
  int bits = 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&bits, p, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return asb::fail(AS_ERR_CUDA, "as_device_status: read failed");
  if (clear && cudaMemsetAsync(p, 0, sizeof(int), s) != cudaSuccess)
    return asb::fail(AS_ERR_CUDA, "as_device_status: clear failed");
  if (cudaStreamSynchronize(s) != cudaSuccess)
    return asb::fail(AS_ERR_CUDA, "as_device_status: sync failed");
  if (out_bits) *out_bits = bits;
  return AS_OK;
}

extern "C" uint64_t as_set_wait_limit_ns(uint64_t limit_ns) {
  if (limit_ns == 0) limit_ns = asb::kDefaultWaitLimitNs;
  return asb::g_wait_limit_ns.exchange(limit_ns);
}

extern "C" int as_debug_starve_next_launch(int kernels) {
  if (kernels & ~(AS_KERNEL_DECODE_ATTENTION | AS_KERNEL_PREFILL_ATTENTION))
    return asb::fail(AS_ERR_INVALID_ARG, "as_debug_starve_next_launch: unknown kernel bits %d",
                     kernels);
  asb::g_starve_next.store(kernels);
  return AS_OK;
}
