// Greedy token selection over the logits of a decode step (agentserve/engine/
// sampling.py:46-58 at temperature <= 1e-6): per row, upcast to fp32, replace NaN by
// 0, +inf by 1e4 and -inf by -1e4, and return the index of the first maximum.
//
// One pass over the logits in HBM: CTA (chunk of 4096 columns, row) reduces its chunk
// to a 64-bit key (order-preserving bits of the value << 32 | ~index, so the largest
// key is the largest value at the smallest index), folds it into the row's key with
// atomicMax, and the last CTA of the row (arrival counter) writes the index and
// resets the key and the counter, so the workspace is zero between calls.
#include "common.cuh"
#include "host_util.h"

namespace asb {
namespace {

constexpr int kChunk = 4096;
constexpr int kThreads = 256;

__device__ __forceinline__ float sanitize(float v) {
  if (v != v) return 0.f;                 // NaN
  if (v == INFINITY) return 1e4f;
  if (v == -INFINITY) return -1e4f;
  if (v == 0.f) return 0.f;               // -0 ties with +0, as in a float comparison
  return v;
}

__device__ __forceinline__ unsigned long long make_key(float v, int idx) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // total order
  return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - uint32_t(idx));
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
greedy_argmax_kernel(int64_t* __restrict__ out, const T* __restrict__ logits, int64_t row_stride,
                     int V, unsigned long long* __restrict__ keys, int* __restrict__ counters) {
  const int row = blockIdx.y;
  const int c0 = blockIdx.x * kChunk;
  const int c1 = min(c0 + kChunk, V);
  const T* x = logits + int64_t(row) * row_stride;
  unsigned long long best = 0;
  for (int c = c0 + threadIdx.x; c < c1; c += kThreads) {
    const unsigned long long k = make_key(sanitize(Elem<T>::to_f32(x[c])), c);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  __shared__ unsigned long long warp_best[kThreads / 32];
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_best[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kThreads / 32; ++w) best = warp_best[w] > best ? warp_best[w] : best;
    atomicMax(keys + row, best);
    __threadfence();
    is_last = atomicAdd(counters + row, 1) == int(gridDim.x) - 1;
  }
  __syncthreads();
  if (is_last && threadIdx.x == 0) {
    __threadfence();
    const unsigned long long k = atomicExch(keys + row, 0ull);  // read and reset
    out[row] = int64_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
    counters[row] = 0;
  }
}

}  // namespace
}  // namespace asb

using namespace asb;

extern "C" size_t as_greedy_workspace_size(int32_t num_rows) {
  if (num_rows <= 0) return 0;
  return (size_t(num_rows) * sizeof(unsigned long long) + 255) / 256 * 256 +
         (size_t(num_rows) * sizeof(int) + 255) / 256 * 256;
}

extern "C" int as_greedy_argmax(int64_t* out, const void* logits, int64_t row_stride,
                                int32_t num_rows, int32_t vocab, int32_t dtype, void* workspace,
                                size_t workspace_bytes, as_stream_t stream) {
  if (!dtype_size(dtype)) return fail(AS_ERR_INVALID_ARG, "as_greedy_argmax: unknown dtype");
  if (num_rows < 0 || vocab <= 0 || row_stride < vocab)
    return fail(AS_ERR_INVALID_ARG, "as_greedy_argmax: bad sizes");
  if (num_rows == 0) return AS_OK;
  if (num_rows > 65535) return fail(AS_ERR_INVALID_ARG, "as_greedy_argmax: too many rows");
  if (!out || !logits || !workspace)
    return fail(AS_ERR_INVALID_ARG, "as_greedy_argmax: null pointer");
  if (workspace_bytes < as_greedy_workspace_size(num_rows))
    return fail(AS_ERR_WORKSPACE, "as_greedy_argmax: workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(AS_ERR_INVALID_ARG, "as_greedy_argmax: workspace not 256-byte aligned");
  auto* keys = static_cast<unsigned long long*>(workspace);
  auto* counters = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) +
                                          (size_t(num_rows) * 8 + 255) / 256 * 256);
  const dim3 grid((vocab + kChunk - 1) / kChunk, num_rows);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case AS_DTYPE_F32:
      greedy_argmax_kernel<float><<<grid, kThreads, 0, s>>>(
          out, static_cast<const float*>(logits), row_stride, vocab, keys, counters);
      break;
    case AS_DTYPE_F16:
      greedy_argmax_kernel<__half><<<grid, kThreads, 0, s>>>(
          out, static_cast<const __half*>(logits), row_stride, vocab, keys, counters);
      break;
    default:
      greedy_argmax_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(
          out, static_cast<const __nv_bfloat16*>(logits), row_stride, vocab, keys, counters);
  }
  return check_launch("as_greedy_argmax");
}
