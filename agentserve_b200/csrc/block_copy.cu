// (5) Block gather / copy for prefix-cache seeding and gather_kv.
//
// Device-to-device, 16-byte vectors, one CTA per (block, plane) pair.  Replaces
// the per-layer clone of the prefix KV on store and its reuse on a hit
// (agentserve/engine/engine.py:274-281, 338-345) and the per-block torch.cat of
// BlockAllocator.gather_kv (agentserve/engine/cache.py:158-189).  Byte copies:
// bit-exact by construction.
#include "common.cuh"
#include "host_util.h"

namespace asb {
namespace {

// grid: (n, num_planes) folded into x; block: 256 threads copying int4 vectors.
__global__ void block_copy_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src,
                                  const int32_t* __restrict__ src_ids,
                                  const int32_t* __restrict__ dst_ids, int32_t n,
                                  int64_t bytes_per_block, int32_t num_planes,
                                  int64_t src_plane_stride, int64_t dst_plane_stride,
                                  int32_t src_num_blocks, int32_t dst_num_blocks, int* status) {
  const int64_t work = int64_t(n) * num_planes;
  for (int64_t w = blockIdx.x; w < work; w += gridDim.x) {
    const int i = int(w % n);
    const int p = int(w / n);
    const int32_t s = src_ids[i];
    const int32_t d = dst_ids ? dst_ids[i] : i;
    if (s < 0 || s >= src_num_blocks || d < 0 || d >= dst_num_blocks) {
      if (threadIdx.x == 0) flag_status(status, kStatusBadBlockId);
      continue;
    }
    const int4* from =
        reinterpret_cast<const int4*>(src + p * src_plane_stride + int64_t(s) * bytes_per_block);
    int4* to = reinterpret_cast<int4*>(dst + p * dst_plane_stride + int64_t(d) * bytes_per_block);
    const int64_t nvec = bytes_per_block >> 4;
    for (int64_t j = threadIdx.x; j < nvec; j += blockDim.x) to[j] = __ldcs(from + j);
  }
}

}  // namespace
}  // namespace asb

using namespace asb;

extern "C" int as_block_copy(void* dst, const void* src, const int32_t* src_ids,
                             const int32_t* dst_ids, int32_t n, int64_t bytes_per_block,
                             int32_t num_planes, int64_t src_plane_stride,
                             int64_t dst_plane_stride, int32_t src_num_blocks,
                             int32_t dst_num_blocks, as_stream_t stream) {
  if (n < 0 || num_planes <= 0 || bytes_per_block <= 0)
    return fail(AS_ERR_INVALID_ARG, "as_block_copy: bad sizes");
  if (n == 0) return AS_OK;
  if (!dst || !src || !src_ids) return fail(AS_ERR_INVALID_ARG, "as_block_copy: null pointer");
  if ((bytes_per_block & 15) || (src_plane_stride & 15) || (dst_plane_stride & 15) ||
      (reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 15))
    return fail(AS_ERR_INVALID_ARG, "as_block_copy: sizes, strides and pointers must be 16-byte aligned");
  int64_t work = int64_t(n) * num_planes;
  const int64_t cap = int64_t(sm_count()) * 8;
  const int grid = int(work < cap ? work : cap);
  block_copy_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src), src_ids, dst_ids, n,
      bytes_per_block, num_planes, src_plane_stride, dst_plane_stride, src_num_blocks,
      dst_num_blocks, device_status_ptr());
  return check_launch("as_block_copy");
}
