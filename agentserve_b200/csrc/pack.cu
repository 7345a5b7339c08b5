// (1) Ragged-batch packing: positions, slot_mapping, seq_lens_k, cu_seqlens_q and a
// packed block table, built on the device from the allocator's device-resident
// block-table rows.  Integer work, bit-exact with the host arithmetic of
// agentserve/engine/engine.py:349-357 and agentserve/engine/cache.py:134-140,152-154.
#include "common.cuh"
#include "host_util.h"

namespace asb {
namespace {

// grid: (ceil(max_blocks / 128), B); block: 128.
__global__ void pack_decode_kernel(const int32_t* __restrict__ bt, int64_t bt_stride,
                                   const int32_t* __restrict__ row_ids,
                                   const int32_t* __restrict__ seq_lens, int32_t B,
                                   int32_t max_blocks, int32_t block_size,
                                   int64_t* __restrict__ positions,
                                   int64_t* __restrict__ slot_mapping,
                                   int32_t* __restrict__ seq_lens_k,
                                   int32_t* __restrict__ cu_seqlens_q,
                                   int32_t* __restrict__ packed_bt, int* status) {
  const int b = blockIdx.y;
  const int64_t row = row_ids ? row_ids[b] : b;
  const int32_t* src = bt + row * bt_stride;
  if (packed_bt) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < max_blocks; j += gridDim.x * blockDim.x)
      packed_bt[int64_t(b) * max_blocks + j] = src[j];
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const int32_t pos = seq_lens[b];
    const int32_t blk = pos / block_size;
    int64_t slot = -1;
    if (pos < 0 || blk >= max_blocks) {
      flag_status(status, kStatusBadLength);
    } else {
      slot = int64_t(src[blk]) * block_size + (pos % block_size);
    }
    positions[b] = pos;
    slot_mapping[b] = slot;
    seq_lens_k[b] = pos + 1;
    cu_seqlens_q[b] = b;
    if (b == B - 1) cu_seqlens_q[B] = B;
  }
}

// grid: (R); block: 256.  CTA r sums num_new[0..r) itself (R is a batch of
// requests, so the O(R^2) sum is a few thousand adds) and then writes its rows.
__global__ void pack_prefill_kernel(const int32_t* __restrict__ bt, int64_t bt_stride,
                                    const int32_t* __restrict__ row_ids,
                                    const int32_t* __restrict__ num_cached,
                                    const int32_t* __restrict__ num_new, int32_t R,
                                    int32_t total_new, int32_t max_blocks, int32_t block_size,
                                    int32_t* __restrict__ cu_seqlens_q,
                                    int64_t* __restrict__ positions,
                                    int64_t* __restrict__ slot_mapping,
                                    int32_t* __restrict__ seq_lens_k,
                                    int32_t* __restrict__ packed_bt, int* status) {
  __shared__ int32_t s_part[32];
  const int r = blockIdx.x;
  int32_t acc = 0;
  for (int i = threadIdx.x; i < r; i += blockDim.x) acc += num_new[i];
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  int32_t start = 0;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) start += s_part[w];

  const int64_t row = row_ids ? row_ids[r] : r;
  const int32_t* src = bt + row * bt_stride;
  const int32_t nc = num_cached[r];
  const int32_t nn = num_new[r];
  if (threadIdx.x == 0) {
    cu_seqlens_q[r] = start;
    if (r == R - 1) cu_seqlens_q[R] = start + nn;
    seq_lens_k[r] = nc + nn;
    if (start + nn > total_new || nc < 0 || nn < 0) flag_status(status, kStatusBadLength);
  }
  if (packed_bt) {
    for (int j = threadIdx.x; j < max_blocks; j += blockDim.x)
      packed_bt[int64_t(r) * max_blocks + j] = src[j];
  }
  for (int i = threadIdx.x; i < nn; i += blockDim.x) {
    const int64_t t = int64_t(start) + i;
    if (t >= total_new) break;
    const int32_t pos = nc + i;
    const int32_t blk = pos / block_size;
    int64_t slot = -1;
    if (blk >= max_blocks) {
      flag_status(status, kStatusBadLength);
    } else {
      slot = int64_t(src[blk]) * block_size + (pos % block_size);
    }
    positions[t] = pos;
    slot_mapping[t] = slot;
  }
}

}  // namespace
}  // namespace asb

using namespace asb;

extern "C" int as_pack_decode(const int32_t* block_tables, int64_t bt_stride,
                              const int32_t* row_ids, const int32_t* seq_lens, int32_t num_seqs,
                              int32_t max_blocks, int32_t block_size, int64_t* positions,
                              int64_t* slot_mapping, int32_t* seq_lens_k, int32_t* cu_seqlens_q,
                              int32_t* packed_bt, as_stream_t stream) {
  if (num_seqs < 0 || max_blocks <= 0 || block_size <= 0 || bt_stride < max_blocks)
    return fail(AS_ERR_INVALID_ARG, "as_pack_decode: bad sizes (B=%d max_blocks=%d bs=%d stride=%lld)",
                num_seqs, max_blocks, block_size, (long long)bt_stride);
  if (num_seqs == 0) return AS_OK;
  if (!block_tables || !seq_lens || !positions || !slot_mapping || !seq_lens_k || !cu_seqlens_q)
    return fail(AS_ERR_INVALID_ARG, "as_pack_decode: null pointer");
  if (num_seqs > 65535) return fail(AS_ERR_INVALID_ARG, "as_pack_decode: too many sequences");
  dim3 grid((max_blocks + 127) / 128, num_seqs);
  pack_decode_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      block_tables, bt_stride, row_ids, seq_lens, num_seqs, max_blocks, block_size, positions,
      slot_mapping, seq_lens_k, cu_seqlens_q, packed_bt, device_status_ptr());
  return check_launch("as_pack_decode");
}

extern "C" int as_pack_prefill(const int32_t* block_tables, int64_t bt_stride,
                               const int32_t* row_ids, const int32_t* num_cached,
                               const int32_t* num_new, int32_t num_seqs, int32_t total_new,
                               int32_t max_blocks, int32_t block_size, int32_t* cu_seqlens_q,
                               int64_t* positions, int64_t* slot_mapping, int32_t* seq_lens_k,
                               int32_t* packed_bt, as_stream_t stream) {
  if (num_seqs < 0 || total_new < 0 || max_blocks <= 0 || block_size <= 0 || bt_stride < max_blocks)
    return fail(AS_ERR_INVALID_ARG, "as_pack_prefill: bad sizes");
  if (num_seqs == 0) return AS_OK;
  if (!block_tables || !num_cached || !num_new || !cu_seqlens_q || !seq_lens_k ||
      (total_new > 0 && (!positions || !slot_mapping)))
    return fail(AS_ERR_INVALID_ARG, "as_pack_prefill: null pointer");
  pack_prefill_kernel<<<num_seqs, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      block_tables, bt_stride, row_ids, num_cached, num_new, num_seqs, total_new, max_blocks,
      block_size, cu_seqlens_q, positions, slot_mapping, seq_lens_k, packed_bt,
      device_status_ptr());
  return check_launch("as_pack_prefill");
}
