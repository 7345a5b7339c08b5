// (4) Varlen prefill attention over cached prefix blocks + new tokens: entry point
// and the CUDA-core kernel used for fp32 and for head dims the tensor-core kernel
// does not cover.  The bf16/fp16 tensor-core kernel (tcgen05 + TMEM) lives in
// prefill_pair.cu.
//
// Semantics follow LlamaAttention.forward with a cached prefix
// (agentserve/model/llama.py:128-186): new token i of a sequence whose first P
// tokens are cached attends to keys 0..P+i; the prefix is unmasked and the new
// tokens are causal (the additive mask of llama.py:171-180).  Keys and values are
// read in place from the paged pool (the new tokens' K/V were written there by
// as_rope_reshape_and_cache), so the prefix is never concatenated or copied.
#include "common.cuh"
#include "host_util.h"
#include "prefill_tcgen05.h"

namespace asb {
namespace {

constexpr int kBlockSize = 16;
constexpr int kGenWarps = 4;

// Sequence r with cu[r] <= t < cu[r+1] (cu is non-decreasing, cu[0] = 0).
__device__ __forceinline__ int find_seq(const int32_t* __restrict__ cu, int R, int t) {
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// grid: (total_q, H); block: 4 warps interleaved over the visible keys.
template <typename T, int EPL>
__global__ void __launch_bounds__(kGenWarps * 32)
prefill_generic_kernel(T* __restrict__ out, const T* __restrict__ q, int64_t q_stride,
                       const T* __restrict__ k_cache, const T* __restrict__ v_cache,
                       const int32_t* __restrict__ bt, int64_t bt_stride,
                       const int32_t* __restrict__ cu, const int32_t* __restrict__ seq_lens_k,
                       int R, int H, int Kh, int D, int num_blocks, int max_blocks, float scale,
                       int* status) {
  const int t = blockIdx.x;
  const int h = blockIdx.y;
  const int g = h / (H / Kh);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int r = find_seq(cu, R, t);
  const int nnew = cu[r + 1] - cu[r];
  const int lk = seq_lens_k[r];
  const int i = t - cu[r];
  int kv_end = lk - nnew + i + 1;  // keys 0 .. P+i
  if (kv_end > max_blocks * kBlockSize) {
    if (threadIdx.x == 0) flag_status(status, kStatusBadLength);
    kv_end = max_blocks * kBlockSize;
  }

  float qv[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const int d = lane + 32 * e;
    qv[e] = d < D ? Elem<T>::to_f32(q[int64_t(t) * q_stride + int64_t(h) * D + d]) : 0.f;
  }
  float m = -INFINITY, l = 0.f, o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) o[e] = 0.f;
  for (int j = warp; j < kv_end; j += kGenWarps) {
    const int blk = bt[int64_t(r) * bt_stride + j / kBlockSize];
    if (blk < 0 || blk >= num_blocks) {
      if (lane == 0) flag_status(status, kStatusBadBlockId);
      continue;
    }
    const int64_t row = (int64_t(blk) * kBlockSize + j % kBlockSize) * Kh + g;
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int d = lane + 32 * e;
      if (d < D) s += qv[e] * Elem<T>::to_f32(k_cache[row * D + d]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    s *= scale;
    const float mn = fmaxf(m, s);
    const float alpha = expf(m - mn);
    const float p = expf(s - mn);
    l = l * alpha + p;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int d = lane + 32 * e;
      const float vv = d < D ? Elem<T>::to_f32(v_cache[row * D + d]) : 0.f;
      o[e] = o[e] * alpha + p * vv;
    }
    m = mn;
  }
  __shared__ float red_m[kGenWarps], red_l[kGenWarps];
  __shared__ float red_o[kGenWarps][256];
  if (lane == 0) {
    red_m[warp] = m;
    red_l[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const int d = lane + 32 * e;
    if (d < D) red_o[warp][d] = o[e];
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < kGenWarps; ++w) M = fmaxf(M, red_m[w]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < kGenWarps; ++w) {
        const float wt = expf(red_m[w] - M);
        L += wt * red_l[w];
        O += wt * red_o[w][d];
      }
    }
    out[(int64_t(t) * H + h) * D + d] = Elem<T>::from_f32(L > 0.f ? O / L : 0.f);
  }
}

template <typename T>
int launch_prefill_generic(void* out, const void* q, int64_t q_stride, const void* k_cache,
                           const void* v_cache, const int32_t* bt, int64_t bt_stride,
                           const int32_t* cu, const int32_t* seq_lens_k, int R, int total_q,
                           int H, int Kh, int D, int num_blocks, int max_blocks, float scale,
                           cudaStream_t stream) {
  dim3 grid(total_q, H);
  T* o = static_cast<T*>(out);
  const T* qq = static_cast<const T*>(q);
  const T* kc = static_cast<const T*>(k_cache);
  const T* vc = static_cast<const T*>(v_cache);
  int* st = device_status_ptr();
#define AS_PREFILL_GENERIC(EPL)                                                               \
  prefill_generic_kernel<T, EPL><<<grid, kGenWarps * 32, 0, stream>>>(                       \
      o, qq, q_stride, kc, vc, bt, bt_stride, cu, seq_lens_k, R, H, Kh, D, num_blocks,         \
      max_blocks, scale, st)
  if (D <= 32) AS_PREFILL_GENERIC(1);
  else if (D <= 64) AS_PREFILL_GENERIC(2);
  else if (D <= 128) AS_PREFILL_GENERIC(4);
  else AS_PREFILL_GENERIC(8);
#undef AS_PREFILL_GENERIC
  return check_launch("as_varlen_prefill_attention");
}

}  // namespace
}  // namespace asb

using namespace asb;

namespace {

// the tensor-core shapes take the query-tile-pair kernel, which can split KV
bool pair_path(int32_t dtype, int32_t H, int32_t Kh, int32_t D, const void* q, int64_t q_stride,
               const void* k_cache, const void* v_cache, const void* out) {
  return (D == 64 || D == 128) &&
         prefill_tc_supported(dtype, H, Kh, D, q, q_stride, k_cache, v_cache, out);
}

int prefill_entry(void* out, const void* q, int64_t q_stride, const void* k_cache,
                  const void* v_cache, const int32_t* block_tables, int64_t bt_stride,
                  const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int32_t num_seqs,
                  int32_t max_seqlen_q, int32_t total_q, int32_t num_heads, int32_t num_kv_heads,
                  int32_t head_dim, int32_t block_size, int32_t num_blocks, int32_t max_blocks,
                  float scale, int32_t dtype, int32_t num_splits, void* workspace,
                  size_t workspace_bytes, as_stream_t stream) {
  if (!dtype_size(dtype)) return fail(AS_ERR_INVALID_ARG, "as_varlen_prefill_attention: unknown dtype");
  if (block_size != kBlockSize)
    return fail(AS_ERR_UNSUPPORTED, "as_varlen_prefill_attention: block_size must be 16");
  if (num_seqs < 0 || total_q < 0 || num_heads <= 0 || num_kv_heads <= 0 ||
      num_heads % num_kv_heads || head_dim <= 0 || head_dim > 256 || num_blocks <= 0 ||
      max_blocks <= 0 || bt_stride < max_blocks || max_seqlen_q < 0 || num_splits < 0)
    return fail(AS_ERR_INVALID_ARG, "as_varlen_prefill_attention: bad sizes");
  if (num_seqs == 0 || total_q == 0) return AS_OK;
  if (!out || !q || !k_cache || !v_cache || !block_tables || !cu_seqlens_q || !seq_lens_k)
    return fail(AS_ERR_INVALID_ARG, "as_varlen_prefill_attention: null pointer");
  if (q_stride < int64_t(num_heads) * head_dim)
    return fail(AS_ERR_INVALID_ARG, "as_varlen_prefill_attention: q_stride < H*D");
  if (num_heads > 65535) return fail(AS_ERR_INVALID_ARG, "as_varlen_prefill_attention: H too large");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  if (prefill_tc_supported(dtype, num_heads, num_kv_heads, head_dim, q, q_stride, k_cache,
                           v_cache, out)) {
    int n_split = 1;
    if (pair_path(dtype, num_heads, num_kv_heads, head_dim, q, q_stride, k_cache, v_cache, out) &&
        num_splits != 1) {
      n_split = prefill_pair_splits(num_seqs, max_seqlen_q, num_heads, num_kv_heads, max_blocks,
                                    num_splits);
      const size_t need = prefill_pair_workspace_size(num_seqs, max_seqlen_q, num_heads,
                                                      num_kv_heads, head_dim, n_split);
      if (need > 0 && (!workspace || workspace_bytes < need)) {
        if (num_splits > 1)
          return fail(AS_ERR_WORKSPACE, "as_varlen_prefill_attention: workspace of %zu bytes < %zu",
                      workspace_bytes, need);
        n_split = 1;  // automatic split: fall back to one CTA per pair
      }
      if (n_split > 1 && (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(AS_ERR_INVALID_ARG, "as_varlen_prefill_attention: workspace not 256-byte aligned");
    }
    return prefill_tc_launch(out, q, q_stride, k_cache, v_cache, block_tables, bt_stride,
                             cu_seqlens_q, seq_lens_k, num_seqs, max_seqlen_q, total_q, num_heads,
                             num_kv_heads, head_dim, num_blocks, max_blocks, scale, dtype, n_split,
                             workspace, s);
  }
  switch (dtype) {
    case AS_DTYPE_F32:
      return launch_prefill_generic<float>(out, q, q_stride, k_cache, v_cache, block_tables,
                                           bt_stride, cu_seqlens_q, seq_lens_k, num_seqs, total_q,
                                           num_heads, num_kv_heads, head_dim, num_blocks,
                                           max_blocks, scale, s);
    case AS_DTYPE_F16:
      return launch_prefill_generic<__half>(out, q, q_stride, k_cache, v_cache, block_tables,
                                            bt_stride, cu_seqlens_q, seq_lens_k, num_seqs,
                                            total_q, num_heads, num_kv_heads, head_dim,
                                            num_blocks, max_blocks, scale, s);
    default:
      return launch_prefill_generic<__nv_bfloat16>(out, q, q_stride, k_cache, v_cache,
                                                   block_tables, bt_stride, cu_seqlens_q,
                                                   seq_lens_k, num_seqs, total_q, num_heads,
                                                   num_kv_heads, head_dim, num_blocks, max_blocks,
                                                   scale, s);
  }
}

}  // namespace

extern "C" int as_varlen_prefill_attention(void* out, const void* q, int64_t q_stride,
                                           const void* k_cache, const void* v_cache,
                                           const int32_t* block_tables, int64_t bt_stride,
                                           const int32_t* cu_seqlens_q, const int32_t* seq_lens_k,
                                           int32_t num_seqs, int32_t max_seqlen_q,
                                           int32_t total_q, int32_t num_heads,
                                           int32_t num_kv_heads, int32_t head_dim,
                                           int32_t block_size, int32_t num_blocks,
                                           int32_t max_blocks, float scale, int32_t dtype,
                                           as_stream_t stream) {
  return prefill_entry(out, q, q_stride, k_cache, v_cache, block_tables, bt_stride, cu_seqlens_q,
                       seq_lens_k, num_seqs, max_seqlen_q, total_q, num_heads, num_kv_heads,
                       head_dim, block_size, num_blocks, max_blocks, scale, dtype, 1, nullptr, 0,
                       stream);
}

extern "C" int as_varlen_prefill_attention_ws(
    void* out, const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
    const int32_t* block_tables, int64_t bt_stride, const int32_t* cu_seqlens_q,
    const int32_t* seq_lens_k, int32_t num_seqs, int32_t max_seqlen_q, int32_t total_q,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int32_t num_blocks, int32_t max_blocks, float scale, int32_t dtype, int32_t num_splits,
    void* workspace, size_t workspace_bytes, as_stream_t stream) {
  return prefill_entry(out, q, q_stride, k_cache, v_cache, block_tables, bt_stride, cu_seqlens_q,
                       seq_lens_k, num_seqs, max_seqlen_q, total_q, num_heads, num_kv_heads,
                       head_dim, block_size, num_blocks, max_blocks, scale, dtype, num_splits,
                       workspace, workspace_bytes, stream);
}

extern "C" size_t as_varlen_prefill_workspace_size(int32_t num_seqs, int32_t max_seqlen_q,
                                                   int32_t num_heads, int32_t num_kv_heads,
                                                   int32_t head_dim, int32_t max_blocks,
                                                   int32_t num_splits, int32_t dtype) {
  if (num_seqs <= 0 || max_seqlen_q <= 0 || num_heads <= 0 || num_kv_heads <= 0 ||
      num_heads % num_kv_heads || max_blocks <= 0 || num_splits == 1 || num_splits < 0)
    return 0;
  const int group = num_heads / num_kv_heads;
  if ((head_dim != 64 && head_dim != 128) || (dtype != AS_DTYPE_BF16 && dtype != AS_DTYPE_F16) ||
      group > 128 || 128 % group)
    return 0;
  const int n = prefill_pair_splits(num_seqs, max_seqlen_q, num_heads, num_kv_heads, max_blocks,
                                    num_splits);
  return prefill_pair_workspace_size(num_seqs, max_seqlen_q, num_heads, num_kv_heads, head_dim,
                                     n);
}
