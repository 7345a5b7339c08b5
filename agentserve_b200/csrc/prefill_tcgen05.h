// Tensor-core (tcgen05 + TMEM) varlen prefill attention (prefill_pair.cu): internal
// interface.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace asb {

// True when the tcgen05 kernel handles this shape/dtype/alignment.
bool prefill_tc_supported(int dtype, int H, int Kh, int D, const void* q, int64_t q_stride,
                          const void* k_cache, const void* v_cache, const void* out);

int prefill_tc_launch(void* out, const void* q, int64_t q_stride, const void* k_cache,
                      const void* v_cache, const int32_t* bt, int64_t bt_stride,
                      const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int R,
                      int max_seqlen_q, int total_q, int H, int Kh, int D, int num_blocks,
                      int max_blocks, float scale, int dtype, int n_split, void* workspace,
                      cudaStream_t stream);

// head_dim 64 or 128: two query tiles per CTA sharing each K/V tile, P in tensor
// memory.  n_split > 1 splits each pair's KV range over n_split CTAs (partials in
// `workspace`, prefill_pair_workspace_size bytes) and merges them in a second kernel.
int prefill_pair_launch(void* out, const void* q, int64_t q_stride, const void* k_cache,
                        const void* v_cache, const int32_t* bt, int64_t bt_stride,
                        const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int R,
                        int max_seqlen_q, int total_q, int H, int Kh, int D, int num_blocks,
                        int max_blocks, float scale, int dtype, int n_split, void* workspace,
                        cudaStream_t stream);
// Split count: `requested` if > 0 (capped at 16), else chosen from the grid shape.
int prefill_pair_splits(int R, int max_seqlen_q, int H, int Kh, int max_blocks, int requested);
size_t prefill_pair_workspace_size(int R, int max_seqlen_q, int H, int Kh, int D, int n_split);

}  // namespace asb
