// Tensor-core (tcgen05 + TMEM) varlen prefill attention: internal interface.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace asb {

// True when the tcgen05 kernel handles this shape/dtype/alignment.
bool prefill_tc_supported(int dtype, int H, int Kh, int D, const void* q, int64_t q_stride,
                          const void* k_cache, const void* v_cache, const void* out);

int prefill_tc_launch(void* out, const void* q, int64_t q_stride, const void* k_cache,
                      const void* v_cache, const int32_t* bt, int64_t bt_stride,
                      const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int R,
                      int max_seqlen_q, int total_q, int H, int Kh, int D, int num_blocks,
                      int max_blocks, float scale, int dtype, cudaStream_t stream);

// head_dim 64: two query tiles per CTA sharing each K/V tile, P in tensor memory.
int prefill_pair_launch(void* out, const void* q, int64_t q_stride, const void* k_cache,
                        const void* v_cache, const int32_t* bt, int64_t bt_stride,
                        const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int R,
                        int max_seqlen_q, int total_q, int H, int Kh, int num_blocks,
                        int max_blocks, float scale, int dtype, cudaStream_t stream);

}  // namespace asb
