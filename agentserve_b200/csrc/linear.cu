// (6) Decode-step projections for a small batch: Y[M, N] = X[M, K] W[N, K]^T
// (nn.Linear without bias: q/k/v, o_proj, gate/up, down at agentserve/model/llama.py:
// 123-126, 203-211, 430-471), bf16/fp16 in, fp32 accumulation, M <= 256.
//
// At decode batch sizes the product is a stream over the weights (2 bytes per weight,
// 2*M FLOPs per weight): it has to read W at HBM bandwidth, which needs every SM busy
// even when N/128 is only 16-24 tiles.  So the grid is (N tile of 128 weight rows) x
// (K split), and each CTA computes D[128 x Mpad] = W_tile X^T on the tensor cores
// (tcgen05.mma kind::f16, M=128, N=Mpad, both operands K-major 128B-swizzled in shared
// memory, accumulator in TMEM) over its K range (M <= 256):
//   warp 0     TMA producer: W box 128 rows x 64 K and X box Mpad rows x 64 K per stage
//              (X rows >= M read as zeros), 4-stage ring;
//   warp 1     MMA issuer (one thread), commits each stage back to the producer;
//   warps 2-5  epilogue, one TMEM lane (= weight row n) per thread: with one split it
//              stores Y directly; with several it stores its fp32 partial tile (which
//              stays in L2), and the last CTA of the N tile (arrival counter) sums the
//              splits in a fixed order into Y and resets the counter, so results are
//              deterministic and the counters are zero between calls.
// Every wait is bounded (status bit 4).
#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "tcgen05.cuh"

namespace asb {

constexpr int kLinTileN = 128;
constexpr int kLinMaxSplits = 16;
// K splits: enough CTAs for two per SM (at least 2 K steps each, at most 16 splits)
int linear_max_splits(int N) {
  const int n_tiles = (N + kLinTileN - 1) / kLinTileN;
  const int want = (2 * sm_count() + n_tiles - 1) / n_tiles;
  return want < 1 ? 1 : (want > kLinMaxSplits ? kLinMaxSplits : want);
}
// [ceil(N/128)] int arrival counters, rounded to 256 bytes, then fp32 partial sums
// [splits, N, M4] (M4 = M rounded up to 4: one weight row's batch column is 16-byte
// vectors)
inline int round4(int m) { return (m + 3) / 4 * 4; }
size_t linear_counter_bytes(int N) {
  return (size_t((N + kLinTileN - 1) / kLinTileN) * sizeof(int) + 255) / 256 * 256;
}
size_t linear_workspace_bytes(int M, int N) {
  return linear_counter_bytes(N) +
         size_t(linear_max_splits(N)) * N * round4(M) * sizeof(float);
}

namespace {

constexpr int kTileN = kLinTileN;
constexpr int kTileK = 64;
#ifndef AS_LINEAR_STAGES
#define AS_LINEAR_STAGES 4
#endif
constexpr int kStages = AS_LINEAR_STAGES;
constexpr int kMaxM = 256;
constexpr int kWBytes = kTileN * 128;  // 128 rows x 64 16-bit elements

struct LinBars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  int is_last;
  int abort;
};

__device__ __forceinline__ bool aborted_flag(volatile int* f) { return *f != 0; }

__host__ __device__ inline int pad_m(int M) { return (M + 15) / 16 * 16; }
__host__ __device__ inline int stage_bytes(int Mpad) { return kWBytes + Mpad * 128; }
__host__ __device__ inline int smem_bytes(int Mpad) { return kStages * stage_bytes(Mpad) + 256; }
__host__ __device__ inline uint32_t tmem_cols(int Mpad) {
  return Mpad <= 32 ? 32u : (Mpad <= 64 ? 64u : (Mpad <= 128 ? 128u : 256u));
}

template <typename T>
__global__ void __launch_bounds__(192)
linear_small_m_kernel(const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_x, T* __restrict__ y,
                      int64_t y_stride, float* __restrict__ acc, int* __restrict__ counters,
                      int M, int Mpad, int N, int k_steps, int k_splits, int* status) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  const int n_tile = blockIdx.x;
  const int split = blockIdx.y;
  const int s0 = int(int64_t(split) * k_steps / k_splits);
  const int s1 = int(int64_t(split + 1) * k_steps / k_splits);
  const int nsteps = s1 - s0;
  const int sbytes = stage_bytes(Mpad);

  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) flag_status(status, kStatusWaitTimeout);
    return;
  }
  LinBars* bars = reinterpret_cast<LinBars*>(smem + kStages * sbytes);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ncols = tmem_cols(Mpad);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    bars->abort = 0;
    bars->is_last = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&bars->tmem_base, ncols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_x);
      const uint64_t pol_w = l2_policy_evict_first();  // each weight is read once
      const uint64_t pol_x = l2_policy_evict_last();   // X is re-read by every CTA
      for (int i = 0; i < nsteps; ++i) {
        const int st = i % kStages;
        if (i >= kStages && !mbar_wait(&bars->empty[st], ((i / kStages) + 1) & 1, status)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* base = smem + st * sbytes;
        mbar_arrive_expect_tx(&bars->full[st], uint32_t(sbytes));
        const int k = (s0 + i) * kTileK;
        tma_load_2d(base, &tmap_w, &bars->full[st], k, n_tile * kTileN, pol_w);
        tma_load_2d(base + kWBytes, &tmap_x, &bars->full[st], k, 0, pol_x);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(kBF16, 128, Mpad, false, false);
      bool ok = true;
      for (int i = 0; i < nsteps && ok; ++i) {
        const int st = i % kStages;
        if (aborted_flag(abort_flag) || !mbar_wait(&bars->full[st], (i / kStages) & 1, status)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t w = smem_u32(smem + st * sbytes);
        const uint32_t x = w + kWBytes;
#pragma unroll
        for (int kk = 0; kk < kTileK / 16; ++kk)
          tc::mma_f16(tmem, tc::sdesc_sw128(w + kk * 32, 16, 1024),
                      tc::sdesc_sw128(x + kk * 32, 16, 1024), idesc, (i > 0 || kk > 0) ? 1u : 0u);
        tc::commit(&bars->empty[st]);
      }
      if (!ok) *abort_flag = 1;
      // also the drain: acc_full fires once every MMA issued above has completed
      tc::commit(&bars->acc_full);
      mbar_wait(&bars->acc_full, 0, status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int n = n_tile * kTileN + row;
    const uint32_t trow = tmem + (uint32_t(quad * 32) << 16);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full, 0, status)) &&
                    !aborted_flag(abort_flag);
    const int M4 = (M + 3) / 4 * 4;
    if (ok) {
      tc::fence_after_sync();
      for (int c = 0; c < Mpad; c += 16) {
        uint32_t v[16];
        tc::ld_32x32b_x16(trow + c, v);
        tc::wait_ld();
        if (n < N) {
          if (k_splits == 1) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < M) y[int64_t(c + e) * y_stride + n] = Elem<T>::from_f32(__uint_as_float(v[e]));
          } else {  // this split's partial column, kept in L2 for the finishing CTA
            float* dst = acc + (int64_t(split) * N + n) * M4 + c;
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              if (c + e < M4)
                __stcg(reinterpret_cast<float4*>(dst + e),
                       make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]),
                                   __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3])));
          }
        }
      }
    }
    if (k_splits > 1) {
      // Last-arriving CTA of this N tile finishes it (no spin: whoever arrives last
      // sees the count).  Every CTA counts, so the counter always returns to zero.
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        const int old = atomicAdd(counters + n_tile, 1);
        bars->is_last = (old == k_splits - 1);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (bars->is_last) {
        __threadfence();
        if (n < N) {
          for (int c = 0; c < M4; c += 16) {  // 16 batch rows at a time, vector loads
            float sum[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) sum[e] = 0.f;
            for (int sp = 0; sp < k_splits; ++sp) {  // fixed order: deterministic result
              const float* src = acc + (int64_t(sp) * N + n) * M4 + c;
#pragma unroll
              for (int e = 0; e < 16; e += 4) {
                if (c + e < M4) {
                  const float4 p = __ldcg(reinterpret_cast<const float4*>(src + e));
                  sum[e] += p.x;
                  sum[e + 1] += p.y;
                  sum[e + 2] += p.z;
                  sum[e + 3] += p.w;
                }
              }
            }
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < M) y[int64_t(c + e) * y_stride + n] = Elem<T>::from_f32(sum[e]);
          }
        }
        if (threadIdx.x == 64) counters[n_tile] = 0;
      }
    }
    tc::fence_before_sync();
  }

  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, ncols);
  }
}

template <typename T>
CUtensorMapDataType tmap_dtype() {
  return std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

int choose_splits(int N, int k_steps) {
  const int s = linear_max_splits(N);
  const int cap = k_steps / 2 > 0 ? k_steps / 2 : 1;  // at least 2 K steps per CTA
  return s > cap ? cap : s;
}

template <typename T>
int launch_linear(void* y, int64_t y_stride, const void* x, int64_t x_stride, const void* w,
                  int M, int N, int K, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream) {
  const int Mpad = pad_m(M);
  const int n_tiles = (N + kTileN - 1) / kTileN;
  const int k_steps = (K + kTileK - 1) / kTileK;
  int k_splits = choose_splits(N, k_steps);
  const size_t need = linear_workspace_bytes(M, N);
  if (k_splits > 1 && (!workspace || workspace_bytes < need)) k_splits = 1;
  CUtensorMap mw, mx;
  const uint64_t es = sizeof(T);
  {
    const uint64_t dims[2] = {uint64_t(K), uint64_t(N)};
    const uint64_t strides[1] = {uint64_t(K) * es};
    const uint32_t box[2] = {uint32_t(kTileK), uint32_t(kTileN)};
    int rc = encode_tensor_map(&mw, tmap_dtype<T>(), 2, const_cast<void*>(w), dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {uint64_t(K), uint64_t(M)};
    const uint64_t strides[1] = {uint64_t(x_stride) * es};
    const uint32_t box[2] = {uint32_t(kTileK), uint32_t(Mpad)};
    int rc = encode_tensor_map(&mx, tmap_dtype<T>(), 2, const_cast<void*>(x), dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  int* counters = static_cast<int*>(workspace);
  float* acc = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                        linear_counter_bytes(N));
  auto kern = linear_small_m_kernel<T>;
  const int smem = smem_bytes(Mpad);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  kern<<<dim3(n_tiles, k_splits), 192, smem, stream>>>(
      mw, mx, static_cast<T*>(y), y_stride, k_splits > 1 ? acc : nullptr,
      k_splits > 1 ? counters : nullptr, M, Mpad, N, k_steps, k_splits, device_status_ptr());
  return check_launch("as_linear_small_m");
}

}  // namespace
}  // namespace asb

using namespace asb;

extern "C" size_t as_linear_small_m_workspace_size(int32_t M, int32_t N) {
  if (M <= 0 || M > kMaxM || N <= 0) return 0;
  return linear_workspace_bytes(M, N);
}

extern "C" int as_linear_small_m(void* y, int64_t y_stride, const void* x, int64_t x_stride,
                                 const void* w, int32_t M, int32_t N, int32_t K, int32_t dtype,
                                 void* workspace, size_t workspace_bytes, as_stream_t stream) {
  if (dtype != AS_DTYPE_BF16 && dtype != AS_DTYPE_F16)
    return fail(AS_ERR_UNSUPPORTED, "as_linear_small_m: bf16 or fp16 only");
  if (M < 0 || N <= 0 || K <= 0) return fail(AS_ERR_INVALID_ARG, "as_linear_small_m: bad sizes");
  if (M == 0) return AS_OK;
  if (M > kMaxM) return fail(AS_ERR_UNSUPPORTED, "as_linear_small_m: M > %d", kMaxM);
  if (!y || !x || !w) return fail(AS_ERR_INVALID_ARG, "as_linear_small_m: null pointer");
  if (y_stride < N || x_stride < K)
    return fail(AS_ERR_INVALID_ARG, "as_linear_small_m: row stride shorter than the row");
  // TMA: 16-byte aligned bases and row strides
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15 ||
      (x_stride * 2) % 16 || (int64_t(K) * 2) % 16)
    return fail(AS_ERR_INVALID_ARG, "as_linear_small_m: x, w and their rows must be 16-byte aligned");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(AS_ERR_INVALID_ARG, "as_linear_small_m: workspace not 256-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == AS_DTYPE_BF16)
    return launch_linear<__nv_bfloat16>(y, y_stride, x, x_stride, w, M, N, K, workspace,
                                        workspace_bytes, s);
  return launch_linear<__half>(y, y_stride, x, x_stride, w, M, N, K, workspace, workspace_bytes,
                               s);
}
