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
//              stores Y directly; with several it copies its fp32 partial tile into
//              its own shared memory (over the drained stage ring).
// The K splits of one N tile form a thread-block cluster (2, 4 or 8 CTAs): after a
// cluster barrier, member r sums rows [r*128/splits, (r+1)*128/splits) of every
// member's partial through distributed shared memory, in member order (deterministic),
// and a second cluster barrier keeps the partials alive until all reads are done.  No
// global workspace, no atomics.  Every mbarrier wait is bounded (status bit 4); every
// thread of every member reaches both cluster barriers on every path.
#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "tcgen05.cuh"

namespace asb {
namespace {

constexpr int kTileN = 128;
constexpr int kTileK = 64;
constexpr int kStages = 4;
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr int kMaxM = 256;
constexpr int kWBytes = kTileN * 128;  // 128 rows x 64 16-bit elements
// split partial row pitch in floats: 128 weight rows + 16, so the 8 threads of one
// float4 load phase that span two batch rows hit different banks
constexpr int kPartStride = kTileN + 16;

struct LinBars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool aborted_flag(volatile int* f) { return *f != 0; }

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__host__ __device__ inline int pad_m(int M) { return (M + 15) / 16 * 16; }
__host__ __device__ inline int stage_bytes(int Mpad) { return kWBytes + Mpad * 128; }
__host__ __device__ inline int smem_bytes(int Mpad) { return kStages * stage_bytes(Mpad) + 256; }
// the partial [M][kPartStride] fp32 reuses the stage ring
static_assert(kMaxM * kPartStride * 4 <= kStages * (kWBytes + kMaxM * 128),
              "stage ring too small for the split partial");
__host__ __device__ inline uint32_t tmem_cols(int Mpad) {
  return Mpad <= 32 ? 32u : (Mpad <= 64 ? 64u : (Mpad <= 128 ? 128u : 256u));
}

template <typename T>
__global__ void __launch_bounds__(192)
linear_small_m_kernel(const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_x, T* __restrict__ y,
                      int64_t y_stride, int M, int Mpad, int N, int k_steps, int k_splits,
                      int* status) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  pdl_trigger();  // the next kernel may start its prologue; it waits for this one
  const int n_tile = blockIdx.x;
  const int split = blockIdx.y;
  const int s0 = int(int64_t(split) * k_steps / k_splits);
  const int s1 = int(int64_t(split + 1) * k_steps / k_splits);
  const int nsteps = s1 - s0;
  const int sbytes = stage_bytes(Mpad);

  extern __shared__ __align__(1024) uint8_t smem[];
  // (uniform over the cluster: every member has the same shared memory layout)
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
      // The weights do not depend on the previous kernel: the first ring's worth of W
      // boxes is requested before the programmatic-launch wait, X (its output) after.
      const int early = nsteps < kStages ? nsteps : kStages;
      for (int i = 0; i < early; ++i) {
        mbar_arrive_expect_tx(&bars->full[i], uint32_t(sbytes));
        tma_load_2d(smem + i * sbytes, &tmap_w, &bars->full[i], (s0 + i) * kTileK,
                    n_tile * kTileN, pol_w);
      }
      pdl_wait();
      for (int i = 0; i < early; ++i)
        tma_load_2d(smem + i * sbytes + kWBytes, &tmap_x, &bars->full[i], (s0 + i) * kTileK, 0,
                    pol_x);
      for (int i = early; i < nsteps; ++i) {
        const int st = i % kStages;
        if (!mbar_wait(&bars->empty[st], ((i / kStages) + 1) & 1, status)) {
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
    const int row = quad * 32 + lane;  // TMEM lane = weight row of the tile
    const int n = n_tile * kTileN + row;
    const uint32_t trow = tmem + (uint32_t(quad * 32) << 16);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full, 0, status)) &&
                    !aborted_flag(abort_flag);
    if (ok) {
      tc::fence_after_sync();
      // split partial: [m][kPartStride] fp32 over the stage ring (every MMA reading it
      // has completed); lanes write consecutive weight rows, conflict-free
      float* part = reinterpret_cast<float*>(smem);
      for (int c = 0; c < Mpad; c += 16) {
        uint32_t v[16];
        tc::ld_32x32b_x16(trow + c, v);
        tc::wait_ld();
        if (k_splits == 1) {
          if (n < N) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e < M) y[int64_t(c + e) * y_stride + n] = Elem<T>::from_f32(__uint_as_float(v[e]));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c + e < M) part[(c + e) * kPartStride + row] = __uint_as_float(v[e]);
        }
      }
    }
    tc::fence_before_sync();
  }

  __syncthreads();  // TMEM reads done
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, ncols);
  }
  if (k_splits > 1) {
    // every member's partial is complete and visible after this barrier
    cluster_sync_all();
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    const int rows = kTileN / k_splits;  // weight rows this member finishes
    const int q = rows / 4;              // float4 vectors per batch row
    const int r0 = int(rank) * rows;
    const uint32_t base = smem_u32(smem);
    for (int it = threadIdx.x; it < M * q; it += blockDim.x) {
      const int m = it / q;
      const int nl = r0 + (it - m * q) * 4;
      const uint32_t off = base + uint32_t(m * kPartStride + nl) * 4u;
      // all remote loads in flight before the first add
      float4 p[kMaxSplits];
#pragma unroll
      for (int sp = 0; sp < kMaxSplits; ++sp)
        if (sp < k_splits) p[sp] = ld_dsmem_f4(mapa_shared(off, uint32_t(sp)));
      float4 acc = p[0];
#pragma unroll
      for (int sp = 1; sp < kMaxSplits; ++sp) {  // member order: deterministic result
        if (sp < k_splits) {
          acc.x += p[sp].x;
          acc.y += p[sp].y;
          acc.z += p[sp].z;
          acc.w += p[sp].w;
        }
      }
      const int n0 = n_tile * kTileN + nl;
      T* dst = y + int64_t(m) * y_stride + n0;
      if (n0 + 3 < N && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
        uint2 pk;
        pk.x = pack2<T>(acc.x, acc.y);
        pk.y = pack2<T>(acc.z, acc.w);
        *reinterpret_cast<uint2*>(dst) = pk;
      } else {
        const float a[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (n0 + e < N) dst[e] = Elem<T>::from_f32(a[e]);
      }
    }
    // peers may still be reading this member's partial
    cluster_sync_all();
  }
}

template <typename T>
CUtensorMapDataType tmap_dtype() {
  return std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// K splits: a power of two <= 8 (so 128 divides evenly among the members), enough
// CTAs for two per SM, at least 2 K steps per member.
int choose_splits(int N, int k_steps) {
  const int n_tiles = (N + kTileN - 1) / kTileN;
  const int want = (2 * sm_count() + n_tiles - 1) / n_tiles;
  int s = 1;
  while (s * 2 <= kMaxSplits && s * 2 <= want && s * 2 <= k_steps / 2) s *= 2;
  return s;
}

template <typename T>
int launch_linear(void* y, int64_t y_stride, const void* x, int64_t x_stride, const void* w,
                  int M, int N, int K, cudaStream_t stream) {
  const int Mpad = pad_m(M);
  const int n_tiles = (N + kTileN - 1) / kTileN;
  const int k_steps = (K + kTileK - 1) / kTileK;
  const int k_splits = choose_splits(N, k_steps);
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
  auto kern = linear_small_m_kernel<T>;
  const int smem = smem_bytes(Mpad);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_tiles, k_splits);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = k_splits;  // the K splits of one N tile
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = AS_PDL;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, kern, mw, mx, static_cast<T*>(y), y_stride, M, Mpad, N, k_steps,
                     k_splits, device_status_ptr());
  return check_launch("as_linear_small_m");
}

}  // namespace
}  // namespace asb

using namespace asb;

extern "C" int as_linear_small_m(void* y, int64_t y_stride, const void* x, int64_t x_stride,
                                 const void* w, int32_t M, int32_t N, int32_t K, int32_t dtype,
                                 as_stream_t stream) {
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
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == AS_DTYPE_BF16)
    return launch_linear<__nv_bfloat16>(y, y_stride, x, x_stride, w, M, N, K, s);
  return launch_linear<__half>(y, y_stride, x, x_stride, w, M, N, K, s);
}
