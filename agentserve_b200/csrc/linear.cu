// (6) Decode-step projections for a small batch: Y[M, N] = X[M, K] W[N, K]^T
// (nn.Linear without bias: q/k/v, o_proj, gate/up, down at agentserve/model/llama.py:
// 123-126, 203-211, 430-471), bf16/fp16 in, fp32 accumulation, M <= 256; and the
// gate/up projection with SwiGLU applied in the epilogue (llama.py:207-211).
//
// At decode batch sizes the product is a stream over the weights (2 bytes per weight,
// 2*M FLOPs per weight): it has to read W at HBM bandwidth, which needs every SM busy
// even when N/128 is only 16-24 tiles.  So the grid is (N tile of 128 weight rows) x
// (K split), and each CTA computes D[128 x Mpad] = W_tile X^T on the tensor cores
// (tcgen05.mma kind::f16, M=128, N=Mpad, both operands K-major 128B-swizzled in shared
// memory, accumulator in TMEM) over its K range (M <= 256):
//   warp 0     TMA producer: W box 128 rows x 64 K (with SwiGLU two 64-row boxes: the
//              tile's gate rows and the matching up rows) and X box Mpad rows x 64 K per
//              stage (X rows >= M read as zeros), 4-stage ring; launched
//              programmatically, it requests the first ring's W boxes before waiting
//              for the kernel ahead (which produces X);
//   warp 1     MMA issuer (one thread), commits each stage back to the producer;
//   warps 2-5  epilogue, one TMEM lane (= weight row n) per thread: with one split it
//              stores Y (or silu(gate) * up) directly; with several it writes its fp32
//              partial tile into its own shared memory (over the drained stage ring).
// The K splits of one N tile form a thread-block cluster (2, 4 or 8 CTAs); member r
// finishes rows [r*128/splits, (r+1)*128/splits) of the tile (with SwiGLU: that share
// of the gate rows and the matching up rows), summing every member's partial of them
// in member order (deterministic).  The partials are exchanged either by push — each
// member bulk-copies slice r of its partial into member r's shared memory, completing
// on r's mbarrier, after one cluster barrier that guarantees the receivers' rings are
// drained — or, when the partial and the receive slots do not fit the ring together,
// by pull: after a cluster barrier every member reads the slices over distributed
// shared memory, and a second barrier keeps them alive until all reads are done.  No
// global workspace, no atomics.  Every mbarrier wait is bounded (status bit 4); every
// thread of every member reaches each cluster barrier on every path.
#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "tcgen05.cuh"

namespace asb {
namespace {

constexpr int kTileN = 128;
constexpr int kTileK = 64;
constexpr int kMaxStages = 8;
// K steps in flight per CTA.  Fewer stages mean less shared memory per CTA, so a
// programmatically launched projection can become resident beside the tail of the
// kernel before it (and the next one beside it) and stream its weights earlier:
// measured in the decode step, 4 stages at 64 rows beat 6 and 8 by a wide margin.
#ifndef AS_LINEAR_STAGES
#define AS_LINEAR_STAGES 4
#endif
constexpr int kMaxSplits = 8;  // portable cluster size
#ifndef AS_LINEAR_PUSH
#define AS_LINEAR_PUSH 1  // 0: every K split reduced by the pull path
#endif
constexpr int kMaxM = 256;
constexpr int kWBytes = kTileN * 128;  // 128 rows x 64 16-bit elements
// split partial row pitch in floats: 128 weight rows + 16, so the 8 threads of one
// float4 load phase that span two batch rows hit different banks
constexpr int kPartStride = kTileN + 16;

struct LinBars {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full;
  uint64_t recv;  // the other K-split members' slices of this member's rows have landed
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ bool aborted_flag(volatile int* f) { return *f != 0; }

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// bulk copy of this CTA's shared memory into a cluster peer's, completing on the
// peer's mbarrier (both addresses shared::cluster, 16-byte aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, uint32_t src, uint32_t bytes,
                                                  uint32_t peer_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst),
      "r"(src), "r"(bytes), "r"(peer_bar)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_reads() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// K-split exchange by push: member r finishes the tile rows of "slice" r (rp = 128 / splits
// rows; with SwiGLU rp / 2 gate rows and the matching up rows).  Every member writes its
// fp32 partial slice-major ([slice][m][pos], slices slice_floats apart), sends slice r to
// member r with one bulk copy and sums the slices it receives in member order.
__device__ __forceinline__ void slice_of(int row, int rp, int swiglu, int& slice, int& pos) {
  if (swiglu) {
    const int h = rp / 2, g = row & 63;
    slice = g / h;
    pos = (row >> 6) * h + g % h;
  } else {
    slice = row / rp;
    pos = row % rp;
  }
}
__host__ __device__ inline int slice_floats(int M, int k_splits) {
  return M * (kTileN / k_splits) + 16;  // 16-byte multiple; +16 spreads the banks
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
// the stage ring also holds the split partial [M][kPartStride] fp32 and the SwiGLU up
// values [64][Mpad + 1] fp32 once the MMAs are done: at least that many stages
__host__ __device__ inline int num_stages(int Mpad) {
  const int need_part = Mpad * kPartStride * 4;
  const int need_up = 64 * (Mpad + 1) * 4;
  const int need = need_part > need_up ? need_part : need_up;
  const int fit = (227 * 1024 - 256) / stage_bytes(Mpad);  // >= 4: the assert below
  int st = (need + stage_bytes(Mpad) - 1) / stage_bytes(Mpad);
  if (st < 2) st = 2;
  if (st < AS_LINEAR_STAGES) st = AS_LINEAR_STAGES;
  if (st > fit) st = fit;
  return st > kMaxStages ? kMaxStages : st;
}
__host__ __device__ inline int smem_bytes(int Mpad, int stages) {
  return stages * stage_bytes(Mpad) + 256;
}
static_assert(AS_LINEAR_STAGES >= 1 && AS_LINEAR_STAGES <= kMaxStages, "stage count");
// at the largest batch 4 stages fit in 227 KB and hold the 256-row partial
static_assert(4 * (kWBytes + kMaxM * 128) + 256 <= 227 * 1024, "ring");
static_assert(kMaxM * kPartStride * 4 <= 4 * (kWBytes + kMaxM * 128), "partial");
__host__ __device__ inline uint32_t tmem_cols(int Mpad) {
  return Mpad <= 32 ? 32u : (Mpad <= 64 ? 64u : (Mpad <= 128 ? 128u : 256u));
}

template <typename T>
__global__ void __launch_bounds__(192)
linear_small_m_kernel(const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_x, T* __restrict__ y,
                      int64_t y_stride, int M, int Mpad, int N, int k_steps, int k_splits,
                      int stages, int swiglu, int push, int* status) {
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
  LinBars* bars = reinterpret_cast<LinBars*>(smem + stages * sbytes);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ncols = tmem_cols(Mpad);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    if (push) {
      mbar_init(&bars->recv, 1);
      mbar_arrive_expect_tx(&bars->recv,
                            uint32_t((k_splits - 1) * M * (kTileN / k_splits) * 4));
    }
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
      // W box of the tile: 128 consecutive weight rows, or with SwiGLU 64 gate rows of
      // [gate; up] and the matching 64 up rows (64-row boxes, the second 8 KB further:
      // whole 1024-byte swizzle atoms, so the MMA sees one 128-row operand)
      auto load_w = [&](uint8_t* dst, uint64_t* bar, int k) {
        if (swiglu) {
          tma_load_2d(dst, &tmap_w, bar, k, n_tile * 64, pol_w);
          tma_load_2d(dst + kWBytes / 2, &tmap_w, bar, k, N / 2 + n_tile * 64, pol_w);
        } else {
          tma_load_2d(dst, &tmap_w, bar, k, n_tile * kTileN, pol_w);
        }
      };
      const int early = nsteps < stages ? nsteps : stages;
      for (int i = 0; i < early; ++i) {
        mbar_arrive_expect_tx(&bars->full[i], uint32_t(sbytes));
        load_w(smem + i * sbytes, &bars->full[i], (s0 + i) * kTileK);
      }
      pdl_wait();
      for (int i = 0; i < early; ++i)
        tma_load_2d(smem + i * sbytes + kWBytes, &tmap_x, &bars->full[i], (s0 + i) * kTileK, 0,
                    pol_x);
      for (int i = early; i < nsteps; ++i) {
        const int st = i % stages;
        if (!mbar_wait(&bars->empty[st], ((i / stages) + 1) & 1, status)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* base = smem + st * sbytes;
        mbar_arrive_expect_tx(&bars->full[st], uint32_t(sbytes));
        const int k = (s0 + i) * kTileK;
        load_w(base, &bars->full[st], k);
        tma_load_2d(base + kWBytes, &tmap_x, &bars->full[st], k, 0, pol_x);
      }
    }
    __syncwarp();
    if (push) cluster_arrive_release();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(kBF16, 128, Mpad, false, false);
      bool ok = true;
      for (int i = 0; i < nsteps && ok; ++i) {
        const int st = i % stages;
        if (aborted_flag(abort_flag) || !mbar_wait(&bars->full[st], (i / stages) & 1, status)) {
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
    // (with push: this CTA's MMAs are done, so its stage ring may receive the peers'
    // slices once every member has arrived)
    if (push) cluster_arrive_release();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // TMEM lane = weight row of the tile
    const int n = n_tile * kTileN + row;
    const uint32_t trow = tmem + (uint32_t(quad * 32) << 16);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full, 0, status)) &&
                    !aborted_flag(abort_flag);
    if (push) cluster_arrive_release();
    if (swiglu && k_splits == 1) {
      // Gate/up with SwiGLU in the epilogue: tile rows [0, 64) are gate rows and
      // [64, 128) the matching up rows (the two W boxes of each stage).  The up
      // threads park their values, rounded to T as a separate projection's output
      // would be, in shared memory over the drained stage ring; after a barrier of the
      // four epilogue warps each gate thread forms to_T(to_T(silu(g)) * u)
      // (llama.py:207-211, as_silu_mul's rounding) for output column 64 t + row.
      // (With K splits the partials take the path below and the cluster reduction
      // applies the same formula.)
      float* up = reinterpret_cast<float*>(smem);
      const int us = Mpad + 1;
      if (ok && row >= 64) {
        tc::fence_after_sync();
        for (int c = 0; c < Mpad; c += 16) {
          uint32_t v[16];
          tc::ld_32x32b_x16(trow + c, v);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e)
            up[(row - 64) * us + c + e] = Elem<T>::to_f32(Elem<T>::from_f32(__uint_as_float(v[e])));
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // every epilogue thread, ok or not
      const int j = n_tile * 64 + row;
      if (ok && row < 64 && j < N / 2) {
        tc::fence_after_sync();
        for (int c = 0; c < Mpad; c += 16) {
          uint32_t v[16];
          tc::ld_32x32b_x16(trow + c, v);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (c + e < M) {
              const float g = Elem<T>::to_f32(Elem<T>::from_f32(__uint_as_float(v[e])));
              const float sg = Elem<T>::to_f32(Elem<T>::from_f32(g / (1.0f + expf(-g))));
              y[int64_t(c + e) * y_stride + j] = Elem<T>::from_f32(sg * up[row * us + c + e]);
            }
          }
        }
      }
    } else if (ok) {
      tc::fence_after_sync();
      // split partial over the stage ring (every MMA reading it has completed): pull
      // layout [m][kPartStride], or push layout [slice][m][pos]; lanes write
      // consecutive weight rows
      float* part = reinterpret_cast<float*>(smem);
      int sl = 0, pos = 0;
      if (push) slice_of(row, kTileN / k_splits, swiglu, sl, pos);
      float* pdst = part + sl * slice_floats(M, k_splits) + pos;
      const int prow = kTileN / k_splits;
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
        } else if (push) {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c + e < M) pdst[(c + e) * prow] = __uint_as_float(v[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c + e < M) part[(c + e) * kPartStride + row] = __uint_as_float(v[e]);
        }
      }
      if (push) fence_proxy_async_smem();  // the partial is read by bulk copies
    }
    tc::fence_before_sync();
  }

  __syncthreads();  // TMEM reads done
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, ncols);
  }
  if (push) {
    const uint32_t rank = cluster_rank();
    const int rp = kTileN / k_splits;
    const int sf = slice_floats(M, k_splits);
    float* part = reinterpret_cast<float*>(smem);
    float* recv = part + k_splits * sf;  // slot per sending member
    cluster_wait_acquire();  // every member's MMAs are done: its ring may be written
    if (threadIdx.x == 0) {
      const uint32_t bytes = uint32_t(M * rp * 4);
      for (int d = 1; d < k_splits; ++d) {
        const uint32_t peer = (rank + uint32_t(d)) % uint32_t(k_splits);
        bulk_copy_to_peer(mapa_shared(smem_u32(recv + rank * sf), peer),
                          smem_u32(part + peer * sf), bytes,
                          mapa_shared(smem_u32(&bars->recv), peer));
      }
      bulk_commit();
    }
    if (mbar_wait(&bars->recv, 0, status)) {
      const float* mine = part + rank * sf;
      if (swiglu) {
        const int h = rp / 2, q = h / 4;
        for (int it = threadIdx.x; it < M * q; it += blockDim.x) {
          const int m = it / q;
          const int g4 = (it - m * q) * 4;
          float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
          for (int sp = 0; sp < k_splits; ++sp) {  // member order, as the pull reduction
            const float* src = (sp == int(rank) ? mine : recv + sp * sf) + m * rp;
            const float4 a = *reinterpret_cast<const float4*>(src + g4);
            const float4 b = *reinterpret_cast<const float4*>(src + h + g4);
            if (sp == 0) {
              g = a;
              u = b;
            } else {
              g.x += a.x; g.y += a.y; g.z += a.z; g.w += a.w;
              u.x += b.x; u.y += b.y; u.z += b.z; u.w += b.w;
            }
          }
          const float ga[4] = {g.x, g.y, g.z, g.w};
          const float ua[4] = {u.x, u.y, u.z, u.w};
          float o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float gf = Elem<T>::to_f32(Elem<T>::from_f32(ga[e]));
            const float sg = Elem<T>::to_f32(Elem<T>::from_f32(gf / (1.0f + expf(-gf))));
            o[e] = sg * Elem<T>::to_f32(Elem<T>::from_f32(ua[e]));
          }
          T* dst = y + int64_t(m) * y_stride + n_tile * 64 + int(rank) * h + g4;
          if ((reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
            uint2 pk;
            pk.x = pack2<T>(o[0], o[1]);
            pk.y = pack2<T>(o[2], o[3]);
            *reinterpret_cast<uint2*>(dst) = pk;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = Elem<T>::from_f32(o[e]);
          }
        }
      } else {
        const int q = rp / 4;
        for (int it = threadIdx.x; it < M * q; it += blockDim.x) {
          const int m = it / q;
          const int p4 = (it - m * q) * 4;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int sp = 0; sp < k_splits; ++sp) {  // member order, as the pull reduction
            const float* src = (sp == int(rank) ? mine : recv + sp * sf) + m * rp;
            const float4 a = *reinterpret_cast<const float4*>(src + p4);
            if (sp == 0) {
              acc = a;
            } else {
              acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
            }
          }
          const int n0 = n_tile * kTileN + int(rank) * rp + p4;
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
      }
    }
    // this CTA's shared memory is the source of its outgoing copies until they are read
    if (threadIdx.x == 0) bulk_wait_reads();
  } else if (k_splits > 1) {
    // every member's partial is complete and visible after this barrier
    cluster_sync_all();
    const uint32_t rank = cluster_rank();
    const uint32_t base = smem_u32(smem);
    if (swiglu) {
      // this member finishes gate rows [r0, r0 + rows) and the matching up rows + 64
      const int rows = 64 / k_splits;
      const int q = rows / 4;
      const int r0 = int(rank) * rows;
      for (int it = threadIdx.x; it < M * q; it += blockDim.x) {
        const int m = it / q;
        const int nl = r0 + (it - m * q) * 4;
        const uint32_t off_g = base + uint32_t(m * kPartStride + nl) * 4u;
        const uint32_t off_u = off_g + 64u * 4u;
        float4 pg[kMaxSplits], pu[kMaxSplits];
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp)
          if (sp < k_splits) {
            pg[sp] = ld_dsmem_f4(mapa_shared(off_g, uint32_t(sp)));
            pu[sp] = ld_dsmem_f4(mapa_shared(off_u, uint32_t(sp)));
          }
        float4 g = pg[0], u = pu[0];
#pragma unroll
        for (int sp = 1; sp < kMaxSplits; ++sp) {  // member order, as the plain reduction
          if (sp < k_splits) {
            g.x += pg[sp].x; g.y += pg[sp].y; g.z += pg[sp].z; g.w += pg[sp].w;
            u.x += pu[sp].x; u.y += pu[sp].y; u.z += pu[sp].z; u.w += pu[sp].w;
          }
        }
        const float ga[4] = {g.x, g.y, g.z, g.w};
        const float ua[4] = {u.x, u.y, u.z, u.w};
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float gf = Elem<T>::to_f32(Elem<T>::from_f32(ga[e]));
          const float sg = Elem<T>::to_f32(Elem<T>::from_f32(gf / (1.0f + expf(-gf))));
          o[e] = sg * Elem<T>::to_f32(Elem<T>::from_f32(ua[e]));
        }
        T* dst = y + int64_t(m) * y_stride + n_tile * 64 + nl;  // inside [0, N / 2)
        if ((reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
          uint2 pk;
          pk.x = pack2<T>(o[0], o[1]);
          pk.y = pack2<T>(o[2], o[3]);
          *reinterpret_cast<uint2*>(dst) = pk;
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = Elem<T>::from_f32(o[e]);
        }
      }
    } else {
      const int rows = kTileN / k_splits;  // weight rows this member finishes
      const int q = rows / 4;              // float4 vectors per batch row
      const int r0 = int(rank) * rows;
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

// K splits: a power of two <= AS_LINEAR_MAX_SPLITS (so 128 divides evenly among the
// members), enough CTAs for AS_LINEAR_CTAS_PER_SM per SM, at least 2 K steps per member.
#ifndef AS_LINEAR_CTAS_PER_SM
#define AS_LINEAR_CTAS_PER_SM 2  // measured in the decode step with the push exchange
#endif
#ifndef AS_LINEAR_MAX_SPLITS
#define AS_LINEAR_MAX_SPLITS kMaxSplits
#endif
int choose_splits(int N, int k_steps) {
  const int n_tiles = (N + kTileN - 1) / kTileN;
  const int want = (AS_LINEAR_CTAS_PER_SM * sm_count() + n_tiles - 1) / n_tiles;
  int s = 1;
  while (s * 2 <= AS_LINEAR_MAX_SPLITS && s * 2 <= want && s * 2 <= k_steps / 2) s *= 2;
  return s;
}

template <typename T>
int launch_linear(void* y, int64_t y_stride, const void* x, int64_t x_stride, const void* w,
                  int M, int N, int K, cudaStream_t stream, int swiglu = 0) {
  const int Mpad = pad_m(M);
  const int n_tiles = (N + kTileN - 1) / kTileN;
  const int k_steps = (K + kTileK - 1) / kTileK;
  const int k_splits = choose_splits(N, k_steps);
  CUtensorMap mw, mx;
  const uint64_t es = sizeof(T);
  {
    const uint64_t dims[2] = {uint64_t(K), uint64_t(N)};
    const uint64_t strides[1] = {uint64_t(K) * es};
    const uint32_t box[2] = {uint32_t(kTileK), uint32_t(swiglu ? kTileN / 2 : kTileN)};
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
  const int stages = num_stages(Mpad);
  const int smem = smem_bytes(Mpad, stages);
  // K-split exchange: push (bulk copies between members) when the partial and the
  // receive slots fit in the stage ring together, else the pull reduction
  const int push = (AS_LINEAR_PUSH && k_splits > 1 &&
                    2 * k_splits * slice_floats(M, k_splits) * 4 <= stages * stage_bytes(Mpad))
                       ? 1
                       : 0;
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
                     k_splits, stages, swiglu, push, device_status_ptr());
  return check_launch(swiglu ? "as_linear_small_m_swiglu" : "as_linear_small_m");
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

extern "C" int as_linear_small_m_swiglu(void* y, int64_t y_stride, const void* x,
                                        int64_t x_stride, const void* w_gate_up, int32_t M,
                                        int32_t inter, int32_t K, int32_t dtype,
                                        as_stream_t stream) {
  if (dtype != AS_DTYPE_BF16 && dtype != AS_DTYPE_F16)
    return fail(AS_ERR_UNSUPPORTED, "as_linear_small_m_swiglu: bf16 or fp16 only");
  if (M < 0 || inter <= 0 || K <= 0 || inter % 64)
    return fail(AS_ERR_INVALID_ARG,
                "as_linear_small_m_swiglu: bad sizes (inter must be a positive multiple of 64)");
  if (M == 0) return AS_OK;
  if (M > kMaxM) return fail(AS_ERR_UNSUPPORTED, "as_linear_small_m_swiglu: M > %d", kMaxM);
  if (!y || !x || !w_gate_up)
    return fail(AS_ERR_INVALID_ARG, "as_linear_small_m_swiglu: null pointer");
  if (y_stride < inter || x_stride < K)
    return fail(AS_ERR_INVALID_ARG, "as_linear_small_m_swiglu: row stride shorter than the row");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_gate_up)) & 15 ||
      (x_stride * 2) % 16 || (int64_t(K) * 2) % 16)
    return fail(AS_ERR_INVALID_ARG,
                "as_linear_small_m_swiglu: x, w and their rows must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == AS_DTYPE_BF16)
    return launch_linear<__nv_bfloat16>(y, y_stride, x, x_stride, w_gate_up, M, 2 * inter,
                                        K, s, 1);
  return launch_linear<__half>(y, y_stride, x, x_stride, w_gate_up, M, 2 * inter, K, s, 1);
}
