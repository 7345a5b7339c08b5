// (4) Varlen prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Semantics: LlamaAttention.forward over a cached prefix (agentserve/model/llama.py:
// 128-186): new token i of a sequence whose first P tokens are cached attends to keys
// 0..P+i (prefix unmasked, new tokens causal, mask of llama.py:171-180).  K/V are read
// in place from the paged pool.
//
// CTA = (query tile, KV head g, sequence).  A query tile is 128 rows = tq tokens x the
// `group` query heads that share KV head g (row = token*group + head), so every K/V
// tile loaded is used by the whole GQA group.  Warp roles (192 threads):
//   warp 0     TMA producer: the Q tile (3-D map over q) once, then per KV tile of
//              128 keys the 8 paged blocks of K and of V (4-D maps over the pool,
//              128-byte swizzle), 2-stage ring on full/empty mbarriers;
//   warp 1     MMA issuer (one thread): S = Q K^T into TMEM (M=128, N=128, K=D,
//              both operands K-major), then O += P V into TMEM (M=128, N=D, K=128;
//              P K-major from shared memory, V MN-major); tcgen05.commit arrives on
//              the mbarriers; S of tile j+1 is issued as soon as the softmax warps
//              have copied S of tile j into registers;
//   warps 2-5  softmax, one TMEM lane (= one row) per thread: tcgen05.ld of the S
//              row, causal/length mask, online softmax in fp32 (exp2 domain), P
//              written as bf16/fp16 into 128B-swizzled shared memory, O rescaled in
//              TMEM when the row max grows; epilogue reads O, divides by the row sum
//              and stores the row.
// TMEM: 256 columns (S: 128, O: D).  Every wait is bounded; a wait that runs out
// sets status bit 4, the CTA stops issuing work, drains its MMAs, frees TMEM and
// writes nothing.
#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "prefill_tcgen05.h"
#include "tcgen05.cuh"

namespace asb {
namespace {

constexpr int kBS = 16;
constexpr float kLazySlack = 8.0f;  // log2 units: rescale only when a row max grows > 2^8

#ifndef AS_PREFILL_STAGES
#define AS_PREFILL_STAGES 2
#endif

template <int D>
struct PfCfg {
  static constexpr int kBM = 128;                 // Q-tile rows
  static constexpr int kBN = 128;                 // keys per KV tile (8 blocks)
  static constexpr int kSub = D / 64;             // 64-element (128 B) swizzle sub-tiles
  static constexpr int kStages = AS_PREFILL_STAGES;
  static constexpr int kSubBytes = 128 * 128;     // 128 rows x 128 B
  static constexpr int kQBytes = kSub * kSubBytes;
  static constexpr int kKVBytes = kSub * kSubBytes;  // one of K or V for one KV tile
  static constexpr int kPBytes = 2 * kSubBytes;      // 128 rows x 128 keys x 2 B
  static constexpr int kOffQ = 0;
  static constexpr int kOffKV = kOffQ + kQBytes;
  static constexpr int kOffP = kOffKV + kStages * 2 * kKVBytes;
  static constexpr int kOffBar = kOffP + kPBytes;
  // The dynamic shared window is declared 1024-byte aligned (128B-swizzle atoms), so
  // no alignment slack is reserved: at D=64 two CTAs fit on one SM.
  static constexpr int kSmemBytes = kOffBar + 256;
  static constexpr int kThreads = 192;
  static constexpr int kTmemCols = 256;
  static constexpr int kMinBlocks = (kOffBar + 256) * 2 <= 225 * 1024 ? 2 : 1;
};

struct PfBars {
  uint64_t q_full;
  uint64_t kv_full[8];
  uint64_t kv_empty[8];
  uint64_t s_full;
  uint64_t s_free;
  uint64_t p_full;
  uint64_t pv_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* p) {
  uint4 v;
  v.x = pack2<T>(p[0], p[1]);
  v.y = pack2<T>(p[2], p[3]);
  v.z = pack2<T>(p[4], p[5]);
  v.w = pack2<T>(p[6], p[7]);
  return v;
}

__device__ __forceinline__ bool aborted(volatile int* f) { return *f != 0; }

template <typename T, int D>
__global__ void __launch_bounds__(192, PfCfg<D>::kMinBlocks)
prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                  const __grid_constant__ CUtensorMap tmap_k,
                  const __grid_constant__ CUtensorMap tmap_v,
                  const __grid_constant__ CUtensorMap tmap_k8,
                  const __grid_constant__ CUtensorMap tmap_v8, T* __restrict__ out,
                  const int32_t* __restrict__ bt, int64_t bt_stride,
                  const int32_t* __restrict__ cu_seqlens_q, const int32_t* __restrict__ seq_lens_k,
                  int H, int group, int num_blocks, int max_blocks, float scale_log2,
                  int run8_ok, int* status) {
  using Cfg = PfCfg<D>;
  constexpr int NS = Cfg::kStages;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = tc::idesc_f16(kBF16, 128, 128, false, false);
  constexpr uint32_t kIdescO = tc::idesc_f16(kBF16, 128, D, false, true);

  const int r = blockIdx.z;
  const int g = blockIdx.y;
  const int q_begin = cu_seqlens_q[r];
  const int nq = cu_seqlens_q[r + 1] - q_begin;
  const int tq = Cfg::kBM / group;
  const int tile = int(gridDim.x) - 1 - int(blockIdx.x);  // longest (last) tiles first
  const int t0 = tile * tq;
  if (t0 >= nq) return;
  int Lk = seq_lens_k[r];
  if (Lk > max_blocks * kBS) {
    if (threadIdx.x == 0) flag_status(status, kStatusBadLength);
    Lk = max_blocks * kBS;
  }
  const int P = Lk - nq;  // cached prefix length
  if (P < 0) {
    if (threadIdx.x == 0) flag_status(status, kStatusBadLength);
    return;
  }
  const int kv_end = P + min(t0 + tq, nq);
  const int n_kv = (kv_end + Cfg::kBN - 1) / Cfg::kBN;
  const int nblk_seq = (Lk + kBS - 1) / kBS;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if (smem_u32(smem) & 1023u) {  // never expected; refuse rather than mis-swizzle
    if (threadIdx.x == 0) flag_status(status, kStatusWaitTimeout);
    return;
  }
  PfBars* bars = reinterpret_cast<PfBars*>(smem + Cfg::kOffBar);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->s_free, 4);
    mbar_init(&bars->p_full, 4);
    mbar_init(&bars->pv_done, 1);
    mbar_init(&bars->drain, 1);
    bars->abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tS = tmem;
  const uint32_t tO = tmem + 128;
  const uint32_t sQ = smem_u32(smem + Cfg::kOffQ);
  const uint32_t sKV = smem_u32(smem + Cfg::kOffKV);
  const uint32_t sP = smem_u32(smem + Cfg::kOffP);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    const int filler = (nblk_seq > 0) ? bt[int64_t(r) * bt_stride] : 0;
    const int fill_ok = (filler >= 0 && filler < num_blocks) ? filler : 0;
    if (lane == 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      tma_prefetch_desc(&tmap_k8);
      tma_prefetch_desc(&tmap_v8);
      mbar_arrive_expect_tx(&bars->q_full, Cfg::kQBytes);
      const uint64_t pol_q = l2_policy_evict_first();
      for (int s = 0; s < Cfg::kSub; ++s)
        tma_load_3d(smem + Cfg::kOffQ + s * Cfg::kSubBytes, &tmap_q, &bars->q_full, s * 64,
                    g * group, q_begin + t0, pol_q);
    }
    // K/V by TMA: lane b issues block b of the tile (K and V boxes of 16 tokens x 64
    // columns of this KV head); block ids of tile j+1 are fetched while tile j issues.
    auto load_id = [&](int jt) -> int {
      const int blk = 8 * jt + (lane & 7);
      int id = fill_ok;  // keys past the sequence: finite filler data, masked to p = 0
      if (blk < nblk_seq) {
        id = __ldg(bt + int64_t(r) * bt_stride + blk);
        if (id < 0 || id >= num_blocks) {
          flag_status(status, kStatusBadBlockId);
          id = fill_ok;
        }
      }
      return id;
    };
    const uint64_t pol_kv = l2_policy_evict_last();
    int id_next = load_id(0);
    for (int j = 0; j < n_kv; ++j) {
      if (__any_sync(0xffffffffu, aborted(abort_flag))) break;
      const int st = j % NS;
      const bool ready = j < NS || mbar_wait(&bars->kv_empty[st], ((j / NS) + 1) & 1, status);
      if (!__all_sync(0xffffffffu, ready)) {
        *abort_flag = 1;
        break;
      }
      const int id = id_next;
      if (j + 1 < n_kv) id_next = load_id(j + 1);
      // A tile whose 8 blocks are consecutive pool ids (a request's blocks handed out
      // together by the FIFO free list) moves as one 16-block box per operand.
      const int id0 = __shfl_sync(0xffffffffu, id, 0);
      const bool run8 = run8_ok && __all_sync(0xffffffffu, id == id0 + (lane & 7));
      if (lane == 0) mbar_arrive_expect_tx(&bars->kv_full[st], 2 * Cfg::kKVBytes);
      __syncwarp();
      if (run8) {
        if (lane == 0) {
          uint8_t* kdst = smem + Cfg::kOffKV + st * 2 * Cfg::kKVBytes;
#pragma unroll
          for (int sb = 0; sb < Cfg::kSub; ++sb) {
            tma_load_4d(kdst + sb * Cfg::kSubBytes, &tmap_k8, &bars->kv_full[st], sb * 64, g, 0,
                        id0, pol_kv);
            tma_load_4d(kdst + Cfg::kKVBytes + sb * Cfg::kSubBytes, &tmap_v8, &bars->kv_full[st],
                        sb * 64, g, 0, id0, pol_kv);
          }
        }
      } else if (lane < 8) {
        uint8_t* kdst = smem + Cfg::kOffKV + st * 2 * Cfg::kKVBytes + lane * 2048;
        uint8_t* vdst = kdst + Cfg::kKVBytes;
#pragma unroll
        for (int sb = 0; sb < Cfg::kSub; ++sb) {
          tma_load_4d(kdst + sb * Cfg::kSubBytes, &tmap_k, &bars->kv_full[st], sb * 64, g, 0, id,
                      pol_kv);
          tma_load_4d(vdst + sb * Cfg::kSubBytes, &tmap_v, &bars->kv_full[st], sb * 64, g, 0, id,
                      pol_kv);
        }
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      auto issue_s = [&](int st) {
        const uint32_t kbase = sKV + st * 2 * Cfg::kKVBytes;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * Cfg::kSubBytes + (k & 3) * 32;
          tc::mma_f16(tS, tc::sdesc_sw128(sQ + off, 16, 1024), tc::sdesc_sw128(kbase + off, 16, 1024),
                      kIdescS, k > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int st, bool acc) {
        const uint32_t vbase = sKV + st * 2 * Cfg::kKVBytes + Cfg::kKVBytes;
#pragma unroll
        for (int k = 0; k < Cfg::kBN / 16; ++k) {
          const uint32_t aoff = (k >> 2) * Cfg::kSubBytes + (k & 3) * 32;
          tc::mma_f16(tO, tc::sdesc_sw128(sP + aoff, 16, 1024),
                      tc::sdesc_sw128(vbase + k * 2048, Cfg::kSubBytes, 1024), kIdescO,
                      (acc || k > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(&bars->q_full, 0, status) && mbar_wait(&bars->kv_full[0], 0, status);
      if (ok && n_kv > 0) {
        tc::fence_after_sync();
        issue_s(0);
        tc::commit(&bars->s_full);
      }
      // S(j+1) needs tile j+1's K/V and the softmax warps' copy of S(j); PV(j) needs
      // P(j).  Poll both and issue whichever is ready first, so PV(j) never waits
      // behind the next tile's load (that load can only start once a stage frees).
      for (int j = 0; ok && j < n_kv; ++j) {
        if (aborted(abort_flag)) break;
        const int st = j % NS;
        bool s_next = j + 1 >= n_kv;  // nothing to issue after the last tile
        const int st1 = (j + 1) % NS;
        const uint32_t kv_par = ((j + 1) / NS) & 1;
        const uint64_t t0 = global_timer_ns();
        bool pv_ready = false;
        for (uint32_t spin = 0; !pv_ready; ++spin) {
          if (!s_next && mbar_try_wait(&bars->kv_full[st1], kv_par) &&
              mbar_try_wait(&bars->s_free, j & 1)) {
            tc::fence_after_sync();
            issue_s(st1);
            tc::commit(&bars->s_full);
            s_next = true;
          }
          pv_ready = mbar_try_wait(&bars->p_full, j & 1);
          if (!pv_ready && (spin & 255u) == 255u && global_timer_ns() - t0 > kWaitLimitNs) {
            flag_status(status, kStatusWaitTimeout);
            ok = false;
            break;
          }
        }
        if (!ok) break;
        tc::fence_after_sync();
        issue_pv(st, j > 0);
        tc::commit(&bars->pv_done);
        tc::commit(&bars->kv_empty[st]);
        if (!s_next) {
          if (!mbar_wait(&bars->kv_full[st1], kv_par, status) ||
              !mbar_wait(&bars->s_free, j & 1, status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          issue_s(st1);
          tc::commit(&bars->s_full);
        }
      }
      if (!ok) *abort_flag = 1;
      // every MMA this thread issued is complete before TMEM is released
      tc::commit(&bars->drain);
      mbar_wait(&bars->drain, 0, status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int t = row / group;
    const int hq = row - t * group;
    const int tok = t0 + t;
    const bool valid = tok < nq;
    const int qpos = valid ? P + tok : P + t0;
    const uint32_t trow = uint32_t(quad * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const bool go = !aborted(abort_flag) && mbar_wait(&bars->s_full, j & 1, status);
      if (!__all_sync(0xffffffffu, go)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      float x[128];
      {
        uint32_t v0[32], v1[32], v2[32], v3[32];
        tc::ld_32x32b_x32(tS + trow + 0, v0);
        tc::ld_32x32b_x32(tS + trow + 32, v1);
        tc::ld_32x32b_x32(tS + trow + 64, v2);
        tc::ld_32x32b_x32(tS + trow + 96, v3);
        tc::wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = __uint_as_float(v0[i]);
          x[32 + i] = __uint_as_float(v1[i]);
          x[64 + i] = __uint_as_float(v2[i]);
          x[96 + i] = __uint_as_float(v3[i]);
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_free);

      // Raw scores; masked only where the causal diagonal or the sequence end cuts
      // this tile (keys c <= lim are visible).
      const int lim = qpos - j * Cfg::kBN;
      if (lim < Cfg::kBN - 1) {
#pragma unroll
        for (int c = 0; c < 128; ++c) x[c] = (c <= lim) ? x[c] : -INFINITY;
      }
      // row max as a tree (8 independent chains), not one 128-long dependency chain
      float mp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mp[i] = x[i];
#pragma unroll
      for (int c = 8; c < 128; c += 8) {
#pragma unroll
        for (int i = 0; i < 8; ++i) mp[i] = fmaxf(mp[i], x[c + i]);
      }
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      // Lazy max (one row per thread, no cross-lane work): scores are exponentiated
      // against the reference max m (log2 units) unless this tile beats it by more
      // than 2^8; only then do m, l and the row of O in TMEM get rescaled.
      float alpha = 1.f;
      if (mx * scale_log2 > m + kLazySlack) {
        const float m_new = mx * scale_log2;
        alpha = fast_exp2(m - m_new);
        m = m_new;
      }
      const float neg_m = -m;
      // P for this tile, packed to the element type, computed before waiting for the
      // previous tile's PV MMA (which still reads the P buffer) so the exponentials
      // overlap it.
      float sp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // 8 independent partial sums
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p0 = fast_exp2(fmaf(x[2 * c], scale_log2, neg_m));
        const float p1 = fast_exp2(fmaf(x[2 * c + 1], scale_log2, neg_m));
        sp[c & 7] += p0 + p1;
        pk[c] = pack2<T>(p0, p1);
      }
      const float sum = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
      if (j > 0) {
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->pv_done, (j - 1) & 1, status))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
      }
#pragma unroll
      for (int c8 = 0; c8 < 16; ++c8) {
        const int sub = c8 >> 3, cc = c8 & 7;
        const uint32_t addr = sP + sub * Cfg::kSubBytes + (row >> 3) * 1024 + (row & 7) * 128 +
                              ((cc ^ (row & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * c8]),
                     "r"(pk[4 * c8 + 1]), "r"(pk[4 * c8 + 2]), "r"(pk[4 * c8 + 3])
                     : "memory");
      }
      l = l * alpha + sum;
      if (j > 0 && __any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tc::ld_32x32b_x32(tO + trow + c * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tc::st_32x32b_x32(tO + trow + c * 32, o);
        }
        tc::wait_st();
      }
      fence_proxy_async_smem();  // P (generic-proxy stores) visible to the MMA
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full);
    }
    if (!ok) *abort_flag = 1;
    const bool done = ok && n_kv > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(&bars->pv_done, (n_kv - 1) & 1, status));
    if (done) {
      tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* dst = out + (int64_t(q_begin) + tok) * int64_t(H) * D + int64_t(g * group + hq) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tc::ld_32x32b_x32(tO + trow + c * 32, o);
        tc::wait_ld();
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o[i + e]) * inv;
            *reinterpret_cast<uint4*>(dst + c * 32 + i) = pack8<T>(f);
          }
        }
      }
    } else if (ok && n_kv > 0) {
      *abort_flag = 1;
    }
    tc::fence_before_sync();
  }

  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <typename T>
CUtensorMapDataType tmap_dtype() {
  return std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

template <typename T, int D>
int launch_tc(void* out, const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
              const int32_t* bt, int64_t bt_stride, const int32_t* cu, const int32_t* lk, int R,
              int max_seqlen_q, int total_q, int H, int Kh, int num_blocks, int max_blocks,
              float scale, cudaStream_t stream) {
  using Cfg = PfCfg<D>;
  const int group = H / Kh;
  const int tq = Cfg::kBM / group;
  const uint64_t es = sizeof(T);
  CUtensorMap mq, mk, mv, mk8, mv8;
  {
    const uint64_t dims[3] = {uint64_t(D), uint64_t(H), uint64_t(total_q)};
    const uint64_t strides[2] = {uint64_t(D) * es, uint64_t(q_stride) * es};
    const uint32_t box[3] = {64, uint32_t(group), uint32_t(tq)};
    int rc = encode_tensor_map(&mq, tmap_dtype<T>(), 3, const_cast<void*>(q), dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[4] = {uint64_t(D), uint64_t(Kh), uint64_t(kBS), uint64_t(num_blocks)};
    const uint64_t strides[3] = {uint64_t(D) * es, uint64_t(Kh) * D * es,
                                 uint64_t(kBS) * Kh * D * es};
    const uint32_t box[4] = {64, 1, uint32_t(kBS), 1};
    int rc = encode_tensor_map(&mk, tmap_dtype<T>(), 4, const_cast<void*>(k_cache), dims, strides,
                               box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tensor_map(&mv, tmap_dtype<T>(), 4, const_cast<void*>(v_cache), dims, strides,
                           box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    // 8 consecutive blocks of one KV head: 128 rows of 128 B, the same shared-memory
    // image as 8 single-block boxes 2 KB apart
    const uint32_t box8[4] = {64, 1, uint32_t(kBS), num_blocks >= 8 ? 8u : 1u};
    rc = encode_tensor_map(&mk8, tmap_dtype<T>(), 4, const_cast<void*>(k_cache), dims, strides,
                           box8, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tensor_map(&mv8, tmap_dtype<T>(), 4, const_cast<void*>(v_cache), dims, strides,
                           box8, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  auto kern = prefill_tc_kernel<T, D>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  const int ntiles = (max_seqlen_q + tq - 1) / tq;
  dim3 grid(ntiles, Kh, R);
  kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(
      mq, mk, mv, mk8, mv8, static_cast<T*>(out),
      bt, bt_stride, cu, lk, H, group, num_blocks, max_blocks,
      scale * kLog2e, num_blocks >= 8 ? 1 : 0, device_status_ptr());
  return check_launch("as_varlen_prefill_attention (tcgen05)");
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool prefill_tc_supported(int dtype, int H, int Kh, int D, const void* q, int64_t q_stride,
                          const void* k_cache, const void* v_cache, const void* out) {
  if (dtype != AS_DTYPE_BF16 && dtype != AS_DTYPE_F16) return false;
  if (D != 64 && D != 128) return false;
  const int group = H / Kh;
  if (group < 1 || group > 128 || 128 % group != 0) return false;
  if (!al16(q) || !al16(k_cache) || !al16(v_cache) || !al16(out)) return false;
  if ((q_stride * 2) % 16 != 0) return false;
  return true;
}

int prefill_tc_launch(void* out, const void* q, int64_t q_stride, const void* k_cache,
                      const void* v_cache, const int32_t* bt, int64_t bt_stride,
                      const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int R,
                      int max_seqlen_q, int total_q, int H, int Kh, int D, int num_blocks,
                      int max_blocks, float scale, int dtype, int n_split, void* workspace,
                      cudaStream_t stream) {
  if (max_seqlen_q <= 0) return AS_OK;
  if (R > 65535) return fail(AS_ERR_INVALID_ARG, "as_varlen_prefill_attention: too many sequences");
#ifndef AS_PREFILL_PAIR
#define AS_PREFILL_PAIR 1
#endif
  if (AS_PREFILL_PAIR && (D == 64 || D == 128))
    return prefill_pair_launch(out, q, q_stride, k_cache, v_cache, bt, bt_stride, cu_seqlens_q,
                               seq_lens_k, R, max_seqlen_q, total_q, H, Kh, D, num_blocks,
                               max_blocks, scale, dtype, n_split, workspace, stream);
  if (dtype == AS_DTYPE_BF16) {
    using T = __nv_bfloat16;
    if (D == 64)
      return launch_tc<T, 64>(out, q, q_stride, k_cache, v_cache, bt, bt_stride, cu_seqlens_q,
                              seq_lens_k, R, max_seqlen_q, total_q, H, Kh, num_blocks, max_blocks,
                              scale, stream);
    return launch_tc<T, 128>(out, q, q_stride, k_cache, v_cache, bt, bt_stride, cu_seqlens_q,
                             seq_lens_k, R, max_seqlen_q, total_q, H, Kh, num_blocks, max_blocks,
                             scale, stream);
  }
  using T = __half;
  if (D == 64)
    return launch_tc<T, 64>(out, q, q_stride, k_cache, v_cache, bt, bt_stride, cu_seqlens_q,
                            seq_lens_k, R, max_seqlen_q, total_q, H, Kh, num_blocks, max_blocks,
                            scale, stream);
  return launch_tc<T, 128>(out, q, q_stride, k_cache, v_cache, bt, bt_stride, cu_seqlens_q,
                           seq_lens_k, R, max_seqlen_q, total_q, H, Kh, num_blocks, max_blocks,
                           scale, stream);
}

}  // namespace asb
