// (4) Varlen prefill attention, head_dim 64 and 128: two query tiles per CTA sharing
// every K/V tile, P kept in tensor memory.
//
// Semantics: LlamaAttention.forward over a cached prefix (agentserve/model/llama.py:
// 128-186): token i of a sequence with P cached tokens attends to keys 0..P+i (prefix
// unmasked, new tokens causal, the mask of llama.py:171-180), K/V read in place from
// the paged pool.
//
// CTA = (pair of query tiles, KV head g, sequence).  Query tile i (i = 0, 1) holds
// 128 rows = tq tokens x the `group` query heads of KV head g.  Per KV tile (128 keys
// = 8 paged blocks at head_dim 64, 64 keys = 4 blocks at 128) the K and V boxes land
// in shared memory once and feed both query tiles, halving TMA work and shared-memory
// traffic per query row compared with one tile per CTA.  Warp roles (320 threads, one CTA per SM):
//   warp 0      TMA producer: both Q tiles once, then K/V tiles into a 4-stage ring;
//   warp 1      MMA issuer (one thread), polling: S_i = Q_i K^T (both operands from
//               shared memory, 128B swizzle) as soon as tile j's K/V is in and
//               softmax i has read S_i(j-1); O_i += P_i V with P_i read from TMEM
//               as soon as softmax i has written it;
//   warps 2-5   softmax of query tile 0, warps 6-9 softmax of query tile 1: one TMEM
//               lane (row) per thread; online softmax in the exp2 domain with a lazy
//               maximum (O rescaled in TMEM only when a row maximum grows by > 2^8),
//               paired fp32 arithmetic (f32x2) and 3-input max; P packed to 16-bit
//               pairs and stored to TMEM with tcgen05.st.  The two warps that share an
//               SM sub-partition take turns on its exponent unit (ping-pong), so one
//               warp's TMEM loads, stores and waits overlap the other's exponentials.
// TMEM (512 columns): tile i owns [256 i, 256 i + 256): S one column per key of the
// KV tile, P half as many (16-bit pairs), O D columns (see PairCfg).
// Every wait is bounded; a wait that
// runs out sets status bit 4, the CTA stops issuing, drains its MMAs, frees TMEM
// and writes nothing.
#include <type_traits>

#include "common.cuh"
#include "host_util.h"
#include "prefill_tcgen05.h"
#include "tcgen05.cuh"

namespace asb {
namespace {

constexpr int kBS = 16;
constexpr float kLazySlack = 8.0f;
constexpr int kMaxSplits = 16;

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }
// query-tile pairs per (sequence, KV head): 2 x 128 rows = 2 x (128 / group) tokens
int pair_count(int max_seqlen_q, int H, int Kh) {
  const int tq = 128 / (H / Kh);
  return (max_seqlen_q + 2 * tq - 1) / (2 * tq);
}

#ifndef AS_PREFILL_PAIR_STAGES
#define AS_PREFILL_PAIR_STAGES 4
#endif
#ifndef AS_PREFILL_PINGPONG
#define AS_PREFILL_PINGPONG 1
#endif
// The exponent-unit turn passes to the partner warp after this many of the 64 column
// pairs (64: at the end), so the hand-off latency overlaps the remaining pairs
// (measured on B200, 8 requests: 64 -> 566-571, 32 -> 604-606 TFLOP/s).
#ifndef AS_PREFILL_HANDOFF
#define AS_PREFILL_HANDOFF 32
#endif
// ---- packed fp32 pairs (sm_100 f32x2 arithmetic) --------------------------------
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// 2^x for a pair of fp32 values on the FMA pipe instead of the exponent unit (the
// softmax at head_dim 64 is bound by the exponent unit: 16 results per clock per SM).
// Cody-Waite style split x = j + f with j = floor(x), f in [0, 1): adding 1.5 * 2^23
// with round-toward-minus-infinity leaves j in the low mantissa bits; 2^f is a cubic
// fitted here to minimise the relative error on [0, 1) (p(0) = 1 exactly, largest
// relative error 8.6e-5, far below bf16's 3.9e-3 rounding of P); 2^j is added to
// the exponent field.  x is clamped to >= -127 so masked (-inf) scores give ~0.
#ifndef AS_PREFILL_POLY_EVERY
#define AS_PREFILL_POLY_EVERY 0  // 0: every exponential on the exponent unit
#endif
#if AS_PREFILL_POLY_EVERY > 0
__device__ __forceinline__ uint64_t f2_add_rm(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t exp2_poly_f2(uint64_t x2) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  float a, b;
  f2_unpack(x2, a, b);
  const uint64_t xc = f2_pack(fmaxf(a, -127.f), fmaxf(b, -127.f));
  const uint64_t mg = f2_pack(kMagic, kMagic);
  const uint64_t r = f2_add_rm(xc, mg);     // low mantissa bits = floor(x)
  const uint64_t fr = f2_sub(xc, f2_sub(r, mg));
  uint64_t p = f2_fma(fr, f2_pack(0.07706265f, 0.07706265f), f2_pack(0.2276498f, 0.2276498f));
  p = f2_fma(p, fr, f2_pack(0.69511575f, 0.69511575f));
  p = f2_fma(p, fr, f2_pack(1.0f, 1.0f));
  float pa, pb, ra, rb;
  f2_unpack(p, pa, pb);
  f2_unpack(r, ra, rb);
  const float ea = __uint_as_float(__float_as_uint(pa) + (__float_as_uint(ra) << 23));
  const float eb = __uint_as_float(__float_as_uint(pb) + (__float_as_uint(rb) << 23));
  return f2_pack(ea, eb);
}
#endif

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Keys per KV tile at head_dim 128: 128 (default) or 64.  With 128, S (128 columns)
// and O (128) fill a query tile's 256 TMEM columns, so P must alias S and S(j+1) can
// only be issued after PV(j) has read P(j); with 64, S, P and O sit side by side and
// S(j+1) overlaps the softmax of tile j, but the S MMAs run at N=64 and every
// per-tile cost is paid twice as often: measured on B200 (8 requests of 14,336 cached
// + 600 new tokens) 683 TFLOP/s against 752 with 128-key tiles.
#ifndef AS_PREFILL_BN128
#define AS_PREFILL_BN128 128
#endif
#ifndef AS_PREFILL_STAGES128
#define AS_PREFILL_STAGES128 4  // ring stages at head_dim 128 with 64-key tiles (<= 5 fit)
#endif

template <int HD>
struct PairCfg {
  static constexpr int D = HD;
  static constexpr int kBM = 128;
  static constexpr int kBN = D == 128 ? AS_PREFILL_BN128 : 128;  // keys per KV tile
  static constexpr int kBlocks = kBN / kBS;       // paged blocks per KV tile
  static constexpr int kSub = D / 64;             // 64-element (128 B) swizzle sub-tiles
  static constexpr int kSubBytes = 128 * 128;     // Q sub-tile: 128 rows x 128 B
  static constexpr int kKVSubBytes = kBN * 128;   // K/V sub-tile: kBN keys x 128 B
  static constexpr int kQBytes = kSub * kSubBytes;     // one query tile
  static constexpr int kKVBytes = kSub * kKVSubBytes;  // K (or V) of one KV tile
  static constexpr int kStages =
      D == 64 ? AS_PREFILL_PAIR_STAGES : (kBN == 64 ? AS_PREFILL_STAGES128 : 2);
  static constexpr int kOffQ = 0;                    // Q tile i at kOffQ + i * kQBytes
  static constexpr int kOffKV = 2 * kQBytes;         // stage s: K at +2s*kKVBytes, V after it
  static constexpr int kOffBar = kOffKV + kStages * 2 * kKVBytes;
  static constexpr int kSmemBytes = kOffBar + 512;
  static constexpr int kThreads = 320;
  static constexpr int kTmemCols = 512;
  // TMEM columns of query tile i, from 256 i: S [0, kBN), P [kBN, kBN + kBN / 2) (16-bit
  // pairs), O [256 - D, 256); at D=128 with 128-key tiles P is aliased onto S [0, 64)
  // (S(j+1) is then issued only after PV(j), which reads P, in the MMA thread's
  // in-order pipeline).
  static constexpr bool kAliasP = kBN + kBN / 2 > 256 - D;
  static constexpr int kColP = kAliasP ? 0 : kBN;
  static constexpr int kColO = 256 - D;
  static_assert(kBN == 64 || kBN == 128, "KV tile");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

struct PairBars {
  uint64_t q_full;
  uint64_t kv_full[8];
  uint64_t kv_empty[8];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t turn[2][4];  // exponent-phase hand-off between the two warps sharing an SM sub-partition
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

static_assert(sizeof(PairBars) <= 512, "barrier block exceeds its shared-memory slot");

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

template <typename T, int HD>
__global__ void __launch_bounds__(320, 1)
prefill_pair_kernel(const __grid_constant__ CUtensorMap tmap_q,
                    const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v,
                    const __grid_constant__ CUtensorMap tmap_k8,
                    const __grid_constant__ CUtensorMap tmap_v8, T* __restrict__ out,
                    const int32_t* __restrict__ bt, int64_t bt_stride,
                    const int32_t* __restrict__ cu_seqlens_q,
                    const int32_t* __restrict__ seq_lens_k, int H, int group, int num_blocks,
                    int max_blocks, float scale_log2, int run8_ok, int n_split,
                    float* __restrict__ part_o, float2* __restrict__ part_ml, int* status,
                    uint64_t wait_limit, int starve) {
  using Cfg = PairCfg<HD>;
  constexpr int D = Cfg::D;
  constexpr int NS = Cfg::kStages;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescS = tc::idesc_f16(kBF16, 128, Cfg::kBN, false, false);
  constexpr uint32_t kIdescO = tc::idesc_f16(kBF16, 128, D, false, true);

  const int r = blockIdx.z;
  const int g = blockIdx.y;
  const int q_begin = cu_seqlens_q[r];
  const int nq = cu_seqlens_q[r + 1] - q_begin;
  const int tq = Cfg::kBM / group;
  // x = pair * n_split + split, pairs in reverse order (longest, last pairs first)
  const int npairs = int(gridDim.x) / n_split;
  const int pair = npairs - 1 - int(blockIdx.x) / n_split;
  const int split = int(blockIdx.x) % n_split;
  const int t0 = pair * 2 * tq;
  if (t0 >= nq) return;
  int Lk = seq_lens_k[r];
  if (Lk > max_blocks * kBS) {
    if (threadIdx.x == 0) flag_status(status, kStatusBadLength);
    Lk = max_blocks * kBS;
  }
  const int P = Lk - nq;
  if (P < 0) {
    if (threadIdx.x == 0) flag_status(status, kStatusBadLength);
    return;
  }
  const bool two = t0 + tq < nq;  // query tile 1 holds at least one token
  // KV tiles each query tile attends to (causal: tile 1 may need one more)
  const int n_kv0 = (P + min(t0 + tq, nq) + Cfg::kBN - 1) / Cfg::kBN;
  const int n_kv1 = two ? (P + min(t0 + 2 * tq, nq) + Cfg::kBN - 1) / Cfg::kBN : 0;
  const int n_kv = two ? n_kv1 : n_kv0;
  // This CTA's share of the KV tiles (split-KV): [j0, j1); query tile i attends to
  // cnt_i of them (tile 0 may end earlier under the causal mask).
  const int j0 = int(int64_t(split) * n_kv / n_split);
  const int j1 = int(int64_t(split + 1) * n_kv / n_split);
  const int cnt0 = max(0, min(j1, n_kv0) - j0);
  const int cnt1 = two ? max(0, min(j1, n_kv1) - j0) : 0;
  const int n_load = max(cnt0, cnt1);
  const int nblk_seq = (Lk + kBS - 1) / kBS;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) flag_status(status, kStatusWaitTimeout);
    return;
  }
  PairBars* bars = reinterpret_cast<PairBars*>(smem + Cfg::kOffBar);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 4);
      mbar_init(&bars->p_full[i], 4);
      mbar_init(&bars->pv_done[i], 1);
      for (int q = 0; q < 4; ++q) mbar_init(&bars->turn[i][q], 1);
    }
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
  const uint32_t sQ = smem_u32(smem + Cfg::kOffQ);
  const uint32_t sKV = smem_u32(smem + Cfg::kOffKV);

  int kv_issued = 0;  // producer warp: K/V tiles whose loads were issued
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // (starve != 0 is the test hook of as_debug_starve_next_launch: no loads at all,
    // so every wait on them runs out)
    if (!starve) {
    const int filler = (nblk_seq > 0) ? bt[int64_t(r) * bt_stride] : 0;
    const int fill_ok = (filler >= 0 && filler < num_blocks) ? filler : 0;
    if (lane == 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      tma_prefetch_desc(&tmap_k8);
      tma_prefetch_desc(&tmap_v8);
      mbar_arrive_expect_tx(&bars->q_full, (two ? 2 : 1) * Cfg::kQBytes);
      const uint64_t pol_q = l2_policy_evict_first();
      for (int qi = 0; qi < (two ? 2 : 1); ++qi)
        for (int sb = 0; sb < Cfg::kSub; ++sb)
          tma_load_3d(smem + Cfg::kOffQ + qi * Cfg::kQBytes + sb * Cfg::kSubBytes, &tmap_q,
                      &bars->q_full, sb * 64, g * group, q_begin + t0 + qi * tq, pol_q);
    }
    constexpr int NB = Cfg::kBlocks;  // paged blocks per KV tile
    auto load_id = [&](int jt) -> int {
      const int blk = NB * jt + (lane & (NB - 1));
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
    int id_next = load_id(j0);
    for (int j = 0; j < n_load; ++j) {  // local tile index; global tile j0 + j
      if (__any_sync(0xffffffffu, aborted(abort_flag))) break;
      const int st = j % NS;
      const bool ready = j < NS || mbar_wait(&bars->kv_empty[st], ((j / NS) + 1) & 1, status, wait_limit);
      if (!__all_sync(0xffffffffu, ready)) {
        *abort_flag = 1;
        break;
      }
      const int id = id_next;
      if (j + 1 < n_load) id_next = load_id(j0 + j + 1);
      const int id0 = __shfl_sync(0xffffffffu, id, 0);
      const bool run8 = run8_ok && __all_sync(0xffffffffu, id == id0 + (lane & (NB - 1)));
      if (lane == 0) mbar_arrive_expect_tx(&bars->kv_full[st], 2 * Cfg::kKVBytes);
      __syncwarp();
      uint8_t* kst = smem + Cfg::kOffKV + st * 2 * Cfg::kKVBytes;
      if (run8) {
        if (lane == 0) {
#pragma unroll
          for (int sb = 0; sb < Cfg::kSub; ++sb) {
            tma_load_4d(kst + sb * Cfg::kKVSubBytes, &tmap_k8, &bars->kv_full[st], sb * 64, g, 0,
                        id0, pol_kv);
            tma_load_4d(kst + Cfg::kKVBytes + sb * Cfg::kKVSubBytes, &tmap_v8,
                        &bars->kv_full[st], sb * 64, g, 0, id0, pol_kv);
          }
        }
      } else if (lane < NB) {
#pragma unroll
        for (int sb = 0; sb < Cfg::kSub; ++sb) {
          tma_load_4d(kst + sb * Cfg::kKVSubBytes + lane * 2048, &tmap_k, &bars->kv_full[st],
                      sb * 64, g, 0, id, pol_kv);
          tma_load_4d(kst + Cfg::kKVBytes + sb * Cfg::kKVSubBytes + lane * 2048, &tmap_v,
                      &bars->kv_full[st], sb * 64, g, 0, id, pol_kv);
        }
      }
      kv_issued = j + 1;
      __syncwarp();
    }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const int nk[2] = {cnt0, cnt1};  // local tile counts
      auto issue_s = [&](int i, int st) {
        const uint32_t q = sQ + i * Cfg::kQBytes;
        const uint32_t k = sKV + st * 2 * Cfg::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t oq = (kk >> 2) * Cfg::kSubBytes + (kk & 3) * 32;
          const uint32_t ok_ = (kk >> 2) * Cfg::kKVSubBytes + (kk & 3) * 32;
          tc::mma_f16(tmem + 256 * i, tc::sdesc_sw128(q + oq, 16, 1024),
                      tc::sdesc_sw128(k + ok_, 16, 1024), kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int i, int st, bool acc) {
        const uint32_t v = sKV + st * 2 * Cfg::kKVBytes + Cfg::kKVBytes;
        const uint32_t tP = tmem + 256 * i + Cfg::kColP;
        const uint32_t tO = tmem + 256 * i + Cfg::kColO;
#pragma unroll
        for (int kk = 0; kk < Cfg::kBN / 16; ++kk)
          tc::mma_f16_ts(tO, tP + kk * 8, tc::sdesc_sw128(v + kk * 2048, Cfg::kKVSubBytes, 1024),
                         kIdescO, (acc || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(&bars->q_full, 0, status, wait_limit);
      int js[2] = {0, 0};  // next S tile per query tile
      int jp[2] = {0, 0};  // next PV tile per query tile
      uint64_t t_idle = 0;  // start of the current stretch without progress
      uint32_t spin = 0;    // polls since the last issue
      while (ok && (jp[0] < nk[0] || jp[1] < nk[1])) {
        if (aborted(abort_flag)) break;
        bool did = false;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int j = js[i];
          // with P aliased onto S, S(j) may only follow PV(j-1), which reads P(j-1)
          if (j < nk[i] && (!Cfg::kAliasP || jp[i] >= j) &&
              mbar_try_wait(&bars->kv_full[j % NS], (j / NS) & 1) &&
              (j == 0 || mbar_try_wait(&bars->s_free[i], (j - 1) & 1))) {
            tc::fence_after_sync();
            issue_s(i, j % NS);
            tc::commit(&bars->s_full[i]);
            js[i] = j + 1;
            did = true;
          }
          const int jq = jp[i];
          if (jq < js[i] && mbar_try_wait(&bars->p_full[i], jq & 1)) {
            tc::fence_after_sync();
            issue_pv(i, jq % NS, jq > 0);
            tc::commit(&bars->pv_done[i]);
            jp[i] = jq + 1;
            did = true;
            // the stage is free once every query tile that reads it has issued PV
            const int o = 1 - i;
            if (jp[o] > jq || jq >= nk[o]) tc::commit(&bars->kv_empty[jq % NS]);
          }
        }
        if (did) {
          spin = 0;
        } else if ((++spin & 255u) == 0u) {  // the timer is slow to read: rarely
          const uint64_t now = global_timer_ns();
          if (spin == 256u) {
            t_idle = now;
          } else if (now - t_idle > wait_limit) {
            flag_status(status, kStatusWaitTimeout);
            ok = false;
          }
        }
      }
      if (!ok) *abort_flag = 1;
      tc::commit(&bars->drain);
      mbar_wait(&bars->drain, 0, status, wait_limit);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps
    const int i = (warp - 2) >> 2;  // query tile
    const int quad = warp & 3;      // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    const int t = row / group;
    const int hq = row - t * group;
    const int ti0 = t0 + i * tq;    // first token of this query tile
    const int tok = ti0 + t;
    const bool valid = tok < nq;
    const int qpos = valid ? P + tok : P + ti0;
    const uint32_t trow = uint32_t(quad * 32) << 16;
    const uint32_t tS = tmem + 256 * i + trow;
    const uint32_t tP = tS + Cfg::kColP;
    const uint32_t tO = tS + Cfg::kColO;
    const int nkv = i ? cnt1 : cnt0;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {  // local tile index; global tile j0 + j
      const bool go = !aborted(abort_flag) && mbar_wait(&bars->s_full[i], j & 1, status, wait_limit);
      if (!__all_sync(0xffffffffu, go)) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      constexpr int BN = Cfg::kBN;
      float x[BN];
      {
        uint32_t v[BN / 32][32];
#pragma unroll
        for (int u = 0; u < BN / 32; ++u) tc::ld_32x32b_x32(tS + 32 * u, v[u]);
        tc::wait_ld();
#pragma unroll
        for (int u = 0; u < BN / 32; ++u)
#pragma unroll
          for (int c = 0; c < 32; ++c) x[32 * u + c] = __uint_as_float(v[u][c]);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_free[i]);  // S(j+1) may overwrite S now

      const int lim = qpos - (j0 + j) * Cfg::kBN;  // keys c <= lim are visible
      if (lim < BN - 1) {
#pragma unroll
        for (int c = 0; c < BN; ++c) x[c] = (c <= lim) ? x[c] : -INFINITY;
      }
      float mp[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mp[c] = fmaxf(x[c], x[8 + c]);
#pragma unroll
      for (int c = 16; c < BN; c += 16) {
#pragma unroll
        for (int e = 0; e < 8; ++e) mp[e] = max3f(mp[e], x[c + e], x[c + 8 + e]);
      }
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      float alpha = 1.f;
      if (mx * scale_log2 > m + kLazySlack) {
        const float m_new = mx * scale_log2;
        alpha = fast_exp2(m - m_new);
        m = m_new;
      }
      // A row whose keys in this split are all masked so far keeps m = -inf; its
      // exponentials are then exp2(-inf) = 0 instead of NaN.
      const float neg_m = m == -INFINITY ? 0.f : -m;
      // Warp q of group 0 and warp q of group 1 run on the same SM sub-partition and
      // share its exponent unit: they take turns (tile j of group 0, tile j of group 1,
      // tile j+1 of group 0, ...), so one warp's TMEM traffic and waits overlap the
      // other's exponentials instead of both stalling together.  A warp waits only
      // for a hand-off its partner will make.
      const bool wait_turn = AS_PREFILL_PINGPONG && (i == 0 ? (j >= 1 && j - 1 < cnt1) : (j < cnt0));
      if (wait_turn) {
        const uint32_t par = (i == 0 ? (j - 1) : j) & 1;
        if (!__all_sync(0xffffffffu, !aborted(abort_flag) && mbar_wait(&bars->turn[i][quad], par, status, wait_limit))) {
          ok = false;
          break;
        }
      }
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
      const uint64_t nm2 = f2_pack(neg_m, neg_m);
      uint64_t sp2[4] = {0, 0, 0, 0};  // 8 independent fp32 partial sums, as pairs
      uint32_t pk[BN / 2];
      // the exponent-unit turn passes on after AS_PREFILL_HANDOFF of every 64 pairs
      constexpr int kHand = AS_PREFILL_HANDOFF * BN / 128;
#pragma unroll
      for (int c = 0; c < BN / 2; ++c) {
        const uint64_t xs = f2_fma(f2_pack(x[2 * c], x[2 * c + 1]), sc2, nm2);
        float a, b;
        f2_unpack(xs, a, b);
#if AS_PREFILL_POLY_EVERY > 0
        const uint64_t p2 = (c % AS_PREFILL_POLY_EVERY == AS_PREFILL_POLY_EVERY - 1)
                                ? exp2_poly_f2(xs)
                                : f2_pack(fast_exp2(a), fast_exp2(b));
#else
        const uint64_t p2 = f2_pack(fast_exp2(a), fast_exp2(b));
#endif
        sp2[c & 3] = f2_add(sp2[c & 3], p2);
        float p0, p1;
        f2_unpack(p2, p0, p1);
        pk[c] = pack2<T>(p0, p1);
        if (AS_PREFILL_PINGPONG && kHand < BN / 2 && c == kHand - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->turn[1 - i][quad]);
        }
      }
      float sum;
      {
        const uint64_t s01 = f2_add(f2_add(sp2[0], sp2[1]), f2_add(sp2[2], sp2[3]));
        float a, b;
        f2_unpack(s01, a, b);
        sum = a + b;
      }
      if (AS_PREFILL_PINGPONG && kHand >= BN / 2) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->turn[1 - i][quad]);
      }
      if (j > 0) {  // PV(j-1) still reads P and accumulates into O
        if (!__all_sync(0xffffffffu, mbar_wait(&bars->pv_done[i], (j - 1) & 1, status, wait_limit))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
      }
#pragma unroll
      for (int u = 0; u < BN / 64; ++u)
        tc::st_32x32b_x32(tP + 32 * u, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32 * u]));
      l = l * alpha + sum;
      if (j > 0 && __any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tc::ld_32x32b_x32(tO + c * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tc::st_32x32b_x32(tO + c * 32, o);
        }
      }
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[i]);
    }
    if (!ok) *abort_flag = 1;
    const bool done = ok && nkv > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[i], (nkv - 1) & 1, status, wait_limit));
    if (n_split > 1) {
      // split-KV partial: unnormalised O row, (m, l); merged by prefill_merge_kernel
      const int64_t rec = ((int64_t(r) * gridDim.y + g) * npairs + pair) * n_split + split;
      const int64_t prow = rec * 256 + i * 128 + row;
      if (done) {
        tc::fence_after_sync();
        float* po = part_o + prow * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tc::ld_32x32b_x32(tO + c * 32, o);
          tc::wait_ld();
          if (valid) {
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              *reinterpret_cast<uint4*>(po + c * 32 + e) = make_uint4(o[e], o[e + 1], o[e + 2], o[e + 3]);
          }
        }
        if (valid) part_ml[prow] = make_float2(m, l);
      } else if (ok && nkv == 0) {
        if (valid) part_ml[prow] = make_float2(-INFINITY, 0.f);  // no keys in this split
      } else if (ok) {
        *abort_flag = 1;
      }
    } else if (done) {
      tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* dst = out + (int64_t(q_begin) + tok) * int64_t(H) * D + int64_t(g * group + hq) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tc::ld_32x32b_x32(tO + c * 32, o);
        tc::wait_ld();
        if (valid) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            float f[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) f[u] = __uint_as_float(o[e + u]) * inv;
            *reinterpret_cast<uint4*>(dst + c * 32 + e) = pack8<T>(f);
          }
        }
      }
    } else if (ok && nkv > 0) {
      *abort_flag = 1;
    }
    tc::fence_before_sync();
  }

  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
  if (warp == 0 && lane == 0 && !starve && aborted(abort_flag)) {
    // A wait ran out somewhere: let the copies this CTA started land (bounded) before
    // its shared memory is released.  A stage already consumed completed long ago.
    mbar_wait(&bars->q_full, 0, status, wait_limit);
    for (int j = max(0, kv_issued - NS); j < kv_issued; ++j)
      mbar_wait(&bars->kv_full[j % NS], (j / NS) & 1, status, wait_limit);
  }
}

// Combines the n_split partials of every (query-tile pair, KV head, sequence):
// O = sum_s O_s 2^(m_s - M) / sum_s l_s 2^(m_s - M), M = max_s m_s.  One warp per row,
// two head-dim columns per lane.  Units and rows the main kernel skipped are skipped.
template <typename T, int HD>
__global__ void __launch_bounds__(256)
prefill_merge_kernel(T* __restrict__ out, const float* __restrict__ part_o,
                     const float2* __restrict__ part_ml, const int32_t* __restrict__ cu_seqlens_q,
                     const int32_t* __restrict__ seq_lens_k, int H, int group, int npairs,
                     int n_split, int max_blocks) {
  constexpr int D = HD;
  constexpr int kPer = D / 32;  // head-dim columns per lane
  const int r = blockIdx.z, g = blockIdx.y, pair = blockIdx.x;
  const int q_begin = cu_seqlens_q[r];
  const int nq = cu_seqlens_q[r + 1] - q_begin;
  const int tq = 128 / group;
  const int t0 = pair * 2 * tq;
  if (t0 >= nq) return;
  const int Lk = min(seq_lens_k[r], max_blocks * kBS);
  if (Lk - nq < 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rec0 = ((int64_t(r) * gridDim.y + g) * npairs + pair) * n_split;
  for (int rr = warp; rr < 256; rr += 8) {
    const int i = rr >> 7, row = rr & 127;
    const int tok = t0 + i * tq + row / group;
    if (tok >= nq) continue;
    const int hq = row % group;
    float M = -INFINITY;
    for (int sp = 0; sp < n_split; ++sp) {
      const float2 ml = part_ml[(rec0 + sp) * 256 + rr];
      if (ml.y > 0.f) M = fmaxf(M, ml.x);
    }
    float L = 0.f, acc[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) acc[e] = 0.f;
    for (int sp = 0; sp < n_split; ++sp) {
      const int64_t prow = (rec0 + sp) * 256 + rr;
      const float2 ml = part_ml[prow];
      if (!(ml.y > 0.f)) continue;
      const float w = fast_exp2(ml.x - M);
      const float* o = part_o + prow * D + kPer * lane;
      L = fmaf(ml.y, w, L);
#pragma unroll
      for (int e = 0; e < kPer; ++e) acc[e] = fmaf(o[e], w, acc[e]);
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    T* dst = out + (int64_t(q_begin) + tok) * int64_t(H) * D + int64_t(g * group + hq) * D +
             kPer * lane;
#pragma unroll
    for (int e = 0; e < kPer; e += 2)
      *reinterpret_cast<uint32_t*>(dst + e) = pack2<T>(acc[e] * inv, acc[e + 1] * inv);
  }
}

template <typename T>
CUtensorMapDataType tmap_dtype() {
  return std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

template <typename T, int HD>
int launch_pair(void* out, const void* q, int64_t q_stride, const void* k_cache,
                const void* v_cache, const int32_t* bt, int64_t bt_stride, const int32_t* cu,
                const int32_t* lk, int R, int max_seqlen_q, int total_q, int H, int Kh,
                int num_blocks, int max_blocks, float scale, int n_split, void* workspace,
                cudaStream_t stream) {
  using Cfg = PairCfg<HD>;
  constexpr int D = Cfg::D;
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
    // a whole KV tile of consecutive blocks in one box (the run fast path)
    const uint32_t box8[4] = {64, 1, uint32_t(kBS),
                              num_blocks >= Cfg::kBlocks ? uint32_t(Cfg::kBlocks) : 1u};
    int rc = encode_tensor_map(&mk, tmap_dtype<T>(), 4, const_cast<void*>(k_cache), dims, strides,
                               box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
      rc = encode_tensor_map(&mv, tmap_dtype<T>(), 4, const_cast<void*>(v_cache), dims, strides,
                             box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
      rc = encode_tensor_map(&mk8, tmap_dtype<T>(), 4, const_cast<void*>(k_cache), dims, strides,
                             box8, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
      rc = encode_tensor_map(&mv8, tmap_dtype<T>(), 4, const_cast<void*>(v_cache), dims, strides,
                             box8, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  auto kern = prefill_pair_kernel<T, HD>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  const int npairs = pair_count(max_seqlen_q, H, Kh);
  float2* part_ml = nullptr;
  float* part_o = nullptr;
  if (n_split > 1) {
    uint8_t* w = static_cast<uint8_t*>(workspace);
    const size_t rows = size_t(npairs) * Kh * R * n_split * 256;
    part_ml = reinterpret_cast<float2*>(w);
    part_o = reinterpret_cast<float*>(w + align256(rows * sizeof(float2)));
  }
  dim3 grid(npairs * n_split, Kh, R);
  kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(
      mq, mk, mv, mk8, mv8, static_cast<T*>(out), bt, bt_stride, cu, lk, H, group, num_blocks,
      max_blocks, scale * kLog2e, num_blocks >= Cfg::kBlocks ? 1 : 0, n_split, part_o, part_ml,
      device_status_ptr(), wait_limit_ns(), take_starve_flag(AS_KERNEL_PREFILL_ATTENTION) ? 1 : 0);
  int rc = check_launch("as_varlen_prefill_attention (tcgen05, query-tile pairs)");
  if (rc || n_split == 1) return rc;
  prefill_merge_kernel<T, HD><<<dim3(npairs, Kh, R), 256, 0, stream>>>(
      static_cast<T*>(out), part_o, part_ml, cu, lk, H, H / Kh, npairs, n_split, max_blocks);
  return check_launch("as_varlen_prefill_attention (split-KV merge)");
}

}  // namespace

int prefill_pair_splits(int R, int max_seqlen_q, int H, int Kh, int max_blocks, int requested) {
  if (requested > 0) return requested > kMaxSplits ? kMaxSplits : requested;
  // Split the KV range of each query-tile pair when too few CTAs (one per SM) would
  // otherwise run, e.g. a long cached prefix with a short new suffix.  Cost model:
  // waves * (KV tiles per CTA + a fixed per-CTA cost measured at ~14.5 tile times
  // on B200 (prologue, pipeline fill, epilogue, partial write and merge)); a split is
  // taken only when it is predicted 25% faster.
  constexpr double kCtaOverheadTiles = 14.5;
  const int units = pair_count(max_seqlen_q, H, Kh) * Kh * R;
  const int tiles = (max_blocks * kBS + 127) / 128;  // KV tiles of 128 keys
  const int slots = sm_count();
  int best = 1;
  double best_cost = 0.0;
  for (int sp = 1; sp <= kMaxSplits; ++sp) {
    if (sp > 1 && tiles < 4 * sp) break;
    const double waves = double((int64_t(units) * sp + slots - 1) / slots);
    const double cost = waves * (double(tiles) / sp + kCtaOverheadTiles);
    if (sp == 1 || cost < 0.75 * best_cost) {
      best = sp;
      best_cost = cost;
    }
  }
  return best;
}

size_t prefill_pair_workspace_size(int R, int max_seqlen_q, int H, int Kh, int D, int n_split) {
  if (n_split <= 1) return 0;
  const size_t rows = size_t(pair_count(max_seqlen_q, H, Kh)) * Kh * R * n_split * 256;
  return align256(rows * sizeof(float2)) + align256(rows * size_t(D) * sizeof(float));
}

int prefill_pair_launch(void* out, const void* q, int64_t q_stride, const void* k_cache,
                        const void* v_cache, const int32_t* bt, int64_t bt_stride,
                        const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int R,
                        int max_seqlen_q, int total_q, int H, int Kh, int D, int num_blocks,
                        int max_blocks, float scale, int dtype, int n_split, void* workspace,
                        cudaStream_t stream) {
#define AS_PAIR_LAUNCH(T, HD)                                                                    \
  launch_pair<T, HD>(out, q, q_stride, k_cache, v_cache, bt, bt_stride, cu_seqlens_q,            \
                     seq_lens_k, R, max_seqlen_q, total_q, H, Kh, num_blocks, max_blocks, scale, \
                     n_split, workspace, stream)
  if (dtype == AS_DTYPE_BF16)
    return D == 64 ? AS_PAIR_LAUNCH(__nv_bfloat16, 64) : AS_PAIR_LAUNCH(__nv_bfloat16, 128);
  return D == 64 ? AS_PAIR_LAUNCH(__half, 64) : AS_PAIR_LAUNCH(__half, 128);
#undef AS_PAIR_LAUNCH
}

namespace {
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

bool prefill_tc_supported(int dtype, int H, int Kh, int D, const void* q, int64_t q_stride,
                          const void* k_cache, const void* v_cache, const void* out) {
  if (dtype != AS_DTYPE_BF16 && dtype != AS_DTYPE_F16) return false;
  if (D != 64 && D != 128) return false;
  const int group = H / Kh;
  if (group < 1 || group > 128 || 128 % group != 0) return false;  // whole tokens per tile
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
  return prefill_pair_launch(out, q, q_stride, k_cache, v_cache, bt, bt_stride, cu_seqlens_q,
                             seq_lens_k, R, max_seqlen_q, total_q, H, Kh, D, num_blocks,
                             max_blocks, scale, dtype, n_split, workspace, stream);
}

}  // namespace asb
