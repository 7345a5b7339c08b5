// (3) Paged GQA split-K decode attention (flash-decoding over block tables).
//
// Replaces the reference decode attention: per request gather_kv -> pad to the
// longest sequence -> expand KV heads to H -> masked SDPA
// (agentserve/model/llama.py:419-469, agentserve/engine/cache.py:158-189) and the
// padded-list variant (llama.py:303-361).  Here every KV byte is read once, in
// place, from its paged block; the query heads of one GQA group share each tile.
//
// Fast path (bf16 / fp16, head_dim 64 or 128, block_size 16, group <= 8):
//   CTA = (split, kv head, sequence), 4 consumer warps + 1 TMA producer warp.
//   A stage holds 4 paged blocks (one per consumer warp) of K and V for this KV
//   head, loaded by cp.async.bulk.tensor into 128B-swizzled shared memory and
//   tracked by mbarriers (bounded waits).  Each warp computes S^T = K Q^T
//   (m16n8k16, tokens x heads), an online softmax in the fp32 accumulator
//   registers (per-head max/sum with three xor-shuffles), transposes P with
//   movmatrix and accumulates O^T += V^T P^T.  Warps are merged in shared memory;
//   splits are merged in-kernel by the last CTA of each (sequence, kv head),
//   found with an atomic counter that the same CTA resets (no spin-wait).
// Generic path (fp32, or other head dims / group sizes): CUDA-core warps with
//   the same online softmax, used for the fp32 parity configuration and the tiny
//   test geometry.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace asb {
namespace {

constexpr int kBlockSize = 16;
constexpr int kMaxGroup = 8;
constexpr int kMinAutoSplit = 32;  // smallest split chosen automatically (blocks_per_split 0)

// blocks_per_split == 0: about three waves of CTAs over the SMs (4 fast-path CTAs fit
// on an SM) for the largest possible batch (every sequence at max_blocks), never below
// kMinAutoSplit blocks per CTA.  Shorter splits cost a partial merge; longer ones
// leave SMs idle at the tail.
inline int auto_blocks_per_split(int B, int Kh, int max_blocks, bool fast) {
  const int64_t slots = int64_t(sm_count()) * (fast ? 4 : 8);
  int64_t bps = (int64_t(B) * Kh * max_blocks + 3 * slots - 1) / (3 * slots);
  if (bps < kMinAutoSplit) bps = kMinAutoSplit;
  if (bps > 256) bps = 256;
  return int(bps);
}

// ---------------------------------------------------------------------------
// Workspace layout for split-K partials.
// ---------------------------------------------------------------------------
struct DecodeWorkspace {
  int32_t* counters;  // [B * Kh]
  float* part_m;      // [B * H * max_splits]
  float* part_l;      // [B * H * max_splits]
  float* part_o;      // [B * H * max_splits * D]
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline size_t workspace_bytes(int B, int H, int Kh, int D, int max_splits) {
  size_t n = align_up(size_t(B) * Kh * sizeof(int32_t), 256);
  n += 2 * align_up(size_t(B) * H * max_splits * sizeof(float), 256);
  n += align_up(size_t(B) * H * max_splits * D * sizeof(float), 256);
  return n;
}

inline DecodeWorkspace carve_workspace(void* base, int B, int H, int Kh, int D, int max_splits) {
  uint8_t* p = static_cast<uint8_t*>(base);
  DecodeWorkspace ws;
  ws.counters = reinterpret_cast<int32_t*>(p);
  p += align_up(size_t(B) * Kh * sizeof(int32_t), 256);
  ws.part_m = reinterpret_cast<float*>(p);
  p += align_up(size_t(B) * H * max_splits * sizeof(float), 256);
  ws.part_l = reinterpret_cast<float*>(p);
  p += align_up(size_t(B) * H * max_splits * sizeof(float), 256);
  ws.part_o = reinterpret_cast<float*>(p);
  return ws;
}

// Merge `nparts` partial (m, l, o) triples of one (sequence, head) and write the
// normalised row.  m is in log2 units (scores were pre-multiplied by log2 e).
template <typename T>
__device__ __forceinline__ void write_row(T* out, float o, float l) {
  out[0] = Elem<T>::from_f32(l > 0.f ? o / l : 0.f);
}

// After this CTA's partial for (b, kv head g, split) is in the workspace, count
// arrivals; the last CTA merges all splits of the group's heads.  All threads
// of the CTA call this; returns after the merge (if any) is written.
template <typename T>
__device__ void splitk_finish(const DecodeWorkspace& ws, T* __restrict__ out, int b, int g, int H,
                              int Kh, int D, int group, int nsplit, int max_splits, int os_h,
                              int os_d) {
  __shared__ int s_last;
  // The barrier orders every thread's partial stores before thread 0's fence, which
  // (cumulatively) publishes them before the counter update; the last CTA's thread 0
  // fences again before the barrier that releases the merge reads.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(ws.counters + b * Kh + g, 1);
    s_last = (prev == nsplit - 1);
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  for (int idx = threadIdx.x; idx < group * D; idx += blockDim.x) {
    const int hl = idx / D;
    const int d = idx - hl * D;
    const int h = g * group + hl;
    const size_t base = (size_t(b) * H + h) * max_splits;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(ws.part_m + base + s));
    float L = 0.f, O = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float w = fast_exp2(__ldcg(ws.part_m + base + s) - M);
      L += w * __ldcg(ws.part_l + base + s);
      O += w * __ldcg(ws.part_o + (base + s) * D + d);
    }
    write_row<T>(out + size_t(b) * H * D + h * os_h + d * os_d, O, L);
  }
  if (threadIdx.x == 0) ws.counters[b * Kh + g] = 0;  // ready for the next call
}

// Fold n <= G paged blocks of one sequence at once (G independent S^T accumulator
// chains for instruction-level parallelism).  Block k's K/V tiles are at kb[k]/vb[k]
// and its first token at tok0 + k*tok_step.  The running max is lazy: scores are
// exponentiated against the current max m_run unless some score exceeds it by more
// than 2^8 (one warp vote); only then is the max reduced across the 8 lanes that
// share a head column and O, l rescaled.  p stays <= 256, well inside bf16/fp32
// range, and l, O, m stay mutually consistent, so the result is unchanged.
constexpr float kLazyMaxSlack = 8.0f;  // log2 units

template <typename T, int D, int G>
__device__ __forceinline__ void fold_blocks(const uint32_t (&kb)[G], const uint32_t (&vb)[G], int n,
                                            const uint32_t (&qb)[D / 16][2], int tok0,
                                            int tok_step, int seq_len, float scale_log2,
                                            float (&m_run)[2], float (&l_run)[2],
                                            float (&o_acc)[D / 16][4], int lane,
                                            uint32_t sub_bytes) {
  constexpr int KT = D / 16;
  float sc[G][4];
#pragma unroll
  for (int k = 0; k < G; ++k) sc[k][0] = sc[k][1] = sc[k][2] = sc[k][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < KT; ++kk) {
    const int mi = lane >> 3;
    const int row = (lane & 7) + 8 * (mi & 1);
    const int chunk = 2 * (kk & 3) + (mi >> 1);
    const uint32_t off = (kk >> 2) * sub_bytes + row * 128 + ((chunk ^ (row & 7)) << 4);
#pragma unroll
    for (int k = 0; k < G; ++k) {
      if (k < n) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(kb[k] + off, a0, a1, a2, a3);
        mma_16816<T>(sc[k], a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
    }
  }
  const int gq = lane >> 2;
  float lm0 = -INFINITY, lm1 = -INFINITY;
#pragma unroll
  for (int k = 0; k < G; ++k) {
    const int t = tok0 + k * tok_step + gq;
    const bool v0 = k < n && t < seq_len;
    const bool v1 = k < n && t + 8 < seq_len;
    sc[k][0] = v0 ? sc[k][0] * scale_log2 : -INFINITY;
    sc[k][1] = v0 ? sc[k][1] * scale_log2 : -INFINITY;
    sc[k][2] = v1 ? sc[k][2] * scale_log2 : -INFINITY;
    sc[k][3] = v1 ? sc[k][3] * scale_log2 : -INFINITY;
    lm0 = fmaxf(lm0, fmaxf(sc[k][0], sc[k][2]));
    lm1 = fmaxf(lm1, fmaxf(sc[k][1], sc[k][3]));
  }
  const bool grow = lm0 > m_run[0] + kLazyMaxSlack || lm1 > m_run[1] + kLazyMaxSlack;
  if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      lm0 = fmaxf(lm0, __shfl_xor_sync(0xffffffffu, lm0, o));
      lm1 = fmaxf(lm1, __shfl_xor_sync(0xffffffffu, lm1, o));
    }
    const float mn0 = fmaxf(m_run[0], lm0), mn1 = fmaxf(m_run[1], lm1);
    const float al0 = fast_exp2(m_run[0] - mn0), al1 = fast_exp2(m_run[1] - mn1);
    m_run[0] = mn0;
    m_run[1] = mn1;
    l_run[0] *= al0;
    l_run[1] *= al1;
#pragma unroll
    for (int mt = 0; mt < KT; ++mt) {
      o_acc[mt][0] *= al0;
      o_acc[mt][1] *= al1;
      o_acc[mt][2] *= al0;
      o_acc[mt][3] *= al1;
    }
  }
#pragma unroll
  for (int k = 0; k < G; ++k) {
    if (k < n) {
      const float p0 = fast_exp2(sc[k][0] - m_run[0]), p1 = fast_exp2(sc[k][1] - m_run[1]);
      const float p2 = fast_exp2(sc[k][2] - m_run[0]), p3 = fast_exp2(sc[k][3] - m_run[1]);
      l_run[0] += p0 + p2;
      l_run[1] += p1 + p3;
      const uint32_t pb0 = movmatrix_trans(pack2<T>(p0, p1));
      const uint32_t pb1 = movmatrix_trans(pack2<T>(p2, p3));
#pragma unroll
      for (int mt = 0; mt < KT; ++mt) {
        const int mi = lane >> 3;
        const int row = (lane & 7) + 8 * (mi >> 1);
        const int chunk = 2 * (mt & 3) + (mi & 1);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(vb[k] + (mt >> 2) * sub_bytes + row * 128 + ((chunk ^ (row & 7)) << 4),
                          a0, a1, a2, a3);
        mma_16816<T>(o_acc[mt], a0, a1, a2, a3, pb0, pb1);
      }
    }
  }
}

// Q^T of the GQA group of KV head g as B-fragments of S^T = K Q^T: column n = query
// head g*group + n (zero columns past the group).
template <typename T, int D>
__device__ __forceinline__ void load_q_frags(uint32_t (&qb)[D / 16][2], const T* __restrict__ q,
                                             int64_t q_stride, int b, int g, int group, int lane) {
  const int gq = lane >> 2, tq = lane & 3;
  const bool has_head = gq < group;
  const T* qrow = q + int64_t(b) * q_stride + int64_t(g * group + (has_head ? gq : 0)) * D;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    qb[kk][0] = has_head ? *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * tq) : 0u;
    qb[kk][1] = has_head ? *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * tq + 8) : 0u;
  }
}

// The decode step's new token, for the variant that also does the RoPE + cache write
// of that token (as_rope_paged_decode_attention): unrotated q / k / v rows, their
// position and pool slot, the fp32 cos||sin table and the pool planes.
template <typename T>
struct NewToken {
  const T* q;
  int64_t q_stride;
  const T* k;
  int64_t k_stride;
  const T* v;
  int64_t v_stride;
  const int64_t* positions;
  const int64_t* slot_mapping;
  const float* cos_sin;
  int table_len;
  T* k_cache;
  T* v_cache;
  int64_t num_slots;
};

// Rotate-half RoPE of element d of one head row x (llama.py:80-99), each product and
// the sum / difference rounded on its own in fp32 as torch evaluates it, so the
// result has the bits of the separate RoPE kernel's.
template <typename T, int D>
__device__ __forceinline__ float rope_elem(const T* __restrict__ x, const float* __restrict__ cs,
                                           int d) {
  constexpr int half = D / 2;
  const int j = d < half ? d : d - half;
  const float a = Elem<T>::to_f32(x[j]);
  const float b = Elem<T>::to_f32(x[j + half]);
  const float c = __ldg(cs + j), sn = __ldg(cs + half + j);
  return d < half ? __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn))
                  : __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, sn));
}

// load_q_frags for an unrotated q: each element is rotated for the token's position on
// the way in (a position outside the table leaves q as it is, as the RoPE kernel does).
template <typename T, int D>
__device__ __forceinline__ void load_q_frags_rope(uint32_t (&qb)[D / 16][2], const NewToken<T>& nt,
                                                  int b, int g, int group, int lane) {
  const int gq = lane >> 2, tq = lane & 3;
  const bool has_head = gq < group;
  const T* qrow = nt.q + int64_t(b) * nt.q_stride + int64_t(g * group + (has_head ? gq : 0)) * D;
  const int64_t pos = nt.positions[b];
  const bool rot = pos >= 0 && pos < nt.table_len;
  const float* cs = nt.cos_sin + (rot ? pos : 0) * int64_t(D);
  auto val = [&](int d) -> float {
    return rot ? rope_elem<T, D>(qrow, cs, d) : Elem<T>::to_f32(qrow[d]);
  };
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int e = 16 * kk + 2 * tq;
    qb[kk][0] = has_head ? pack2<T>(val(e), val(e + 1)) : 0u;
    qb[kk][1] = has_head ? pack2<T>(val(e + 8), val(e + 9)) : 0u;
  }
}

// The new token's rotated k and its v into pool slot slot_mapping[b] for KV head g, by
// one warp; the async-proxy fence makes the stores visible to the TMA loads that
// follow.  A bad position skips the token (flagged), a slot past the pool is flagged
// and skipped, a negative slot skipped silently: as the RoPE kernel does.
template <typename T, int D>
__device__ __forceinline__ void write_new_token(const NewToken<T>& nt, int b, int g, int Kh,
                                                int lane, int* status) {
  constexpr int half = D / 2;
  const int64_t pos = nt.positions[b];
  if (pos < 0 || pos >= nt.table_len) {
    if (lane == 0 && g == 0) flag_status(status, kStatusBadPosition);
    return;
  }
  const int64_t slot = nt.slot_mapping[b];
  if (slot < 0 || slot >= nt.num_slots) {
    if (slot >= nt.num_slots && lane == 0 && g == 0) flag_status(status, kStatusBadSlot);
    return;
  }
  const T* kr = nt.k + int64_t(b) * nt.k_stride + int64_t(g) * D;
  const T* vr = nt.v + int64_t(b) * nt.v_stride + int64_t(g) * D;
  T* kd = nt.k_cache + (slot * Kh + g) * int64_t(D);
  T* vd = nt.v_cache + (slot * Kh + g) * int64_t(D);
  const float* cs = nt.cos_sin + pos * int64_t(D);
#pragma unroll
  for (int j = lane; j < half; j += 32) {
    kd[j] = Elem<T>::from_f32(rope_elem<T, D>(kr, cs, j));
    kd[j + half] = Elem<T>::from_f32(rope_elem<T, D>(kr, cs, j + half));
    vd[j] = vr[j];
    vd[j + half] = vr[j + half];
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ===========================================================================
// Fast path: TMA + mma.sync, bf16/fp16, D in {64, 128}
// ===========================================================================
#ifndef AS_DECODE_SPLIT_WARPS
#define AS_DECODE_SPLIT_WARPS 4
#endif
#ifndef AS_DECODE_SPLIT_STAGES_D64
#define AS_DECODE_SPLIT_STAGES_D64 3
#endif
#ifndef AS_DECODE_SPLIT_STAGES_D128
#define AS_DECODE_SPLIT_STAGES_D128 2
#endif
#ifndef AS_DECODE_SPLIT_FOLD
#define AS_DECODE_SPLIT_FOLD 1
#endif

template <int D>
struct FastCfg {
  static constexpr int kConsumerWarps = AS_DECODE_SPLIT_WARPS;
  static constexpr int kFold = AS_DECODE_SPLIT_FOLD;  // blocks a warp folds per stage
  static constexpr int kThreads = (kConsumerWarps + 1) * 32;
  static constexpr int kSubTiles = D / 64;                 // 128-byte-wide swizzle sub-tiles
  static constexpr int kSubTileBytes = kBlockSize * 128;   // 16 rows x 128 B
  static constexpr int kTileBytes = kSubTiles * kSubTileBytes;  // one block, one head, K or V
  static constexpr int kSlotBytes = 2 * kTileBytes;        // K + V
  static constexpr int kStageBytes = kConsumerWarps * kFold * kSlotBytes;
  static constexpr int kStages = D == 64 ? AS_DECODE_SPLIT_STAGES_D64 : AS_DECODE_SPLIT_STAGES_D128;
  static constexpr int kMaxBlocksPerSplit = 256;
  static constexpr int kSmemBytes =
      1024 /*alignment slack*/ + kStages * kStageBytes + 2 * kStages * 8 +
      kMaxBlocksPerSplit * 4;
};

// kNewToken: q arrives unrotated and this kernel also does the new token's RoPE and
// cache write (nt); otherwise q is already rotated and the token already in the pool.
template <typename T, int D, bool kNewToken>
__global__ void __launch_bounds__(FastCfg<D>::kThreads)
decode_fast_kernel(const __grid_constant__ CUtensorMap tmap_k,
                   const __grid_constant__ CUtensorMap tmap_v, T* __restrict__ out,
                   const T* __restrict__ q, int64_t q_stride, const int32_t* __restrict__ bt,
                   int64_t bt_stride, const int32_t* __restrict__ seq_lens_k, int H, int Kh,
                   int group, int num_blocks, int max_blocks, float scale_log2, int bps,
                   int max_splits, int os_h, int os_d, DecodeWorkspace ws, int* status,
                   uint64_t wait_limit, int starve, const __grid_constant__ NewToken<T> nt) {
  using Cfg = FastCfg<D>;
  constexpr int NS = Cfg::kStages;
  constexpr int KT = D / 16;  // k-steps of QK^T == m-tiles of O^T
  pdl_wait();  // programmatic launch: q and the new token's K/V come from the kernel before
  pdl_trigger();

  const int split = blockIdx.x;
  const int g = blockIdx.y;
  const int b = blockIdx.z;

  int seq_len = seq_lens_k[b];
  int nblk = (seq_len + kBlockSize - 1) / kBlockSize;
  if (nblk > max_blocks) {
    if (threadIdx.x == 0 && split == 0 && g == 0) flag_status(status, kStatusBadLength);
    nblk = max_blocks;
    seq_len = max_blocks * kBlockSize;
  }
  const int nsplit = (nblk + bps - 1) / bps;
  if (seq_len <= 0) {
    if (split == 0) {
      for (int idx = threadIdx.x; idx < group * D; idx += blockDim.x)
        out[size_t(b) * H * D + (g * group + idx / D) * os_h + (idx % D) * os_d] =
            Elem<T>::from_f32(0.f);
    }
    return;
  }
  if (split >= nsplit) return;
  const int blk_begin = split * bps;
  const int blk_count = min(bps, nblk - blk_begin);
  constexpr int kPerStage = Cfg::kConsumerWarps * Cfg::kFold;
  const int niter = (blk_count + kPerStage - 1) / kPerStage;

  extern __shared__ uint8_t smem_raw[];
  // 128B-swizzled TMA tiles need 1024-byte alignment in the shared window.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* stages = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + NS * Cfg::kStageBytes);
  uint64_t* empty_bar = full_bar + NS;
  int32_t* s_blk = reinterpret_cast<int32_t*>(empty_bar + NS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Block ids of this split, validated once.
  for (int i = threadIdx.x; i < blk_count; i += blockDim.x) {
    int id = bt[int64_t(b) * bt_stride + blk_begin + i];
    if (id < 0 || id >= num_blocks) {
      flag_status(status, kStatusBadBlockId);
      id = 0;  // keep the TMA in bounds; the result for this sequence is garbage
    }
    s_blk[i] = id;
  }
  // Set by any thread whose wait ran out; read by all after the barrier that ends the
  // main loop (a static __shared__ word, outside the stage buffers TMA writes to).
  __shared__ int s_timeout;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], Cfg::kConsumerWarps);
    }
    s_timeout = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  int issued = 0;  // producer lane 0: stages whose loads were issued

  if (warp == Cfg::kConsumerWarps) {
    // ------------------------------ producer ------------------------------
    // The split holding the sequence's last block writes the new token first (the
    // other splits never read that slot).
    if (kNewToken && split == nsplit - 1) {
      write_new_token<T, D>(nt, b, g, Kh, lane, status);
      __syncwarp();
      if (lane == 0) asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    // starve != 0 (test hook only): issue nothing, so the consumers' waits run out.
    if (lane == 0 && !starve) {
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
      const uint64_t policy = l2_policy_evict_first();
      for (int it = 0; it < niter; ++it) {
        const int st = it % NS;
        if (it >= NS) {
          if (!mbar_wait(&empty_bar[st], ((it / NS) + 1) & 1, status, wait_limit)) {
            s_timeout = 1;
            break;
          }
        }
        const int nb = min(kPerStage, blk_count - it * kPerStage);
        mbar_arrive_expect_tx(&full_bar[st], uint32_t(nb * Cfg::kSlotBytes));
        uint8_t* stage = stages + st * Cfg::kStageBytes;
        for (int j = 0; j < nb; ++j) {
          const int blk = s_blk[it * kPerStage + j];
          uint8_t* slot = stage + j * Cfg::kSlotBytes;
#pragma unroll
          for (int sub = 0; sub < Cfg::kSubTiles; ++sub) {
            tma_load_4d(slot + sub * Cfg::kSubTileBytes, &tmap_k, &full_bar[st], sub * 64, g, 0,
                        blk, policy);
            tma_load_4d(slot + Cfg::kTileBytes + sub * Cfg::kSubTileBytes, &tmap_v,
                        &full_bar[st], sub * 64, g, 0, blk, policy);
          }
        }
        issued = it + 1;
      }
    }
  }

  // ------------------------------- consumers -------------------------------
  const int gq = lane >> 2;  // fragment row group
  const int tq = lane & 3;   // fragment column pair
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  float o_acc[KT][4];
#pragma unroll
  for (int i = 0; i < KT; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;

  if (warp < Cfg::kConsumerWarps) {
    uint32_t qb[KT][2];
    if (kNewToken)
      load_q_frags_rope<T, D>(qb, nt, b, g, group, lane);
    else
      load_q_frags<T, D>(qb, q, q_stride, b, g, group, lane);

    for (int it = 0; it < niter; ++it) {
      const int st = it % NS;
      const int local = it * kPerStage + warp * Cfg::kFold;  // this warp's first block
      const int n = min(Cfg::kFold, blk_count - local);       // < 1 only in the last stage
      if (n > 0) {
        // warp-uniform: the fold below is full-warp mma / shuffle code
        if (!__all_sync(0xffffffffu, mbar_wait(&full_bar[st], (it / NS) & 1, status,
                                                wait_limit))) {
          s_timeout = 1;
          break;
        }
        uint32_t kb[Cfg::kFold], vb[Cfg::kFold];
#pragma unroll
        for (int k = 0; k < Cfg::kFold; ++k) {
          kb[k] = smem_u32(stages + st * Cfg::kStageBytes +
                           (warp * Cfg::kFold + k) * Cfg::kSlotBytes);
          vb[k] = kb[k] + Cfg::kTileBytes;
        }
        fold_blocks<T, D, Cfg::kFold>(kb, vb, n, qb, (blk_begin + local) * kBlockSize,
                                      kBlockSize, seq_len, scale_log2, m_run, l_run, o_acc, lane,
                                      Cfg::kSubTileBytes);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[st]);
    }
    // per-head sums over the 8 lanes sharing a head column
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], o);
      l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], o);
    }
  }

  __syncthreads();
  const size_t part_base = (size_t(b) * H + g * group) * max_splits + split;
  if (s_timeout) {
    // A wait ran out (status bit 4 is set).  Loads may still be landing in the stage
    // buffers, so the shared-memory merge below is skipped: the producer waits (bounded)
    // for the stages it issued that were not consumed, and this CTA contributes an
    // empty partial (or a zero row) so the split-K counter protocol still completes
    // and leaves the counters at zero for the next call.
    if (warp == Cfg::kConsumerWarps && lane == 0) {
      for (int it = max(0, issued - NS); it < issued; ++it)
        mbar_wait(&full_bar[it % NS], (it / NS) & 1, status, wait_limit);
    }
    for (int idx = threadIdx.x; idx < group * D; idx += blockDim.x) {
      const int hl = idx / D;
      const int d = idx - hl * D;
      if (nsplit == 1) {
        write_row<T>(out + size_t(b) * H * D + (g * group + hl) * os_h + d * os_d, 0.f, 0.f);
      } else {
        const size_t pi = part_base + size_t(hl) * max_splits;
        ws.part_o[pi * D + d] = 0.f;
        if (d == 0) {
          ws.part_m[pi] = -INFINITY;
          ws.part_l[pi] = 0.f;
        }
      }
    }
    if (nsplit > 1)
      splitk_finish<T>(ws, out, b, g, H, Kh, D, group, nsplit, max_splits, os_h, os_d);
    return;
  }

  // ---------------------------- merge the warps -----------------------------
  // Every load issued was consumed (no wait ran out): the stage buffers are free.
  float* red_o = reinterpret_cast<float*>(smem);                      // [4][8][D]
  float* red_m = red_o + Cfg::kConsumerWarps * kMaxGroup * D;          // [4][8]
  float* red_l = red_m + Cfg::kConsumerWarps * kMaxGroup;              // [4][8]
  if (warp < Cfg::kConsumerWarps) {
    float* ow = red_o + warp * kMaxGroup * D;
#pragma unroll
    for (int mt = 0; mt < KT; ++mt) {
      const int d0 = 16 * mt + gq;
      ow[(2 * tq) * D + d0] = o_acc[mt][0];
      ow[(2 * tq + 1) * D + d0] = o_acc[mt][1];
      ow[(2 * tq) * D + d0 + 8] = o_acc[mt][2];
      ow[(2 * tq + 1) * D + d0 + 8] = o_acc[mt][3];
    }
    if (gq == 0) {
      red_m[warp * kMaxGroup + 2 * tq] = m_run[0];
      red_m[warp * kMaxGroup + 2 * tq + 1] = m_run[1];
      red_l[warp * kMaxGroup + 2 * tq] = l_run[0];
      red_l[warp * kMaxGroup + 2 * tq + 1] = l_run[1];
    }
  }
  __syncthreads();

  for (int idx = threadIdx.x; idx < group * D; idx += blockDim.x) {
    const int hl = idx / D;
    const int d = idx - hl * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < Cfg::kConsumerWarps; ++w) M = fmaxf(M, red_m[w * kMaxGroup + hl]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < Cfg::kConsumerWarps; ++w) {
        const float wt = fast_exp2(red_m[w * kMaxGroup + hl] - M);
        L += wt * red_l[w * kMaxGroup + hl];
        O += wt * red_o[(w * kMaxGroup + hl) * D + d];
      }
    }
    if (nsplit == 1) {
      write_row<T>(out + size_t(b) * H * D + (g * group + hl) * os_h + d * os_d, O, L);
    } else {
      const size_t pi = part_base + size_t(hl) * max_splits;
      ws.part_o[pi * D + d] = O;
      if (d == 0) {
        ws.part_m[pi] = M;
        ws.part_l[pi] = L;
      }
    }
  }
  if (nsplit > 1)
    splitk_finish<T>(ws, out, b, g, H, Kh, D, group, nsplit, max_splits, os_h, os_d);
}

// ===========================================================================
// Generic path: CUDA cores, any dtype, D <= 256 and a multiple of 32 / 2.
// CTA = (split, query head, sequence), 4 warps over interleaved tokens.
// ===========================================================================
constexpr int kGenWarps = 4;

template <typename T, int EPL>  // EPL = elements of the head vector per lane
__global__ void __launch_bounds__(kGenWarps * 32)
decode_generic_kernel(T* __restrict__ out, const T* __restrict__ q, int64_t q_stride,
                      const T* __restrict__ k_cache, const T* __restrict__ v_cache,
                      const int32_t* __restrict__ bt, int64_t bt_stride,
                      const int32_t* __restrict__ seq_lens_k, int H, int Kh, int D, int group,
                      int num_blocks, int max_blocks, float scale, int bps, int max_splits,
                      int os_h, int os_d, DecodeWorkspace ws, int* status) {
  const int split = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int g = h / group;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  int seq_len = seq_lens_k[b];
  int nblk = (seq_len + kBlockSize - 1) / kBlockSize;
  if (nblk > max_blocks) {
    if (threadIdx.x == 0 && split == 0 && h == 0) flag_status(status, kStatusBadLength);
    nblk = max_blocks;
    seq_len = max_blocks * kBlockSize;
  }
  const int nsplit = (nblk + bps - 1) / bps;
  if (seq_len <= 0) {
    if (split == 0)
      for (int d = threadIdx.x; d < D; d += blockDim.x)
        out[size_t(b) * H * D + h * os_h + d * os_d] = Elem<T>::from_f32(0.f);
    return;
  }
  if (split >= nsplit) return;
  const int tok_begin = split * bps * kBlockSize;
  const int tok_end = min(seq_len, tok_begin + bps * kBlockSize);

  float qv[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const int d = lane + 32 * e;
    qv[e] = d < D ? Elem<T>::to_f32(q[int64_t(b) * q_stride + int64_t(h) * D + d]) : 0.f;
  }
  float m = -INFINITY, l = 0.f, o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) o[e] = 0.f;

  for (int t = tok_begin + warp; t < tok_end; t += kGenWarps) {
    int blk = bt[int64_t(b) * bt_stride + t / kBlockSize];
    if (blk < 0 || blk >= num_blocks) {
      if (lane == 0) flag_status(status, kStatusBadBlockId);
      continue;
    }
    const int64_t row = (int64_t(blk) * kBlockSize + t % kBlockSize) * Kh + g;
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
  const size_t pi = (size_t(b) * H + h) * max_splits + split;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < kGenWarps; ++w) {
        const float wt = expf(red_m[w] - M);
        L += wt * red_l[w];
        O += wt * red_o[w][d];
      }
    }
    if (nsplit == 1) {
      write_row<T>(out + size_t(b) * H * D + h * os_h + d * os_d, O, L);
    } else {
      // store in log2 units so the shared merge (exp2) applies
      ws.part_o[pi * D + d] = O;
      if (d == 0) {
        ws.part_m[pi] = M * kLog2e;
        ws.part_l[pi] = L;
      }
    }
  }
  if (nsplit > 1) {
    // one CTA per query head here: count arrivals per (sequence, head)
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int prev = atomicAdd(ws.counters + b * H + h, 1);
      s_last = (prev == nsplit - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const size_t base = (size_t(b) * H + h) * max_splits;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float M2 = -INFINITY;
      for (int s = 0; s < nsplit; ++s) M2 = fmaxf(M2, __ldcg(ws.part_m + base + s));
      float L = 0.f, O = 0.f;
      for (int s = 0; s < nsplit; ++s) {
        const float w = exp2f(__ldcg(ws.part_m + base + s) - M2);
        L += w * __ldcg(ws.part_l + base + s);
        O += w * __ldcg(ws.part_o + (base + s) * D + d);
      }
      write_row<T>(out + size_t(b) * H * D + h * os_h + d * os_d, O, L);
    }
    if (threadIdx.x == 0) ws.counters[b * H + h] = 0;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <typename T>
CUtensorMapDataType tma_dtype();
template <>
CUtensorMapDataType tma_dtype<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }
template <>
CUtensorMapDataType tma_dtype<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }

// 4-D map over one layer's K or V plane [NB, 16, Kh, D] viewed innermost-first as
// (D, Kh, 16, NB); box = 64 elements (128 B, swizzled) x 1 head x 16 tokens x 1 block.
template <typename T>
int make_pool_map(CUtensorMap* map, const void* base, int Kh, int D, int num_blocks) {
  const uint64_t es = sizeof(T);
  const uint64_t dims[4] = {uint64_t(D), uint64_t(Kh), uint64_t(kBlockSize), uint64_t(num_blocks)};
  const uint64_t strides[3] = {D * es, uint64_t(Kh) * D * es, uint64_t(kBlockSize) * Kh * D * es};
  const uint32_t box[4] = {64, 1, uint32_t(kBlockSize), 1};
  return encode_tensor_map(map, tma_dtype<T>(), 4, const_cast<void*>(base), dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, int D>
int launch_fast(T* out, const T* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                const int32_t* bt, int64_t bt_stride, const int32_t* seq_lens_k, int B, int H,
                int Kh, int num_blocks, int max_blocks, float scale, int bps, int max_splits,
                int os_h, int os_d, DecodeWorkspace ws, cudaStream_t stream,
                const NewToken<T>* nt = nullptr) {
  using Cfg = FastCfg<D>;
  CUtensorMap mk, mv;
  int rc = make_pool_map<T>(&mk, k_cache, Kh, D, num_blocks);
  if (rc) return rc;
  rc = make_pool_map<T>(&mv, v_cache, Kh, D, num_blocks);
  if (rc) return rc;
  dim3 grid(max_splits, Kh, B);
  const int starve = take_starve_flag(AS_KERNEL_DECODE_ATTENTION) ? 1 : 0;
  if (nt) {
    auto kern = decode_fast_kernel<T, D, true>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    launch_pdl(kern, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, mk, mv, out, q,
               q_stride, bt, bt_stride, seq_lens_k, H, Kh, H / Kh, num_blocks, max_blocks,
               scale * kLog2e, bps, max_splits, os_h, os_d, ws, device_status_ptr(),
               wait_limit_ns(), starve, *nt);
    return check_launch("as_rope_paged_decode_attention");
  }
  auto kern = decode_fast_kernel<T, D, false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  NewToken<T> none{};
  launch_pdl(kern, grid, dim3(Cfg::kThreads), Cfg::kSmemBytes, stream, mk, mv, out, q, q_stride,
             bt, bt_stride, seq_lens_k, H, Kh, H / Kh, num_blocks, max_blocks, scale * kLog2e, bps,
             max_splits, os_h, os_d, ws, device_status_ptr(), wait_limit_ns(), starve, none);
  return check_launch("as_paged_decode_attention");
}

template <typename T>
int launch_generic(T* out, const T* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                   const int32_t* bt, int64_t bt_stride, const int32_t* seq_lens_k, int B, int H,
                   int Kh, int D, int num_blocks, int max_blocks, float scale, int bps,
                   int max_splits, int os_h, int os_d, DecodeWorkspace ws,
                   cudaStream_t stream) {
  dim3 grid(max_splits, H, B);
  const T* kc = static_cast<const T*>(k_cache);
  const T* vc = static_cast<const T*>(v_cache);
  int* st = device_status_ptr();
  if (D <= 32)
    decode_generic_kernel<T, 1><<<grid, kGenWarps * 32, 0, stream>>>(
        out, q, q_stride, kc, vc, bt, bt_stride, seq_lens_k, H, Kh, D, H / Kh, num_blocks,
        max_blocks, scale, bps, max_splits, os_h, os_d, ws, st);
  else if (D <= 64)
    decode_generic_kernel<T, 2><<<grid, kGenWarps * 32, 0, stream>>>(
        out, q, q_stride, kc, vc, bt, bt_stride, seq_lens_k, H, Kh, D, H / Kh, num_blocks,
        max_blocks, scale, bps, max_splits, os_h, os_d, ws, st);
  else if (D <= 128)
    decode_generic_kernel<T, 4><<<grid, kGenWarps * 32, 0, stream>>>(
        out, q, q_stride, kc, vc, bt, bt_stride, seq_lens_k, H, Kh, D, H / Kh, num_blocks,
        max_blocks, scale, bps, max_splits, os_h, os_d, ws, st);
  else
    decode_generic_kernel<T, 8><<<grid, kGenWarps * 32, 0, stream>>>(
        out, q, q_stride, kc, vc, bt, bt_stride, seq_lens_k, H, Kh, D, H / Kh, num_blocks,
        max_blocks, scale, bps, max_splits, os_h, os_d, ws, st);
  return check_launch("as_paged_decode_attention");
}

bool fast_path_ok(int dtype, int D, int group, const void* q, int64_t q_stride,
                  const void* k_cache, const void* v_cache) {
  if (dtype != AS_DTYPE_BF16 && dtype != AS_DTYPE_F16) return false;
  if (D != 64 && D != 128) return false;
  if (group > kMaxGroup) return false;
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (q_stride & 1)) return false;
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
    return false;
  return true;
}

}  // namespace
}  // namespace asb

using namespace asb;

extern "C" size_t as_paged_decode_workspace_size(int32_t num_seqs, int32_t num_heads,
                                                 int32_t num_kv_heads, int32_t head_dim,
                                                 int32_t max_blocks, int32_t blocks_per_split) {
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_blocks <= 0 ||
      blocks_per_split < 0 || num_heads % num_kv_heads)
    return 0;
  if (blocks_per_split == 0) blocks_per_split = kMinAutoSplit;  // covers every automatic choice
  const int max_splits = (max_blocks + blocks_per_split - 1) / blocks_per_split;
  // counters are per (sequence, query head) to cover both kernel variants
  return workspace_bytes(num_seqs, num_heads, num_heads, head_dim, max_splits);
}

namespace {
// Argument checks shared by both decode entry points (nothing here touches the GPU).
// Returns AS_OK when the call may proceed; num_seqs == 0 passes (nothing to do).
int check_decode_args(const char* who, const void* out, const void* q, int64_t q_stride,
                      const void* k_cache, const void* v_cache, const int32_t* block_tables,
                      int64_t bt_stride, const int32_t* seq_lens_k, int32_t num_seqs,
                      int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                      int32_t block_size, int32_t num_blocks, int32_t max_blocks,
                      int32_t blocks_per_split, int32_t out_layout, int32_t dtype) {
  if (!dtype_size(dtype)) return fail(AS_ERR_INVALID_ARG, "%s: unknown dtype", who);
  if (block_size != kBlockSize)
    return fail(AS_ERR_UNSUPPORTED, "%s: block_size must be 16 (got %d)", who, block_size);
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads ||
      head_dim <= 0 || head_dim > 256 || num_blocks <= 0 || max_blocks <= 0 ||
      bt_stride < max_blocks || blocks_per_split < 0)
    return fail(AS_ERR_INVALID_ARG, "%s: bad sizes (B=%d H=%d Kh=%d D=%d NB=%d maxb=%d bps=%d)",
                who, num_seqs, num_heads, num_kv_heads, head_dim, num_blocks, max_blocks,
                blocks_per_split);
  if (out_layout != AS_LAYOUT_HEAD_MAJOR && out_layout != AS_LAYOUT_DIM_MAJOR)
    return fail(AS_ERR_INVALID_ARG, "%s: unknown out_layout %d", who, out_layout);
  if (num_seqs == 0) return AS_OK;
  if (num_seqs > 65535) return fail(AS_ERR_INVALID_ARG, "%s: B > 65535", who);
  if (!out || !q || !k_cache || !v_cache || !block_tables || !seq_lens_k)
    return fail(AS_ERR_INVALID_ARG, "%s: null pointer", who);
  if (q_stride < int64_t(num_heads) * head_dim)
    return fail(AS_ERR_INVALID_ARG, "%s: q_stride < H*D", who);
  return AS_OK;
}
}  // namespace

extern "C" int as_paged_decode_attention(void* out, const void* q, int64_t q_stride,
                                         const void* k_cache, const void* v_cache,
                                         const int32_t* block_tables, int64_t bt_stride,
                                         const int32_t* seq_lens_k, int32_t num_seqs,
                                         int32_t num_heads, int32_t num_kv_heads,
                                         int32_t head_dim, int32_t block_size,
                                         int32_t num_blocks, int32_t max_blocks, float scale,
                                         int32_t blocks_per_split, void* workspace,
                                         size_t workspace_bytes_given, int32_t out_layout,
                                         int32_t dtype, as_stream_t stream) {
  const int rc0 = check_decode_args("as_paged_decode_attention", out, q, q_stride, k_cache,
                                    v_cache, block_tables, bt_stride, seq_lens_k, num_seqs,
                                    num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                                    max_blocks, blocks_per_split, out_layout, dtype);
  if (rc0 != AS_OK) return rc0;
  if (num_seqs == 0) return AS_OK;
  const int group = num_heads / num_kv_heads;
  const bool fast = fast_path_ok(dtype, head_dim, group, q, q_stride, k_cache, v_cache);
  if (blocks_per_split == 0)
    blocks_per_split = auto_blocks_per_split(num_seqs, num_kv_heads, max_blocks, fast);
  const int max_splits = (max_blocks + blocks_per_split - 1) / blocks_per_split;
  if (fast && blocks_per_split > FastCfg<64>::kMaxBlocksPerSplit)
    return fail(AS_ERR_INVALID_ARG, "as_paged_decode_attention: blocks_per_split > %d",
                FastCfg<64>::kMaxBlocksPerSplit);
  DecodeWorkspace ws{nullptr, nullptr, nullptr, nullptr};
  if (max_splits > 1) {
    const size_t need = workspace_bytes(num_seqs, num_heads, num_heads, head_dim, max_splits);
    if (!workspace || workspace_bytes_given < need)
      return fail(AS_ERR_WORKSPACE, "as_paged_decode_attention: workspace of %zu bytes needed",
                  need);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
      return fail(AS_ERR_INVALID_ARG, "as_paged_decode_attention: workspace must be 256-byte aligned");
    ws = carve_workspace(workspace, num_seqs, num_heads, num_heads, head_dim, max_splits);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int B = num_seqs, H = num_heads, Kh = num_kv_heads, D = head_dim;
  const int os_h = out_layout == AS_LAYOUT_HEAD_MAJOR ? D : 1;
  const int os_d = out_layout == AS_LAYOUT_HEAD_MAJOR ? 1 : H;
  if (fast) {
    if (dtype == AS_DTYPE_BF16) {
      using T = __nv_bfloat16;
      if (D == 64)
        return launch_fast<T, 64>(static_cast<T*>(out), static_cast<const T*>(q), q_stride,
                                  k_cache, v_cache, block_tables, bt_stride, seq_lens_k, B, H, Kh,
                                  num_blocks, max_blocks, scale, blocks_per_split, max_splits, os_h, os_d, ws, s);
      return launch_fast<T, 128>(static_cast<T*>(out), static_cast<const T*>(q), q_stride, k_cache,
                                 v_cache, block_tables, bt_stride, seq_lens_k, B, H, Kh,
                                 num_blocks, max_blocks, scale, blocks_per_split, max_splits, os_h, os_d, ws, s);
    } else {
      using T = __half;
      if (D == 64)
        return launch_fast<T, 64>(static_cast<T*>(out), static_cast<const T*>(q), q_stride,
                                  k_cache, v_cache, block_tables, bt_stride, seq_lens_k, B, H, Kh,
                                  num_blocks, max_blocks, scale, blocks_per_split, max_splits, os_h, os_d, ws, s);
      return launch_fast<T, 128>(static_cast<T*>(out), static_cast<const T*>(q), q_stride, k_cache,
                                 v_cache, block_tables, bt_stride, seq_lens_k, B, H, Kh,
                                 num_blocks, max_blocks, scale, blocks_per_split, max_splits, os_h, os_d, ws, s);
    }
  }
  switch (dtype) {
    case AS_DTYPE_F32:
      return launch_generic<float>(static_cast<float*>(out), static_cast<const float*>(q), q_stride,
                                   k_cache, v_cache, block_tables, bt_stride, seq_lens_k, B, H, Kh,
                                   D, num_blocks, max_blocks, scale, blocks_per_split, max_splits,
                                   os_h, os_d, ws, s);
    case AS_DTYPE_F16:
      return launch_generic<__half>(static_cast<__half*>(out), static_cast<const __half*>(q),
                                    q_stride, k_cache, v_cache, block_tables, bt_stride,
                                    seq_lens_k, B, H, Kh, D, num_blocks, max_blocks, scale,
                                    blocks_per_split, max_splits, os_h, os_d, ws, s);
    default:
      return launch_generic<__nv_bfloat16>(
          static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(q), q_stride,
          k_cache, v_cache, block_tables, bt_stride, seq_lens_k, B, H, Kh, D, num_blocks,
          max_blocks, scale, blocks_per_split, max_splits, os_h, os_d, ws, s);
  }
}

extern "C" int as_rope_paged_decode_attention(
    void* out, const void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
    int64_t v_stride, const int64_t* positions, const int64_t* slot_mapping,
    const float* cos_sin, int32_t table_len, void* k_cache, void* v_cache,
    const int32_t* block_tables, int64_t bt_stride, const int32_t* seq_lens_k, int32_t num_seqs,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int32_t num_blocks, int32_t max_blocks, float scale, int32_t blocks_per_split,
    void* workspace, size_t workspace_bytes_given, int32_t out_layout, int32_t dtype,
    as_stream_t stream) {
  const char* who = "as_rope_paged_decode_attention";
  const int rc0 = check_decode_args(who, out, q, q_stride, k_cache, v_cache, block_tables,
                                    bt_stride, seq_lens_k, num_seqs, num_heads, num_kv_heads,
                                    head_dim, block_size, num_blocks, max_blocks,
                                    blocks_per_split, out_layout, dtype);
  if (rc0 != AS_OK) return rc0;
  if (num_seqs == 0) return AS_OK;
  if (!k || !v || !positions || !slot_mapping || !cos_sin)
    return fail(AS_ERR_INVALID_ARG, "%s: null pointer", who);
  if (table_len <= 0 || k_stride < int64_t(num_kv_heads) * head_dim ||
      v_stride < int64_t(num_kv_heads) * head_dim)
    return fail(AS_ERR_INVALID_ARG, "%s: bad table length or k / v row stride", who);
  const int group = num_heads / num_kv_heads;
  if (!fast_path_ok(dtype, head_dim, group, q, q_stride, k_cache, v_cache))
    return fail(AS_ERR_UNSUPPORTED,
                "%s: needs bf16 / fp16, head_dim 64 or 128, at most 8 query heads per KV head "
                "and 4-byte aligned rows (use as_rope_reshape_and_cache + "
                "as_paged_decode_attention)", who);
  if (blocks_per_split == 0)
    blocks_per_split = auto_blocks_per_split(num_seqs, num_kv_heads, max_blocks, true);
  if (blocks_per_split > FastCfg<64>::kMaxBlocksPerSplit)
    return fail(AS_ERR_INVALID_ARG, "%s: blocks_per_split > %d", who,
                FastCfg<64>::kMaxBlocksPerSplit);
  const int max_splits = (max_blocks + blocks_per_split - 1) / blocks_per_split;
  DecodeWorkspace ws{nullptr, nullptr, nullptr, nullptr};
  if (max_splits > 1) {
    const size_t need = workspace_bytes(num_seqs, num_heads, num_heads, head_dim, max_splits);
    if (!workspace || workspace_bytes_given < need)
      return fail(AS_ERR_WORKSPACE, "%s: workspace of %zu bytes needed", who, need);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
      return fail(AS_ERR_INVALID_ARG, "%s: workspace must be 256-byte aligned", who);
    ws = carve_workspace(workspace, num_seqs, num_heads, num_heads, head_dim, max_splits);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int B = num_seqs, H = num_heads, Kh = num_kv_heads, D = head_dim;
  const int os_h = out_layout == AS_LAYOUT_HEAD_MAJOR ? D : 1;
  const int os_d = out_layout == AS_LAYOUT_HEAD_MAJOR ? 1 : H;
  const int64_t num_slots = int64_t(num_blocks) * kBlockSize;
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    NewToken<T> nt{static_cast<const T*>(q), q_stride, static_cast<const T*>(k), k_stride,
                   static_cast<const T*>(v), v_stride, positions, slot_mapping, cos_sin,
                   table_len, static_cast<T*>(k_cache), static_cast<T*>(v_cache), num_slots};
    if (D == 64)
      return launch_fast<T, 64>(static_cast<T*>(out), static_cast<const T*>(q), q_stride,
                                k_cache, v_cache, block_tables, bt_stride, seq_lens_k, B, H, Kh,
                                num_blocks, max_blocks, scale, blocks_per_split, max_splits,
                                os_h, os_d, ws, s, &nt);
    return launch_fast<T, 128>(static_cast<T*>(out), static_cast<const T*>(q), q_stride, k_cache,
                               v_cache, block_tables, bt_stride, seq_lens_k, B, H, Kh, num_blocks,
                               max_blocks, scale, blocks_per_split, max_splits, os_h, os_d, ws, s,
                               &nt);
  };
  return dtype == AS_DTYPE_BF16 ? run(__nv_bfloat16()) : run(__half());
}

// ===========================================================================
// Allocation-free variant: split-K scratch in a static device array.
//
// Some callers cannot call cudaMalloc or hand us a workspace: a host runtime
// whose device memory is entirely owned by another allocator (for example a
// framework caching allocator that reserved the GPU up front and has nothing to
// lend), or a serving loop that must never reach cudaMalloc's implicit device
// synchronisation.  They still own q, the pool and out, but have nowhere to get
// split-K scratch from.  This entry point uses a fixed-size array that lives in
// the library's own device memory instead (every GPU that loads the library
// holds AS_DECODE_NOALLOC_SCRATCH_BYTES of it until the process exits).
// ===========================================================================
static __device__ __align__(256) uint8_t g_decode_noalloc_scratch[AS_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoallocMaxDevices = 64;
// Filled once per device under g_noalloc_mu and read without the lock afterwards, so
// the slots are atomics (acquire load, release store).
std::atomic<void*> g_noalloc_scratch_ptr[kNoallocMaxDevices];
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device.  The first call on a
// device resolves it (cudaGetSymbolAddress with that device current) and caches it;
// in host code the array's name is only a host-side stand-in, never a device address.
int noalloc_scratch_on_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices)
    return fail(AS_ERR_CUDA, "as_paged_decode_attention_noalloc: no current device (%s)",
                cudaGetErrorString(e));
  void* p = g_noalloc_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    p = g_noalloc_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (!p) {
      e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return fail(AS_ERR_CUDA,
                    "as_paged_decode_attention_noalloc: cudaGetSymbolAddress failed: %s",
                    cudaGetErrorString(e));
      g_noalloc_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return AS_OK;
}
}  // namespace

extern "C" int as_paged_decode_attention_noalloc(
    void* out, const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
    const int32_t* block_tables, int64_t bt_stride, const int32_t* seq_lens_k, int32_t num_seqs,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int32_t num_blocks, int32_t max_blocks, float scale, int32_t blocks_per_split,
    int32_t out_layout, int32_t dtype, as_stream_t stream) {
  // Bad arguments are reported as such (AS_ERR_INVALID_ARG / AS_ERR_UNSUPPORTED) before
  // the scratch is looked at.
  const int rc0 = check_decode_args("as_paged_decode_attention_noalloc", out, q, q_stride,
                                    k_cache, v_cache, block_tables, bt_stride, seq_lens_k,
                                    num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                                    num_blocks, max_blocks, blocks_per_split, out_layout, dtype);
  if (rc0 != AS_OK) return rc0;
  if (num_seqs == 0) return AS_OK;
  // blocks_per_split == 0 (split chosen by the library) may use scratch
  const bool uses_scratch =
      blocks_per_split == 0 || (max_blocks + blocks_per_split - 1) / blocks_per_split > 1;
  void* scratch = nullptr;
  if (uses_scratch) {
    const size_t need = as_paged_decode_workspace_size(num_seqs, num_heads, num_kv_heads,
                                                       head_dim, max_blocks, blocks_per_split);
    if (need == 0 || need > size_t(AS_DECODE_NOALLOC_SCRATCH_BYTES))
      return fail(AS_ERR_WORKSPACE,
                  "as_paged_decode_attention_noalloc: this call needs %zu bytes of split-K "
                  "scratch but the static array holds %zu; use fewer sequences, a larger "
                  "blocks_per_split, or as_paged_decode_attention with your own workspace",
                  need, size_t(AS_DECODE_NOALLOC_SCRATCH_BYTES));
    int rc = noalloc_scratch_on_current_device(&scratch);
    if (rc != AS_OK) return rc;
    // The array keeps whatever the previous call left.  The arrival counters at its
    // front must start at zero; a previous call with fewer sequences may have put
    // split partials where this call's counters are, so clear them every time.
    const size_t counter_bytes = (size_t(num_seqs) * num_heads * sizeof(int32_t) + 255) / 256 * 256;
    cudaError_t e = cudaMemsetAsync(scratch, 0, counter_bytes, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess)
      return fail(AS_ERR_CUDA, "as_paged_decode_attention_noalloc: clearing counters failed: %s",
                  cudaGetErrorString(e));
  }
  return as_paged_decode_attention(out, q, q_stride, k_cache, v_cache, block_tables, bt_stride,
                                   seq_lens_k, num_seqs, num_heads, num_kv_heads, head_dim,
                                   block_size, num_blocks, max_blocks, scale, blocks_per_split,
                                   scratch, scratch ? size_t(AS_DECODE_NOALLOC_SCRATCH_BYTES) : 0,
                                   out_layout, dtype, stream);
}
