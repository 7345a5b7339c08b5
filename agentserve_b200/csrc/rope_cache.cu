// (2) Fused RoPE + reshape_and_cache.
//
// One pass over the projected q/k/v of T tokens: q is rotated in place, k is
// rotated and written to its pool slot, v is written to its pool slot, all with
// 128-bit loads/stores.  The rotation is the reference's rotate-half RoPE
// (agentserve/model/llama.py:80-99) evaluated exactly as torch does it: each
// product and the sum/difference rounded separately in fp32 (no FMA contraction),
// then one round-to-nearest-even to the element type.  Together with the fp32
// cos/sin table (llama.py:63-77) this makes the cache contents bit-exact with the
// reference's apply_rope + write_kv_prefill / write_kv_decode (cache.py:125-156).
#include "common.cuh"
#include "host_util.h"

namespace asb {
namespace {

template <typename T, int VEC>
struct alignas(sizeof(T) * VEC) Vec {
  T v[VEC];
};

// Flat index over (token, head-slot, chunk).  head-slot < H: q head; < H+Kh: k head;
// otherwise v head.  A chunk is VEC consecutive elements of the first half of the
// head and the matching VEC elements of the second half.
template <typename T, int VEC>
__global__ void rope_cache_kernel(T* __restrict__ q, int64_t q_stride, const T* __restrict__ k,
                                  int64_t k_stride, const T* __restrict__ v, int64_t v_stride,
                                  const int64_t* __restrict__ positions,
                                  const int64_t* __restrict__ slot_mapping,
                                  const float* __restrict__ cos_sin, int32_t table_len,
                                  T* __restrict__ k_cache, T* __restrict__ v_cache,
                                  int64_t num_slots, T* __restrict__ k_out, int32_t T_tokens,
                                  int32_t H, int32_t Kh, int32_t D, int* status) {
  pdl_wait();  // launched programmatically: the projection that produced q/k/v may still run
  pdl_trigger();
  using V = Vec<T, VEC>;
  const int half = D >> 1;
  const int chunks = half / VEC;
  const int slots_per_tok = (H + 2 * Kh) * chunks;
  const int64_t total = int64_t(T_tokens) * slots_per_tok;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(idx / slots_per_tok);
    const int rem = int(idx - int64_t(t) * slots_per_tok);
    const int hs = rem / chunks;
    const int c = rem - hs * chunks;
    const int i0 = c * VEC;  // first-half element index

    const bool rotate = cos_sin != nullptr;
    const int64_t pos = rotate ? positions[t] : 0;
    if (rotate && (pos < 0 || pos >= table_len)) {
      if (c == 0 && hs == 0) flag_status(status, kStatusBadPosition);
      continue;
    }
    const int64_t slot = slot_mapping[t];
    const bool slot_ok = slot >= 0 && slot < num_slots;
    if (slot >= num_slots && c == 0 && hs == H) flag_status(status, kStatusBadSlot);

    if (hs >= H + Kh) {  // v head: copy both halves to the cache
      if (!slot_ok) continue;
      const int h = hs - H - Kh;
      const T* src = v + int64_t(t) * v_stride + int64_t(h) * D;
      T* dst = v_cache + (slot * Kh + h) * int64_t(D);
      *reinterpret_cast<V*>(dst + i0) = *reinterpret_cast<const V*>(src + i0);
      *reinterpret_cast<V*>(dst + half + i0) = *reinterpret_cast<const V*>(src + half + i0);
      continue;
    }

    if (!rotate) {  // plain reshape_and_cache: k copied unrotated, q untouched
      if (hs < H) continue;
      const int h = hs - H;
      const T* src = k + int64_t(t) * k_stride + int64_t(h) * D;
      const V a = *reinterpret_cast<const V*>(src + i0);
      const V b2 = *reinterpret_cast<const V*>(src + half + i0);
      if (slot_ok) {
        T* dst = k_cache + (slot * Kh + h) * int64_t(D);
        *reinterpret_cast<V*>(dst + i0) = a;
        *reinterpret_cast<V*>(dst + half + i0) = b2;
      }
      if (k_out) {
        T* dst = k_out + (int64_t(t) * Kh + h) * D;
        *reinterpret_cast<V*>(dst + i0) = a;
        *reinterpret_cast<V*>(dst + half + i0) = b2;
      }
      continue;
    }
    const float* cs = cos_sin + pos * int64_t(D);
    float cv[VEC], sv[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      cv[j] = __ldg(cs + i0 + j);
      sv[j] = __ldg(cs + half + i0 + j);
    }
    const T* src;
    if (hs < H) {
      src = q + int64_t(t) * q_stride + int64_t(hs) * D;
    } else {
      src = k + int64_t(t) * k_stride + int64_t(hs - H) * D;
    }
    const V x1 = *reinterpret_cast<const V*>(src + i0);
    const V x2 = *reinterpret_cast<const V*>(src + half + i0);
    V o1, o2;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float a = Elem<T>::to_f32(x1.v[j]);
      const float b = Elem<T>::to_f32(x2.v[j]);
      // (x1, x2) -> (x1*cos - x2*sin, x2*cos + x1*sin), each op rounded on its own.
      const float r1 = __fsub_rn(__fmul_rn(a, cv[j]), __fmul_rn(b, sv[j]));
      const float r2 = __fadd_rn(__fmul_rn(b, cv[j]), __fmul_rn(a, sv[j]));
      o1.v[j] = Elem<T>::from_f32(r1);
      o2.v[j] = Elem<T>::from_f32(r2);
    }
    if (hs < H) {
      T* dst = q + int64_t(t) * q_stride + int64_t(hs) * D;
      *reinterpret_cast<V*>(dst + i0) = o1;
      *reinterpret_cast<V*>(dst + half + i0) = o2;
    } else {
      const int h = hs - H;
      if (slot_ok) {
        T* dst = k_cache + (slot * Kh + h) * int64_t(D);
        *reinterpret_cast<V*>(dst + i0) = o1;
        *reinterpret_cast<V*>(dst + half + i0) = o2;
      }
      if (k_out) {
        T* dst = k_out + (int64_t(t) * Kh + h) * D;
        *reinterpret_cast<V*>(dst + i0) = o1;
        *reinterpret_cast<V*>(dst + half + i0) = o2;
      }
    }
  }
}

template <typename T, int VEC>
int launch_rope_cache(void* q, int64_t q_stride, const void* k, int64_t k_stride, const void* v,
                      int64_t v_stride, const int64_t* positions, const int64_t* slot_mapping,
                      const float* cos_sin, int32_t table_len, void* k_cache, void* v_cache,
                      int64_t num_slots, void* k_out, int32_t T_tokens, int32_t H, int32_t Kh,
                      int32_t D, cudaStream_t stream) {
  const int64_t total = int64_t(T_tokens) * (H + 2 * Kh) * (D / 2 / VEC);
  const int threads = 128;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  launch_pdl(rope_cache_kernel<T, VEC>, dim3(unsigned(blocks)), dim3(threads), 0, stream,
      static_cast<T*>(q), q_stride, static_cast<const T*>(k), k_stride,
      static_cast<const T*>(v), v_stride, positions, slot_mapping, cos_sin, table_len,
      static_cast<T*>(k_cache), static_cast<T*>(v_cache), num_slots, static_cast<T*>(k_out),
      T_tokens, H, Kh, D, device_status_ptr());
  return check_launch("as_rope_reshape_and_cache");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace asb

using namespace asb;

extern "C" int as_rope_reshape_and_cache(void* q, int64_t q_stride, const void* k,
                                         int64_t k_stride, const void* v, int64_t v_stride,
                                         const int64_t* positions, const int64_t* slot_mapping,
                                         const float* cos_sin, int32_t table_len, void* k_cache,
                                         void* v_cache, int64_t num_slots, void* k_out,
                                         int32_t num_tokens, int32_t num_heads,
                                         int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                                         as_stream_t stream) {
  const int es = dtype_size(dtype);
  if (!es) return fail(AS_ERR_INVALID_ARG, "as_rope_reshape_and_cache: unknown dtype %d", dtype);
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      (cos_sin && table_len <= 0))
    return fail(AS_ERR_INVALID_ARG, "as_rope_reshape_and_cache: bad sizes");
  if (num_tokens == 0) return AS_OK;
  const int vec = 16 / es;
  if (head_dim % (2 * vec) != 0)
    return fail(AS_ERR_UNSUPPORTED, "as_rope_reshape_and_cache: head_dim %d must be a multiple of %d",
                head_dim, 2 * vec);
  if (!k || !v || !slot_mapping || !k_cache || !v_cache || (cos_sin && (!q || !positions)))
    return fail(AS_ERR_INVALID_ARG, "as_rope_reshape_and_cache: null pointer");
  if (q_stride < int64_t(num_heads) * head_dim || k_stride < int64_t(num_kv_heads) * head_dim ||
      v_stride < int64_t(num_kv_heads) * head_dim)
    return fail(AS_ERR_INVALID_ARG, "as_rope_reshape_and_cache: row stride smaller than a row");
  const bool al = (!q || aligned16(q)) && aligned16(k) && aligned16(v) && aligned16(k_cache) &&
                  aligned16(v_cache) && (!k_out || aligned16(k_out)) &&
                  (q_stride * es) % 16 == 0 && (k_stride * es) % 16 == 0 &&
                  (v_stride * es) % 16 == 0;
  if (!al)
    return fail(AS_ERR_INVALID_ARG,
                "as_rope_reshape_and_cache: pointers and row strides must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case AS_DTYPE_F32:
      return launch_rope_cache<float, 4>(q, q_stride, k, k_stride, v, v_stride, positions,
                                         slot_mapping, cos_sin, table_len, k_cache, v_cache,
                                         num_slots, k_out, num_tokens, num_heads, num_kv_heads,
                                         head_dim, s);
    case AS_DTYPE_F16:
      return launch_rope_cache<__half, 8>(q, q_stride, k, k_stride, v, v_stride, positions,
                                          slot_mapping, cos_sin, table_len, k_cache, v_cache,
                                          num_slots, k_out, num_tokens, num_heads, num_kv_heads,
                                          head_dim, s);
    default:
      return launch_rope_cache<__nv_bfloat16, 8>(q, q_stride, k, k_stride, v, v_stride, positions,
                                                 slot_mapping, cos_sin, table_len, k_cache,
                                                 v_cache, num_slots, k_out, num_tokens,
                                                 num_heads, num_kv_heads, head_dim, s);
  }
}
