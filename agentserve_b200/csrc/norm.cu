// Fused elementwise stages of the decode step around the attention kernels:
//   as_rmsnorm       y = to_T(x * rsqrt(mean(x^2) + eps)) * w        (llama.py:39-56)
//   as_add_rmsnorm   x = to_T(x + d); y = rmsnorm(x)                 (llama.py:234-237 + :39-56)
//   as_silu_mul      y = to_T(to_T(silu(g)) * u) for gu = [g | u]     (llama.py:207-211)
// Each replaces 5-8 separate torch kernels per call with one pass over the rows.
// Rounding follows the reference's torch op sequence: statistics in fp32, the
// normalised row rounded to the element type before the (element-type) weight
// multiply, the residual sum rounded once, silu rounded before the gate multiply.
#include "common.cuh"
#include "host_util.h"

namespace asb {
namespace {

template <typename T, int VEC>
struct alignas(sizeof(T) * VEC) Pack {
  T v[VEC];
};

template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) s += red[i];
  return s;
}

// One CTA per row.  ROW_VECS = dim / (THREADS*VEC) vectors per thread, held in registers.
template <typename T, int VEC, int THREADS, int ROW_VECS, bool ADD>
__global__ void __launch_bounds__(THREADS)
rmsnorm_kernel(T* __restrict__ y, T* __restrict__ x, const T* __restrict__ d,
               const T* __restrict__ w, int dim, float eps) {
  pdl_wait();  // programmatic launch: nothing is touched before the previous kernel ends
  pdl_trigger();
  using P = Pack<T, VEC>;
  __shared__ float red[THREADS / 32];
  const int64_t row = blockIdx.x;
  T* xr = x + row * dim;
  float xf[ROW_VECS][VEC];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < ROW_VECS; ++i) {
    const int col = (i * THREADS + threadIdx.x) * VEC;
    P a = *reinterpret_cast<const P*>(xr + col);
    if (ADD) {
      const P b = *reinterpret_cast<const P*>(d + row * dim + col);
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        a.v[e] = Elem<T>::from_f32(Elem<T>::to_f32(a.v[e]) + Elem<T>::to_f32(b.v[e]));
      *reinterpret_cast<P*>(xr + col) = a;
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      xf[i][e] = Elem<T>::to_f32(a.v[e]);
      ss += xf[i][e] * xf[i][e];
    }
  }
  const float mean = block_sum<THREADS>(ss, red) * (1.0f / float(dim));
  const float r = rsqrtf(mean + eps);
#pragma unroll
  for (int i = 0; i < ROW_VECS; ++i) {
    const int col = (i * THREADS + threadIdx.x) * VEC;
    const P wv = *reinterpret_cast<const P*>(w + col);
    P o;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const T n = Elem<T>::from_f32(xf[i][e] * r);
      o.v[e] = Elem<T>::from_f32(Elem<T>::to_f32(n) * Elem<T>::to_f32(wv.v[e]));
    }
    *reinterpret_cast<P*>(y + row * dim + col) = o;
  }
}

// Generic fallback for dims that do not split evenly into vectors per thread.
template <typename T, bool ADD>
__global__ void __launch_bounds__(256)
rmsnorm_generic_kernel(T* __restrict__ y, T* __restrict__ x, const T* __restrict__ d,
                       const T* __restrict__ w, int dim, float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  T* xr = x + row * dim;
  float ss = 0.f;
  for (int c = threadIdx.x; c < dim; c += 256) {
    float v = Elem<T>::to_f32(xr[c]);
    if (ADD) {
      const T s = Elem<T>::from_f32(v + Elem<T>::to_f32(d[row * dim + c]));
      xr[c] = s;
      v = Elem<T>::to_f32(s);
    }
    ss += v * v;
  }
  const float mean = block_sum<256>(ss, red) * (1.0f / float(dim));
  const float r = rsqrtf(mean + eps);
  for (int c = threadIdx.x; c < dim; c += 256) {
    const T n = Elem<T>::from_f32(Elem<T>::to_f32(xr[c]) * r);
    y[row * dim + c] = Elem<T>::from_f32(Elem<T>::to_f32(n) * Elem<T>::to_f32(w[c]));
  }
}

template <typename T, int VEC>
__global__ void silu_mul_kernel(T* __restrict__ y, const T* __restrict__ gu, int64_t rows,
                                int inter) {
  pdl_wait();
  pdl_trigger();
  using P = Pack<T, VEC>;
  const int per_row = inter / VEC;
  const int64_t total = rows * per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row;
    const int c = int(i - r * per_row) * VEC;
    const P g = *reinterpret_cast<const P*>(gu + r * 2 * inter + c);
    const P u = *reinterpret_cast<const P*>(gu + r * 2 * inter + inter + c);
    P o;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float gf = Elem<T>::to_f32(g.v[e]);
      const T s = Elem<T>::from_f32(gf / (1.0f + expf(-gf)));
      o.v[e] = Elem<T>::from_f32(Elem<T>::to_f32(s) * Elem<T>::to_f32(u.v[e]));
    }
    *reinterpret_cast<P*>(y + r * inter + c) = o;
  }
}

template <typename T, bool ADD>
int launch_rmsnorm(void* y, void* x, const void* d, const void* w, int64_t rows, int dim,
                   float eps, cudaStream_t s) {
  constexpr int VEC = 16 / sizeof(T);
  T* yy = static_cast<T*>(y);
  T* xx = static_cast<T*>(x);
  const T* dd = static_cast<const T*>(d);
  const T* ww = static_cast<const T*>(w);
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(x) |
                        reinterpret_cast<uintptr_t>(w) | (ADD ? reinterpret_cast<uintptr_t>(d) : 0)) &
                       15) == 0;
  if (vec_ok && dim == 256 * VEC * 1)
    launch_pdl(rmsnorm_kernel<T, VEC, 256, 1, ADD>, dim3(unsigned(rows)), dim3(256), 0, s, yy, xx, dd, ww, dim, eps);
  else if (vec_ok && dim == 256 * VEC * 2)
    launch_pdl(rmsnorm_kernel<T, VEC, 256, 2, ADD>, dim3(unsigned(rows)), dim3(256), 0, s, yy, xx, dd, ww, dim, eps);
  else if (vec_ok && dim == 256 * VEC * 3)
    launch_pdl(rmsnorm_kernel<T, VEC, 256, 3, ADD>, dim3(unsigned(rows)), dim3(256), 0, s, yy, xx, dd, ww, dim, eps);
  else if (vec_ok && dim == 256 * VEC * 4)
    launch_pdl(rmsnorm_kernel<T, VEC, 256, 4, ADD>, dim3(unsigned(rows)), dim3(256), 0, s, yy, xx, dd, ww, dim, eps);
  else
    launch_pdl(rmsnorm_generic_kernel<T, ADD>, dim3(unsigned(rows)), dim3(256), 0, s, yy, xx, dd, ww, dim, eps);
  return check_launch(ADD ? "as_add_rmsnorm" : "as_rmsnorm");
}

template <bool ADD>
int rmsnorm_entry(void* y, void* x, const void* d, const void* w, int64_t rows, int32_t dim,
                  float eps, int32_t dtype, as_stream_t stream) {
  const char* name = ADD ? "as_add_rmsnorm" : "as_rmsnorm";
  if (!dtype_size(dtype)) return fail(AS_ERR_INVALID_ARG, "%s: unknown dtype", name);
  if (rows < 0 || dim <= 0) return fail(AS_ERR_INVALID_ARG, "%s: bad sizes", name);
  if (rows == 0) return AS_OK;
  if (rows > 0x7fffffff) return fail(AS_ERR_INVALID_ARG, "%s: too many rows", name);
  if (!y || !x || !w || (ADD && !d)) return fail(AS_ERR_INVALID_ARG, "%s: null pointer", name);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case AS_DTYPE_F32: return launch_rmsnorm<float, ADD>(y, x, d, w, rows, dim, eps, s);
    case AS_DTYPE_F16: return launch_rmsnorm<__half, ADD>(y, x, d, w, rows, dim, eps, s);
    default: return launch_rmsnorm<__nv_bfloat16, ADD>(y, x, d, w, rows, dim, eps, s);
  }
}

template <typename T>
int launch_silu_mul(void* y, const void* gu, int64_t rows, int inter, cudaStream_t s) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t total = rows * (inter / VEC);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = int64_t(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  launch_pdl(silu_mul_kernel<T, VEC>, dim3(unsigned(blocks)), dim3(256), 0, s, static_cast<T*>(y),
             static_cast<const T*>(gu), rows, inter);
  return check_launch("as_silu_mul");
}

}  // namespace
}  // namespace asb

using namespace asb;

extern "C" int as_rmsnorm(void* out, const void* x, const void* weight, int64_t rows, int32_t dim,
                          float eps, int32_t dtype, as_stream_t stream) {
  return rmsnorm_entry<false>(out, const_cast<void*>(x), nullptr, weight, rows, dim, eps, dtype,
                              stream);
}

extern "C" int as_add_rmsnorm(void* out, void* x, const void* delta, const void* weight,
                              int64_t rows, int32_t dim, float eps, int32_t dtype,
                              as_stream_t stream) {
  return rmsnorm_entry<true>(out, x, delta, weight, rows, dim, eps, dtype, stream);
}

extern "C" int as_silu_mul(void* out, const void* gate_up, int64_t rows, int32_t inter,
                           int32_t dtype, as_stream_t stream) {
  const int es = dtype_size(dtype);
  if (!es) return fail(AS_ERR_INVALID_ARG, "as_silu_mul: unknown dtype");
  if (rows < 0 || inter <= 0) return fail(AS_ERR_INVALID_ARG, "as_silu_mul: bad sizes");
  if (rows == 0) return AS_OK;
  if (!out || !gate_up) return fail(AS_ERR_INVALID_ARG, "as_silu_mul: null pointer");
  if ((inter * es) % 16 || ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(gate_up)) & 15))
    return fail(AS_ERR_INVALID_ARG, "as_silu_mul: rows must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case AS_DTYPE_F32: return launch_silu_mul<float>(out, gate_up, rows, inter, s);
    case AS_DTYPE_F16: return launch_silu_mul<__half>(out, gate_up, rows, inter, s);
    default: return launch_silu_mul<__nv_bfloat16>(out, gate_up, rows, inter, s);
  }
}
