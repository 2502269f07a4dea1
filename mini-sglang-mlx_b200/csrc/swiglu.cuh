// SwiGLU activation of the MLP: out = silu(gate) * up in one pass.
//
// Reference: python/minisgl_mlx/models/transformer.py:26-30 (`swiglu`, which
// mx.compile fuses into one kernel) called from MLP.__call__ (:67-69) on the
// two halves of the fused gate/up projection. Row r of the input holds
// [gate (F) | up (F)] at a row stride; the output is a contiguous [rows, F].
// The arithmetic is fp32 with the roundings of the unfused form
// `silu(gate) * up` on 16-bit tensors: silu(g) = g / (1 + e^-g) is rounded to
// the storage type before the product, and the product is rounded again.
// Work per element: 3 loads/stores of sizeof(T) -- an HBM-bound kernel; each
// thread handles two adjacent features so 16-bit rows move as 32-bit words.
#pragma once
#include "common.cuh"

namespace b2a {

template <typename T>
__device__ __forceinline__ float swiglu_one(float g, float u) {
  float s = g / (1.f + expf(-g));
  s = DT<T>::to_f(DT<T>::from_f(s));  // the unfused form stores silu(gate) in T
  return s * u;
}

template <typename T>
__global__ void __launch_bounds__(256)
    swiglu_kernel(const T* __restrict__ gu, int64_t row_stride, T* __restrict__ out, int64_t rows, int F) {
  const int half_f = F >> 1;
  const int64_t n = rows * half_f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / half_f;
    const int c = (int)(i - r * half_f) * 2;
    const T* g = gu + r * row_stride + c;
    const T* u = g + F;
    T* o = out + r * F + c;
    o[0] = DT<T>::from_f(swiglu_one<T>(DT<T>::to_f(g[0]), DT<T>::to_f(u[0])));
    o[1] = DT<T>::from_f(swiglu_one<T>(DT<T>::to_f(g[1]), DT<T>::to_f(u[1])));
  }
}

}  // namespace b2a
