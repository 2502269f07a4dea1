// RMSNorm of the engine harness's hidden rows, with an optional row gather.
//
// Reference: nn.RMSNorm in python/minisgl_mlx/models/transformer.py:77-82
// (input_layernorm / post_attention_layernorm of every decoder layer) and the
// final norm after the last-token gather of CausalLM.__call__ (:109-113):
//   y[i] = x[r] * 1 / sqrt(mean(x[r]^2) + eps) * w,  r = rows ? rows[i] : i
// computed in fp32 and rounded once to the storage type (the rounding of a
// fused norm; torch's F.rms_norm on bf16 rounds the same way).
//
// One warp per output row; a lane holds H / 32 consecutive-chunk elements as
// 16-byte vectors (8 bf16 / fp16 or 4 fp32), so a row is read once and the
// weight row once per warp. Launched with programmatic stream serialization,
// like the attention kernels, so it becomes resident while its predecessor
// drains.
#pragma once

#include "common.cuh"

namespace b2a {

struct RmsNormArgs {
  const void* x;
  int64_t x_stride;      // elements between consecutive input rows
  const int32_t* rows;   // NULL: row i of the input; else gather rows[i]
  int64_t x_rows;        // input rows (bounds of the gather)
  void* y;               // [n_rows, H] contiguous
  const void* w;         // [H]
  int64_t n_rows;
  int H;
  float eps;
};

template <typename T, int VPL>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const RmsNormArgs a) {
  pdl_wait_then_release();
  constexpr int EV = 16 / (int)sizeof(T);  // elements per 16-byte vector
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (i >= a.n_rows) return;
  int64_t r = i;
  if (a.rows != nullptr) {
    r = a.rows[i];
    if (r < 0 || r >= a.x_rows) {  // a bad gather index is skipped and reported
      if (lane == 0) watchdog_set(kWdBadSlot);
      return;
    }
  }
  const T* xr = reinterpret_cast<const T*>(a.x) + r * a.x_stride;
  const T* wr = reinterpret_cast<const T*>(a.w);
  // rows of up to 8 vectors a lane load the weights together with the row (one memory
  // round trip, not two); wider rows load them after the reduction (registers)
  constexpr bool kPre = VPL <= 8;
  constexpr int WV = kPre ? VPL : 1;
  float v[VPL][EV], wv[WV][EV];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    load_vec<T, EV>(xr + (size_t)(k * 32 + lane) * EV, v[k]);
    if constexpr (kPre) load_vec<T, EV>(wr + (size_t)(k * 32 + lane) * EV, wv[k]);
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k)
#pragma unroll
    for (int e = 0; e < EV; ++e) ss = fmaf(v[k][e], v[k][e], ss);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = rsqrtf(ss / (float)a.H + a.eps);
  T* yr = reinterpret_cast<T*>(a.y) + i * (int64_t)a.H;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    float* w = wv[kPre ? k : 0];
    if constexpr (!kPre) load_vec<T, EV>(wr + (size_t)(k * 32 + lane) * EV, wv[0]);
#pragma unroll
    for (int e = 0; e < EV; ++e) v[k][e] = v[k][e] * inv * w[e];
    store_vec<T, EV>(yr + (size_t)(k * 32 + lane) * EV, v[k]);
  }
}

}  // namespace b2a
