// Fused rotary embedding + KV-pool scatter.
//
// Reference behaviour (python/minisgl_mlx/layers.py:45-56 and :103-109,
// kvcache/pool.py:47-50): q and k get rotate-half RoPE (mx.fast.rope,
// traditional=False) at their per-token positions, then the rotated k and the
// untouched v are written to pool slots out_loc[t].
//
// One warp owns one (token, head, kind) row; kind 0 = q, 1 = k, 2 = v. A lane
// handles rotation pairs (i, i + rot/2) for i = lane, lane + 32, ... The pool
// write reuses the rotated k registers, so the stored k is bit-identical to
// the k returned to the caller.
//
// Optionally (q_norm_w / k_norm_w non-null) the row is first normalised with
// the per-head RMSNorm of Qwen3 (models/transformer.py:46-49,54-56, applied to
// q and k before AttentionLayer): y = x * 1/sqrt(mean(x^2) + eps) * w,
// sum of squares in fp32 by a warp reduction, y rounded to the storage dtype
// (the reference's norm is a separate op whose output has that dtype) and
// written back before the rotation reads it.
#pragma once
#include "common.cuh"

namespace b2a {

struct RopeStoreArgs {
  void* q;
  int64_t q_stride;  // elements between token rows
  void* q_out;       // [T, Hq, D] destination of the final q rows, or null (in place)
  void* k;
  int64_t k_stride;
  const void* v;
  int64_t v_stride;
  const int32_t* positions;
  const int32_t* out_loc;
  void* k_pool;
  void* v_pool;
  const float* inv_freq;
  const void* q_norm_w;  // [D] RMSNorm weight of q rows, or null (no norm)
  const void* k_norm_w;  // [D] RMSNorm weight of k rows, or null
  float norm_eps;
  float rope_scale;
  int rot_dim;
  int T, Hq, Hkv, D;
  int64_t num_slots;
};

template <typename T>
__global__ void __launch_bounds__(256) rope_store_kernel(RopeStoreArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int rows_per_tok = a.Hq + 2 * a.Hkv;
  const int64_t total = (int64_t)a.T * rows_per_tok;
  if (row >= total) return;
  const int t = (int)(row / rows_per_tok);
  int r = (int)(row - (int64_t)t * rows_per_tok);
  const bool do_store = a.k_pool != nullptr;

  if (r >= a.Hq + a.Hkv) {
    // ---- v row: byte copy into the pool
    if (!do_store) return;
    const int h = r - a.Hq - a.Hkv;
    const T* src = reinterpret_cast<const T*>(a.v) + (int64_t)t * a.v_stride + (int64_t)h * a.D;
    const int64_t slot = a.out_loc[t];
    if (slot < 0 || slot >= a.num_slots) {
      if (lane == 0) watchdog_set(kWdBadSlot);
      return;
    }
    T* dst = reinterpret_cast<T*>(a.v_pool) + (slot * a.Hkv + h) * a.D;
    for (int d = lane; d < a.D; d += 32) dst[d] = src[d];
    return;
  }

  const bool is_q = r < a.Hq;
  const int h = is_q ? r : r - a.Hq;
  T* x = is_q ? reinterpret_cast<T*>(a.q) + (int64_t)t * a.q_stride + (int64_t)h * a.D
              : reinterpret_cast<T*>(a.k) + (int64_t)t * a.k_stride + (int64_t)h * a.D;
  // final row: in place, or a contiguous q_out row (then x is only scratch)
  T* y = (is_q && a.q_out) ? reinterpret_cast<T*>(a.q_out) + ((int64_t)t * a.Hq + h) * a.D : x;
  T* pool_row = nullptr;
  if (!is_q && do_store) {
    const int64_t slot = a.out_loc[t];
    if (slot >= 0 && slot < a.num_slots) {
      pool_row = reinterpret_cast<T*>(a.k_pool) + (slot * a.Hkv + h) * a.D;
    } else if (lane == 0) {
      watchdog_set(kWdBadSlot);
    }
  }

  const T* nw = reinterpret_cast<const T*>(is_q ? a.q_norm_w : a.k_norm_w);
  if (nw) {
    float ss = 0.f;
    for (int d = lane; d < a.D; d += 32) {
      const float v = DT<T>::to_f(x[d]);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss / (float)a.D + a.norm_eps);
    for (int d = lane; d < a.D; d += 32)
      x[d] = DT<T>::from_f(__fmul_rn(__fmul_rn(DT<T>::to_f(x[d]), inv), DT<T>::to_f(nw[d])));
    __syncwarp();  // the rotation below reads elements other lanes normalised
  }

  const int half = a.rot_dim >> 1;
  if (half > 0) {
    // angle = fl32(fl32(pos * scale) * inv_freq[i]); accurate sincosf (no fast-math).
    const float pos = __fmul_rn((float)a.positions[t], a.rope_scale);
    for (int i = lane; i < half; i += 32) {
      const float ang = __fmul_rn(pos, a.inv_freq[i]);
      float s, c;
      sincosf(ang, &s, &c);
      const float x1 = DT<T>::to_f(x[i]);
      const float x2 = DT<T>::to_f(x[i + half]);
      const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
      const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
      const T o1 = DT<T>::from_f(y1);
      const T o2 = DT<T>::from_f(y2);
      y[i] = o1;
      y[i + half] = o2;
      if (pool_row) {
        pool_row[i] = o1;
        pool_row[i + half] = o2;
      }
    }
  }
  // features that are not rotated (d >= rot_dim) pass through
  if (y != x)
    for (int d = a.rot_dim + lane; d < a.D; d += 32) y[d] = x[d];
  if (pool_row)
    for (int d = a.rot_dim + lane; d < a.D; d += 32) pool_row[d] = x[d];
}

}  // namespace b2a
