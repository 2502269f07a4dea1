// Fused rotary embedding + KV-pool scatter.
//
// Reference behaviour (python/minisgl_mlx/layers.py:45-56 and :103-109,
// kvcache/pool.py:47-50): q and k get rotate-half RoPE (mx.fast.rope,
// traditional=False) at their per-token positions, then the rotated k and the
// untouched v are written to pool slots out_loc[t].
//
// One warp owns one (token, head, kind) row; kind 0 = q, 1 = k, 2 = v. A lane
// handles PAIRS consecutive rotation pairs (i, i + rot/2), so a warp covers
// 32 * PAIRS pairs per pass. The pool write reuses the rotated k registers,
// so the stored k is bit-identical to the k returned to the caller.
#pragma once
#include "common.cuh"

namespace b2a {

struct RopeStoreArgs {
  void* q;
  int64_t q_stride;  // elements between token rows
  void* k;
  int64_t k_stride;
  const void* v;
  int64_t v_stride;
  const int32_t* positions;
  const int32_t* out_loc;
  void* k_pool;
  void* v_pool;
  const float* inv_freq;
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
  T* pool_row = nullptr;
  if (!is_q && do_store) {
    const int64_t slot = a.out_loc[t];
    if (slot >= 0 && slot < a.num_slots) {
      pool_row = reinterpret_cast<T*>(a.k_pool) + (slot * a.Hkv + h) * a.D;
    } else if (lane == 0) {
      watchdog_set(kWdBadSlot);
    }
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
      x[i] = o1;
      x[i + half] = o2;
      if (pool_row) {
        pool_row[i] = o1;
        pool_row[i + half] = o2;
      }
    }
  }
  if (pool_row) {
    // features that are not rotated (d >= rot_dim) are copied as-is
    for (int d = a.rot_dim + lane; d < a.D; d += 32) pool_row[d] = x[d];
  }
}

}  // namespace b2a
