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
  pdl_wait_then_release();
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

// ---------------------------------------------------------------- token-major fast path
//
// The row-per-warp kernel above keeps one 256-byte row in flight per warp, and its
// chain of dependent loads (position, frequency, row) makes it latency-bound at
// ~2 TB/s. This kernel handles 16-bit rows with D = rot_dim = 128. W warps share one
// token, and warp w takes the row groups w, w + W, ... of that token. A group is 4
// rows: lane = 8 * (row in group) + p holds 16-byte chunks p and p + 8 of its row,
// which are rotation partners (features 8p..8p+7 and 64 + 8p..). All of a warp's
// q/k chunks and its share of the v rows are loaded before any arithmetic, so a token's
// ~8 KB is in flight at once. The lane's 8 (cos, sin) pairs are computed once per
// token and reused for every head. The per-element arithmetic and its roundings are
// those of rope_store_kernel, so rotated values and the stored k are identical to it;
// only the sum of squares of the optional RMSNorm is added in another order.
constexpr int kTokMaxGroups = 6;  // q/k row groups of 4 rows held in registers per pass
constexpr int kTokMaxV = 4;       // 16-byte v chunks held in registers per pass

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = DT<T>::to_f(h[e]);
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const T (&h)[8]) {
  uint4 u;
  T* d = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int e = 0; e < 8; ++e) d[e] = h[e];
  return u;
}

template <typename T>
__global__ void __launch_bounds__(256, 2) rope_store_tok_kernel(RopeStoreArgs a, int W) {
  pdl_wait_then_release();
  static_assert(sizeof(T) == 2, "16-bit rows only");
  constexpr int D = 128, HALF = 64;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t t64 = gw / W;
  if (t64 >= a.T) return;
  const int t = (int)t64, w = (int)(gw - t64 * W);
  const int p = lane & 7, rr = lane >> 3;
  const int NR = a.Hq + a.Hkv, NG = (NR + 3) >> 2;
  const bool do_store = a.k_pool != nullptr;
  int64_t slot = -1;
  if (do_store) {
    slot = a.out_loc[t];
    if (slot < 0 || slot >= a.num_slots) {
      if (lane == 0 && w == 0) watchdog_set(kWdBadSlot);
      slot = -1;
    }
  }
  const T* qb = reinterpret_cast<const T*>(a.q) + (int64_t)t * a.q_stride;
  const T* kb = reinterpret_cast<const T*>(a.k) + (int64_t)t * a.k_stride;

  // v rows: this warp's 16-byte chunks, loaded before the q/k arithmetic
  const int nvc = a.Hkv * (D / 8);
  const T* vb = reinterpret_cast<const T*>(a.v) + (int64_t)t * a.v_stride;
  for (int v0 = w * 32; v0 < nvc; v0 += W * 32 * kTokMaxV) {
    uint4 vr[kTokMaxV];
#pragma unroll
    for (int i = 0; i < kTokMaxV; ++i) {
      const int c = v0 + i * W * 32 + lane;
      if (slot >= 0 && c < nvc) vr[i] = *reinterpret_cast<const uint4*>(vb + (c >> 4) * D + (c & 15) * 8);
    }
#pragma unroll
    for (int i = 0; i < kTokMaxV; ++i) {
      const int c = v0 + i * W * 32 + lane;
      if (slot >= 0 && c < nvc)
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.v_pool) + (slot * a.Hkv + (c >> 4)) * D + (c & 15) * 8) = vr[i];
    }
  }

  // (cos, sin) of features 8p..8p+7: angle = fl32(fl32(pos * scale) * inv_freq[i])
  float cs[8], sn[8];
  {
    const float pos = __fmul_rn((float)a.positions[t], a.rope_scale);
    const float4 f0 = reinterpret_cast<const float4*>(a.inv_freq)[2 * p];
    const float4 f1 = reinterpret_cast<const float4*>(a.inv_freq)[2 * p + 1];
    const float fr[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) sincosf(__fmul_rn(pos, fr[e]), &sn[e], &cs[e]);
  }
  const T* qn = reinterpret_cast<const T*>(a.q_norm_w);
  const T* kn = reinterpret_cast<const T*>(a.k_norm_w);

  for (int g0 = w; g0 < NG; g0 += W * kTokMaxGroups) {
    uint4 xa[kTokMaxGroups], xb[kTokMaxGroups];
#pragma unroll
    for (int i = 0; i < kTokMaxGroups; ++i) {
      const int r = (g0 + i * W) * 4 + rr;
      if (r < NR) {
        const T* row = r < a.Hq ? qb + r * D : kb + (r - a.Hq) * D;
        xa[i] = *reinterpret_cast<const uint4*>(row + p * 8);
        xb[i] = *reinterpret_cast<const uint4*>(row + HALF + p * 8);
      }
    }
#pragma unroll
    for (int i = 0; i < kTokMaxGroups; ++i) {
      if ((g0 + i * W) * 4 >= NR) break;  // warp-uniform: no group left
      const int r = (g0 + i * W) * 4 + rr;
      const bool valid = r < NR;
      const bool is_q = r < a.Hq;
      float x1[8], x2[8];
      if (valid) {
        unpack8<T>(xa[i], x1);
        unpack8<T>(xb[i], x2);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) x1[e] = x2[e] = 0.f;
      }
      const T* nw = is_q ? qn : kn;
      // one norm decision per group: q and k rows of one group share it only when
      // both kinds (or neither) are normalised, so every lane joins the shuffles
      if (qn || kn) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(x1[e], x1[e], ss);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(x2[e], x2[e], ss);
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        ss += __shfl_xor_sync(0xffffffffu, ss, 4);
        if (valid && nw) {
          const float inv = 1.0f / sqrtf(ss / (float)D + a.norm_eps);
          float w1[8], w2[8];
          unpack8<T>(*reinterpret_cast<const uint4*>(nw + p * 8), w1);
          unpack8<T>(*reinterpret_cast<const uint4*>(nw + HALF + p * 8), w2);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            x1[e] = DT<T>::to_f(DT<T>::from_f(__fmul_rn(__fmul_rn(x1[e], inv), w1[e])));
            x2[e] = DT<T>::to_f(DT<T>::from_f(__fmul_rn(__fmul_rn(x2[e], inv), w2[e])));
          }
        }
      }
      if (!valid) continue;
      T o1[8], o2[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o1[e] = DT<T>::from_f(__fsub_rn(__fmul_rn(x1[e], cs[e]), __fmul_rn(x2[e], sn[e])));
        o2[e] = DT<T>::from_f(__fadd_rn(__fmul_rn(x2[e], cs[e]), __fmul_rn(x1[e], sn[e])));
      }
      const uint4 u1 = pack8<T>(o1), u2 = pack8<T>(o2);
      T* y;
      if (is_q) {
        y = a.q_out ? reinterpret_cast<T*>(a.q_out) + ((int64_t)t * a.Hq + r) * D
                    : reinterpret_cast<T*>(a.q) + (int64_t)t * a.q_stride + r * D;
      } else {
        y = reinterpret_cast<T*>(a.k) + (int64_t)t * a.k_stride + (r - a.Hq) * D;
        if (slot >= 0) {
          T* pr = reinterpret_cast<T*>(a.k_pool) + (slot * a.Hkv + (r - a.Hq)) * D;
          *reinterpret_cast<uint4*>(pr + p * 8) = u1;
          *reinterpret_cast<uint4*>(pr + HALF + p * 8) = u2;
        }
      }
      *reinterpret_cast<uint4*>(y + p * 8) = u1;
      *reinterpret_cast<uint4*>(y + HALF + p * 8) = u2;
    }
  }
}

}  // namespace b2a
