// Ragged causal extend (prefill) attention, SIMT fp32-accumulating kernel.
//
// Reference: python/minisgl_mlx/attention/base.py:70-105. Request r owns
// query rows [qo_indptr[r], qo_indptr[r+1]) (Lq of them) and Lkv pool tokens
// (prefix + the rows just stored); row i sees keys j <= Lkv - Lq + i
// (bottom-right causal). This kernel is the exact-fp32 path (parity 1e-5) and
// the fallback for shapes the tcgen05 kernel does not cover.
//
// CTA = (work item, kv head h). Tile rows = TQ tokens x G query heads
// (row = token * G + g), so the G heads of a GQA group share one pass over
// K/V. K/V blocks of 32 keys are gathered from the pool page by page and
// widened to fp32 in shared memory (K rows padded to D+1 floats so the
// lane-per-key dot products are bank-conflict free).
#pragma once
#include "common.cuh"

namespace b2a {

struct ExtendArgs {
  const void* q;
  const void* k_pool;
  const void* v_pool;
  const int32_t* qo_indptr;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* kv_last_page_len;
  const int32_t* work;  // int4 {request, q tile begin, q tile rows, 0}
  void* out;
  int64_t num_slots;
  int page_log2;
  int Hq, Hkv;
  float qscale;  // scale * log2(e)
};

constexpr int kSimtRows = 64;  // rows per CTA (TQ * G)
constexpr int kSimtBK = 32;    // keys per block
constexpr int kSimtThreads = 256;

__device__ __forceinline__ int request_kv_len(const int32_t* kv_indptr, const int32_t* last_page_len, int r,
                                              int page_log2) {
  const int np = kv_indptr[r + 1] - kv_indptr[r];
  if (np <= 0) return 0;
  const int last = last_page_len ? last_page_len[r] : (1 << page_log2);
  return ((np - 1) << page_log2) + last;
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(kSimtThreads) extend_simt_kernel(const ExtendArgs a) {
  constexpr int EPT = D / 32;
  constexpr int RPW = kSimtRows / (kSimtThreads / 32);  // rows per warp (8)
  constexpr int BK = kSimtBK;
  constexpr unsigned FULL = 0xffffffffu;
  extern __shared__ __align__(16) float sm[];
  float* Qs = sm;                      // [64][D]
  float* Ks = Qs + kSimtRows * D;      // [BK][D+1]
  float* Vs = Ks + BK * (D + 1);       // [BK][D]

  const int4 w = reinterpret_cast<const int4*>(a.work)[blockIdx.x];
  const int r = w.x, tb = w.y;
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nq = min(w.z, kSimtRows / G);
  if (w.z > nq && tid == 0) watchdog_set(kWdTileTooLarge);
  const int Lq = a.qo_indptr[r + 1] - a.qo_indptr[r];
  const int Lkv = request_kv_len(a.kv_indptr, a.kv_last_page_len, r, a.page_log2);
  const int prefix = Lkv - Lq;
  const int qrow0 = a.qo_indptr[r] + tb;
  const int P = 1 << a.page_log2;
  const int32_t* pages = a.kv_indices + a.kv_indptr[r];

  // ---- Q tile (pre-scaled, zero rows past the tile end)
  const T* qg = reinterpret_cast<const T*>(a.q);
  for (int idx = tid; idx < kSimtRows * (D / 2); idx += kSimtThreads) {
    const int row = idx / (D / 2), c = idx - row * (D / 2);
    const int tok = row / G, g = row - tok * G;
    float v2[2] = {0.f, 0.f};
    if (tok < nq) load_vec<T, 2>(qg + ((size_t)(qrow0 + tok) * a.Hq + h * G + g) * D + 2 * c, v2);
    Qs[row * D + 2 * c] = v2[0] * a.qscale;
    Qs[row * D + 2 * c + 1] = v2[1] * a.qscale;
  }

  float m[RPW], l[RPW], acc[RPW][EPT];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    m[i] = kNegInf;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < EPT; ++e) acc[i][e] = 0.f;
  }
  const int row0 = warp * RPW;
  // keys visible to the last valid row of the tile
  const int kv_end = min(Lkv, prefix + tb + nq);
  const T* kp = reinterpret_cast<const T*>(a.k_pool);
  const T* vp = reinterpret_cast<const T*>(a.v_pool);

  for (int kb = 0; kb < kv_end; kb += BK) {
    __syncthreads();
    for (int idx = tid; idx < BK * (D / 2); idx += kSimtThreads) {
      const int j = idx / (D / 2), c = idx - j * (D / 2);
      const int pos = kb + j;
      float k2[2] = {0.f, 0.f}, v2[2] = {0.f, 0.f};
      const int64_t slot = pos < kv_end ? (int64_t)pages[pos >> a.page_log2] * P + (pos & (P - 1)) : -1;
      if (pos < kv_end && (slot < 0 || slot >= a.num_slots)) watchdog_set(kWdBadSlot);
      if (pos < kv_end && slot >= 0 && slot < a.num_slots) {
        const size_t off = ((size_t)slot * a.Hkv + h) * D + 2 * c;
        load_vec<T, 2>(kp + off, k2);
        load_vec<T, 2>(vp + off, v2);
      }
      Ks[j * (D + 1) + 2 * c] = k2[0];
      Ks[j * (D + 1) + 2 * c + 1] = k2[1];
      Vs[j * D + 2 * c] = v2[0];
      Vs[j * D + 2 * c + 1] = v2[1];
    }
    __syncthreads();

    // ---- scores: lane = key
    float s[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) s[i] = 0.f;
    for (int d = 0; d < D; d += 4) {
      float kk[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) kk[u] = Ks[lane * (D + 1) + d + u];
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        const float4 qv = *reinterpret_cast<const float4*>(&Qs[(row0 + i) * D + d]);
        s[i] = fmaf(qv.x, kk[0], s[i]);
        s[i] = fmaf(qv.y, kk[1], s[i]);
        s[i] = fmaf(qv.z, kk[2], s[i]);
        s[i] = fmaf(qv.w, kk[3], s[i]);
      }
    }
    const int kpos = kb + lane;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int row = row0 + i;
      const int tok = row / G;
      const bool valid = (tok < nq) && (kpos < kv_end) && (kpos <= prefix + tb + tok);
      const float si = valid ? s[i] : kNegInf;
      float mt = si;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(FULL, mt, off));
      const float m_new = fmaxf(m[i], mt);
      const float alpha = (m[i] == m_new) ? 1.f : exp2f(m[i] - m_new);
      s[i] = (si == kNegInf) ? 0.f : exp2f(si - m_new);  // s now holds p
      l[i] = l[i] * alpha + s[i];
      m[i] = m_new;
#pragma unroll
      for (int e = 0; e < EPT; ++e) acc[i][e] *= alpha;
    }
    // ---- PV: lane owns features lane*EPT .. +EPT
    const int nk = min(BK, kv_end - kb);
    for (int j = 0; j < nk; ++j) {
      float vv[EPT];
#pragma unroll
      for (int e = 0; e < EPT; ++e) vv[e] = Vs[j * D + lane * EPT + e];
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        const float pj = __shfl_sync(FULL, s[i], j);
#pragma unroll
        for (int e = 0; e < EPT; ++e) acc[i][e] = fmaf(pj, vv[e], acc[i][e]);
      }
    }
  }

  // ---- epilogue
  T* og = reinterpret_cast<T*>(a.out);
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    float lsum = l[i];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) lsum += __shfl_xor_sync(FULL, lsum, off);
    const int row = row0 + i;
    const int tok = row / G, g = row - tok * G;
    if (tok < nq) {
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      float o[EPT];
#pragma unroll
      for (int e = 0; e < EPT; ++e) o[e] = acc[i][e] * inv;
      store_vec<T, EPT>(og + ((size_t)(qrow0 + tok) * a.Hq + h * G + g) * D + lane * EPT, o);
    }
  }
}

inline size_t extend_simt_smem(int D) {
  return sizeof(float) * ((size_t)kSimtRows * D + (size_t)kSimtBK * (D + 1) + (size_t)kSimtBK * D);
}

}  // namespace b2a
