// Decode-batch projections of the engine harness's model: Y = X W^T for a few
// token rows (M <= 64), bf16 operands, fp32 accumulation, with the RMSNorm in
// front and the residual add or the SwiGLU behind fused into the same launch.
//
// Reference (python/minisgl_mlx/models/transformer.py):
//   qkv_proj / o_proj (:41-42), gate_up_proj / down_proj (:64-65),
//   DecoderLayer.__call__ (:80-82):
//     h = x + o_proj(attn(qkv_proj(input_layernorm(x))))
//     return h + down_proj(swiglu(gate_up_proj(post_attention_layernorm(h))))
//   swiglu (:26-30) on the two halves of gate_up_proj (:67-69).
// The three fused forms are
//   plain     out = [norm](x) W^T                      (qkv_proj after input_layernorm)
//   residual  out = res + x W^T, out may alias res     (o_proj, down_proj with the adds)
//   swiglu    out = silu(g) * u, [g | u] = [norm](x) W^T  (gate_up_proj + swiglu)
//
// Design. A decode step multiplies a handful of rows by every weight of the
// layer once, so a projection is a stream of its weight matrix through the
// SMs (2 bytes per weight, 2M FLOPs per weight): HBM-bound for M <= 64. A CTA
// owns 16 consecutive weight rows (output features; 16 gate + 16 up rows for
// SwiGLU) across all of K. Its first thread copies that slab into shared
// memory with one 1-D bulk copy (TMA) per row, BEFORE the programmatic-
// dependent-launch wait -- weights do not depend on the previous kernel, so
// the stream starts while the previous kernel drains, and the bytes in flight
// are bounded by shared memory, not registers. The warps split K into
// 128-wide slices; each loads its slice of the token rows (from L2, written by
// the previous kernel) after the wait, then the tensor cores (mma.sync
// m16n8k16; the weight rows are the 16-row A operand, the token rows the
// 8-column B operand) take the products. The split-K partials meet in shared
// memory (over the slab, once every warp is past it) and one pass applies the
// epilogue.
//
// Operand order inside a 32-wide k chunk. A lane (g = lane/4, t = lane%4)
// takes 8 consecutive k (16 bytes) of its weight rows g and g+8 and of its
// token row g. A dot product does not depend on the order of its k terms, so
// the chunk's first MMA uses k 8t..8t+3 of every lane and the second MMA
// 8t+4..8t+7, with the same assignment for both operands: the fragments are
// plain 16-byte loads, with no shuffles or transposes. Slab rows are K * 2 + 64
// bytes apart, so the eight lanes of a quarter-warp (rows g, g+1, four
// 16-byte columns each) read 128 distinct bytes: no bank conflicts.
//
// RMSNorm in front: y = W (x * inv * w_n) = inv * (W (x * w_n)) with
// inv = 1 / sqrt(mean(x^2) + eps) one scalar per token row, so the operand is
// x * w_n (rounded once to bf16) and inv multiplies the fp32 result; the sum
// of squares comes from the same loads (each x element is loaded by exactly
// one lane of the CTA) and is reduced with the partial products.
// SwiGLU behind: the CTA's two 16-row tiles are gate rows j..j+15 and up rows
// F+j..F+j+15, so each output column has both of its factors in the CTA. The
// epilogue keeps the roundings of the unfused 16-bit form: gate and up are
// rounded to bf16 (the projection's output), silu(gate) is rounded, then the
// product.
#pragma once
#include "common.cuh"

namespace b2a {

enum ProjMode : int { kProjPlain = 0, kProjResidual = 1, kProjSwiglu = 2 };

struct ProjArgs {
  const __nv_bfloat16* x;       // [M, K], row stride ldx (elements)
  const __nv_bfloat16* w;       // [N, K], contiguous rows
  const __nv_bfloat16* norm_w;  // [K] RMSNorm weight (norm variants only)
  const __nv_bfloat16* res;     // [M, N] residual (residual mode; may equal out)
  __nv_bfloat16* out;           // [M, N] (plain / residual) or [M, N/2] (swiglu)
  int64_t ldx, ldr, ldo;
  int M, K;
  int F;     // swiglu: up rows start at row F (N = 2F)
  int kpw;   // 128-wide k slices per warp
  float eps;
};

__device__ __forceinline__ void proj_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Device error recorded when the weight slab's bulk copies do not land within
// the bounded wait (the watchdog codes of common.cuh continue here).
constexpr int kWdProjWait = 18;

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

__device__ __forceinline__ uint32_t f2_to_bf2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Shared memory: the weight slab (16 A rows of K * 2 + 64 bytes), later reused by
// the split-K reduction -- per warp [NB*8 tokens][A*16 + 4 features] partials (the
// +4 keeps one warp's fragment stores on distinct banks), per warp [NB*8] sums of
// squares, [NB*8] per-token scales -- then the slab's mbarrier.
template <int NB, int A>
struct ProjSmem {
  static constexpr int FP = A * 16 + 4;
  static constexpr int ACC = NB * 8 * FP;
  __host__ __device__ static constexpr uint32_t row_bytes(int K) { return (uint32_t)K * 2 + 64; }
  __host__ __device__ static constexpr size_t red_bytes(int warps) {
    return (size_t)warps * (ACC + NB * 8) * 4 + NB * 8 * 4;
  }
  __host__ __device__ static constexpr size_t region(int K, int warps) {
    const size_t slab = (size_t)16 * A * row_bytes(K);
    const size_t red = red_bytes(warps);
    return ((slab > red ? slab : red) + 15) / 16 * 16;
  }
  __host__ __device__ static constexpr size_t bytes(int K, int warps) { return region(K, warps) + 16; }
};

template <int NB, int A, int MODE, bool NORM, int MAXW>
__global__ void __launch_bounds__(MAXW * 32) proj_kernel(const ProjArgs a) {
  static_assert(MODE != kProjSwiglu || A == 2, "swiglu pairs a gate tile with an up tile");
  using S = ProjSmem<NB, A>;
  extern __shared__ __align__(128) uint8_t proj_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t rb = S::row_bytes(a.K);
  uint64_t* bar = reinterpret_cast<uint64_t*>(proj_smem + S::region(a.K, nw));
  const uint32_t slab = smem_u32(proj_smem);

  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    // the slab: one bulk copy per weight row, lane r copies row r
    const uint32_t bytes = (uint32_t)a.K * 2;
    if (lane == 0) mbar_arrive_expect_tx(bar, bytes * 16 * A);
    __syncwarp();
    if (lane < 16 * A) {
      const int r = lane;
      const int wrow = MODE == kProjSwiglu ? (r < 16 ? 0 : a.F - 16) + (int)blockIdx.x * 16 + r
                                           : (int)blockIdx.x * 16 * A + r;
      bulk_g2s(proj_smem + (size_t)r * rb, a.w + (size_t)wrow * a.K, bytes, bar, l2_evict_first_policy());
    }
  }
  pdl_wait_then_release();  // x, res and out belong to the previous kernels

  float acc[A][NB][4];
#pragma unroll
  for (int i = 0; i < A; ++i)
#pragma unroll
    for (int n = 0; n < NB; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][n][e] = 0.f;
  float ss[NB];
#pragma unroll
  for (int n = 0; n < NB; ++n) ss[n] = 0.f;

  // The token rows of CB chunks are loaded (and normalised) together before the first
  // MMA that needs the slab: the slab's wait is ordered asm, so loads placed after it
  // would each start only once the previous chunk's MMAs were issued.
  constexpr int CB = NB <= 4 ? 4 : 2;
  bool landed = false;
  for (int s = 0; s < a.kpw; ++s) {
    const int kb = (warp * a.kpw + s) * 128 + 8 * t;
#pragma unroll
    for (int c0 = 0; c0 < 4; c0 += CB) {
      uint4 xv[CB][NB];
#pragma unroll
      for (int cc = 0; cc < CB; ++cc) {
        const int k = kb + (c0 + cc) * 32;
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const int tok = n * 8 + g;
          xv[cc][n] = tok < a.M ? *reinterpret_cast<const uint4*>(a.x + (size_t)tok * a.ldx + k) : make_uint4(0, 0, 0, 0);
        }
      }
      if constexpr (NORM) {
#pragma unroll
        for (int cc = 0; cc < CB; ++cc) {
          const uint4 nwv = *reinterpret_cast<const uint4*>(a.norm_w + kb + (c0 + cc) * 32);
          const float2 w0 = bf2_to_f2(nwv.x), w1 = bf2_to_f2(nwv.y), w2 = bf2_to_f2(nwv.z), w3 = bf2_to_f2(nwv.w);
#pragma unroll
          for (int n = 0; n < NB; ++n) {
            uint4& v = xv[cc][n];
            const float2 x0 = bf2_to_f2(v.x), x1 = bf2_to_f2(v.y), x2 = bf2_to_f2(v.z), x3 = bf2_to_f2(v.w);
            ss[n] += x0.x * x0.x + x0.y * x0.y + x1.x * x1.x + x1.y * x1.y + x2.x * x2.x + x2.y * x2.y +
                     x3.x * x3.x + x3.y * x3.y;
            v.x = f2_to_bf2(x0.x * w0.x, x0.y * w0.y);
            v.y = f2_to_bf2(x1.x * w1.x, x1.y * w1.y);
            v.z = f2_to_bf2(x2.x * w2.x, x2.y * w2.y);
            v.w = f2_to_bf2(x3.x * w3.x, x3.y * w3.y);
          }
        }
      }
      if (!landed) {
        // bounded: a slab that never lands records the device error and the CTA
        // finishes on whatever the slab holds (no fault, no hang)
        if (!mbar_wait(bar, 0, kWdProjWait)) mbar_wait(bar, 0, kWdProjWait);
        landed = true;
      }
#pragma unroll
      for (int cc = 0; cc < CB; ++cc) {
        const int k = kb + (c0 + cc) * 32;
#pragma unroll
        for (int i = 0; i < A; ++i) {
          const uint4 w0 = lds128(slab + (uint32_t)(i * 16 + g) * rb + (uint32_t)k * 2);
          const uint4 w1 = lds128(slab + (uint32_t)(i * 16 + g + 8) * rb + (uint32_t)k * 2);
#pragma unroll
          for (int n = 0; n < NB; ++n) {
            proj_mma(acc[i][n], w0.x, w1.x, w0.y, w1.y, xv[cc][n].x, xv[cc][n].y);
            proj_mma(acc[i][n], w0.z, w1.z, w0.w, w1.w, xv[cc][n].z, xv[cc][n].w);
          }
        }
      }
    }
  }
  if (!landed && !mbar_wait(bar, 0, kWdProjWait)) mbar_wait(bar, 0, kWdProjWait);  // no slice: drain the copies
  __syncthreads();  // every warp is past the slab: the reduction may overwrite it

  // ---- split-K partials -> shared memory: C fragment (feature g / g+8, tokens 2t, 2t+1)
  float* red = reinterpret_cast<float*>(proj_smem);
  float* red_ss = red + (size_t)nw * S::ACC;
  float* inv_s = red_ss + nw * NB * 8;
  float* mine = red + (size_t)warp * S::ACC;
#pragma unroll
  for (int i = 0; i < A; ++i)
#pragma unroll
    for (int n = 0; n < NB; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int f = i * 16 + g + 8 * (e >> 1);
        const int tok = n * 8 + 2 * t + (e & 1);
        mine[tok * S::FP + f] = acc[i][n][e];
      }
  if constexpr (NORM) {
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      float v = ss[n];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (t == 0) red_ss[warp * NB * 8 + n * 8 + g] = v;
    }
  }
  __syncthreads();
  if constexpr (NORM) {
    for (int tok = threadIdx.x; tok < NB * 8; tok += blockDim.x) {
      float v = 0.f;
      for (int w = 0; w < nw; ++w) v += red_ss[w * NB * 8 + tok];
      inv_s[tok] = rsqrtf(v / (float)a.K + a.eps);
    }
    __syncthreads();
  }

  // ---- epilogue: one output element per thread and step, features fastest
  constexpr int FO = MODE == kProjSwiglu ? 16 : A * 16;
  const int n_out = a.M * FO;
  for (int e = threadIdx.x; e < n_out; e += blockDim.x) {
    const int tok = e / FO, f = e - tok * FO;
    float v = 0.f;
    for (int w = 0; w < nw; ++w) v += red[(size_t)w * S::ACC + tok * S::FP + f];
    const float sc = NORM ? inv_s[tok] : 1.f;
    if constexpr (MODE == kProjSwiglu) {
      float u = 0.f;
      for (int w = 0; w < nw; ++w) u += red[(size_t)w * S::ACC + tok * S::FP + 16 + f];
      const float gq = bf16_round(v * sc), uq = bf16_round(u * sc);
      const float sl = bf16_round(gq / (1.f + expf(-gq)));
      a.out[(size_t)tok * a.ldo + (int)blockIdx.x * 16 + f] = __float2bfloat16_rn(sl * uq);
    } else {
      const int col = (int)blockIdx.x * FO + f;
      v *= sc;
      if constexpr (MODE == kProjResidual) v += __bfloat162float(a.res[(size_t)tok * a.ldr + col]);
      a.out[(size_t)tok * a.ldo + col] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace b2a
