// Shared device helpers for the B200 attention kernels (sm_100a).
//
// - dtype adapters (fp32 / bf16 / fp16 <-> fp32 registers, vector loads)
// - mbarrier + cp.async.bulk (TMA bulk copy) wrappers in inline PTX
// - bounded spin-waits that record a watchdog code instead of hanging
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b2a {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegInf = -__builtin_huge_valf();

// Watchdog word: a bounded wait that gives up writes a nonzero code here and
// the kernel unwinds. Read (and cleared) by b2a_device_error().
__device__ int g_watchdog;

enum WatchdogCode : int {
  kWdDecodeFull = 1,
  kWdDecodeEmpty = 2,
  kWdDecodeDrain = 3,
  kWdExtendBar = 16,
  kWdExtendDrain = 17,
  kWdTileTooLarge = 33,  // a work tile larger than the kernel's tile: clamped
  kWdBadSlot = 32,  // a page id / slot outside the pool: access skipped
  kWdMetaOverflow = 34,  // device metadata: a row, length or entry outside its buffer: skipped
  kWdBadPlan = 35,       // decode plan: a request id or partial slot outside its bounds: segment skipped
};

__device__ __forceinline__ void watchdog_set(int code) { atomicCAS(&g_watchdog, 0, code); }

// Programmatic dependent launch: kernels launched with the programmatic-stream-
// serialization attribute may become resident while the previous kernel of the
// stream still runs. This waits (first, before touching any memory) until that
// kernel has completed and its writes are visible, then lets the next kernel of the
// stream become resident in turn. Without the attribute both are no-ops.
__device__ __forceinline__ void pdl_wait_then_release() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- dtypes
template <typename T>
struct DT;
template <>
struct DT<float> {
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <>
struct DT<__nv_bfloat16> {
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct DT<__half> {
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};

// Load N consecutive elements of T (N * sizeof(T) in {4, 8, 16, 32} bytes,
// naturally aligned) and widen to fp32.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[N]) {
  constexpr int bytes = N * (int)sizeof(T);
  static_assert(bytes % 4 == 0, "vector must be a multiple of 4 bytes");
  if constexpr (sizeof(T) == 4) {
    if constexpr (N % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N / 4; ++i) {
        float4 v = reinterpret_cast<const float4*>(p)[i];
        out[4 * i + 0] = v.x;
        out[4 * i + 1] = v.y;
        out[4 * i + 2] = v.z;
        out[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        float2 v = reinterpret_cast<const float2*>(p)[i];
        out[2 * i + 0] = v.x;
        out[2 * i + 1] = v.y;
      }
    }
  } else {
    // 16-bit types: move as 32-bit words, 2 elements each.
    constexpr int words = N / 2;
    uint32_t w[words];
    if constexpr (words % 4 == 0) {
#pragma unroll
      for (int i = 0; i < words / 4; ++i) {
        uint4 v = reinterpret_cast<const uint4*>(p)[i];
        w[4 * i + 0] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
      }
    } else if constexpr (words % 2 == 0) {
#pragma unroll
      for (int i = 0; i < words / 2; ++i) {
        uint2 v = reinterpret_cast<const uint2*>(p)[i];
        w[2 * i + 0] = v.x;
        w[2 * i + 1] = v.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < words; ++i) w[i] = reinterpret_cast<const uint32_t*>(p)[i];
    }
#pragma unroll
    for (int i = 0; i < words; ++i) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32.
        out[2 * i + 0] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      } else {
        __half2 h = *reinterpret_cast<__half2*>(&w[i]);
        float2 f = __half22float2(h);
        out[2 * i + 0] = f.x;
        out[2 * i + 1] = f.y;
      }
    }
  }
}

// Narrow N fp32 values to T and store them (same alignment rules).
template <typename T, int N>
__device__ __forceinline__ void store_vec(T* __restrict__ p, const float (&in)[N]) {
  if constexpr (sizeof(T) == 4) {
    if constexpr (N % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N / 4; ++i)
        reinterpret_cast<float4*>(p)[i] =
            make_float4(in[4 * i], in[4 * i + 1], in[4 * i + 2], in[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < N / 2; ++i)
        reinterpret_cast<float2*>(p)[i] = make_float2(in[2 * i], in[2 * i + 1]);
    }
  } else {
    constexpr int words = N / 2;
    uint32_t w[words];
#pragma unroll
    for (int i = 0; i < words; ++i) {
      T lo = DT<T>::from_f(in[2 * i]);
      T hi = DT<T>::from_f(in[2 * i + 1]);
      w[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) |
             ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
    }
    if constexpr (words % 4 == 0) {
#pragma unroll
      for (int i = 0; i < words / 4; ++i)
        reinterpret_cast<uint4*>(p)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else if constexpr (words % 2 == 0) {
#pragma unroll
      for (int i = 0; i < words / 2; ++i)
        reinterpret_cast<uint2*>(p)[i] = make_uint2(w[2 * i], w[2 * i + 1]);
    } else {
#pragma unroll
      for (int i = 0; i < words; ++i) reinterpret_cast<uint32_t*>(p)[i] = w[i];
    }
  }
}

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Each try_wait suspends for at most a hardware time slice, so this bounds the
// wait to well under a few seconds. On timeout the watchdog code is recorded
// and false is returned; callers unwind instead of waiting forever.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int wd_code) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  watchdog_set(wd_code);
  return false;
}

// 1-D TMA bulk copy global -> shared, completion counted in bytes on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 policy for data streamed exactly once (the KV pages of a decode step).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Packed fp32 pairs (sm_100 fma/add/mul .f32x2): two lanes of arithmetic per
// instruction, each half rounded exactly like its scalar form.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

}  // namespace b2a
