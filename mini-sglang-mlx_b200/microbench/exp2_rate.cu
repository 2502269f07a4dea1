// Throughput of 2^x variants per SM per clock on the MUFU and FMA pipes.
// Pure register arithmetic: 8 independent chains per thread, 4 CTAs of 512
// threads per SM, one float stored per thread at the end. The results size
// the softmax of the extend kernel (extend_tc.cuh): a 128-key block of both
// Q tiles needs 32768 exponentials per CTA.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t ex2b(uint32_t x) {
  uint32_t y;
  asm volatile("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2s(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Packed 2^x on the FMA pipe: n = round(x) from the low bits of x + 1.5*2^23,
// f = x - n in [-1/2, 1/2], 2^f by a cubic fitted by least squares to the
// relative error on [-1/2, 1/2] (max 1.8e-4), 2^n added into the exponent.
__device__ __forceinline__ void ex2poly2(float& a0, float& a1) {
  const uint64_t x = f2(fmaxf(a0, -126.f), fmaxf(a1, -126.f));
  const uint64_t t = f2add(x, f2(12582912.f, 12582912.f));
  const uint64_t f = f2fma(f2add(t, f2(-12582912.f, -12582912.f)), f2(-1.f, -1.f), x);
  uint64_t p = f2fma(f, f2(0.0546027f, 0.0546027f), f2(0.24192398f, 0.24192398f));
  p = f2fma(p, f, f2(0.69331645f, 0.69331645f));
  p = f2fma(p, f, f2(1.f, 1.f));
  float p0, p1, t0, t1;
  f2s(p, p0, p1);
  f2s(t, t0, t1);
  a0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  a1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Two fp32 -> bf16x2 (round to nearest even) with integer ops and a byte
// permute: no conversion instruction.
__device__ __forceinline__ uint32_t pack_int(float lo, float hi) {
  uint32_t a = __float_as_uint(lo), b = __float_as_uint(hi);
  a += 0x7fffu + ((a >> 16) & 1u);
  b += 0x7fffu + ((b >> 16) & 1u);
  return __byte_perm(a, b, 0x7632);
}
__device__ __forceinline__ uint32_t pack_cvt(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// MODE 0: ex2.f32   1: ex2.bf16x2 (2 results each)   2: packed polynomial   3: 1:1 MUFU / polynomial
//      4: ex2.f32 + one cvt.rn.bf16x2.f32 per two results (the softmax's P pack)
//      5: ex2.f32 + one integer pack per two results
template <int MODE>
__global__ void rate(float* out, int iters, float seed) {
  float a[8];
  uint32_t b[8];
  for (int i = 0; i < 8; ++i) {
    a[i] = -0.001f * (threadIdx.x + i) + seed;
    b[i] = 0x3c003c00u + i;
  }
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (MODE == 0) a[i] = ex2f(a[i]) - 1.0f;
      if (MODE == 4 || MODE == 5) {
        a[i] = ex2f(a[i]) - 1.0f;
        if (i & 1) b[i] ^= MODE == 4 ? pack_cvt(a[i - 1], a[i]) : pack_int(a[i - 1], a[i]);
      }
      if (MODE == 1) b[i] = ex2b(b[i]) ^ 0x80008000u;
      if (MODE == 2 && (i & 1)) {
        ex2poly2(a[i - 1], a[i]);
        a[i - 1] -= 1.0f;
        a[i] -= 1.0f;
      }
      if (MODE == 3) {
        if ((i & 3) == 3) {
          ex2poly2(a[i - 1], a[i]);
          a[i - 1] -= 1.0f;
          a[i] -= 1.0f;
        } else if ((i & 3) < 2) {
          a[i] = ex2f(a[i]) - 1.0f;
        }
      }
    }
  }
  float s = 0;
  for (int i = 0; i < 8; ++i) s += a[i] + (float)(b[i] & 1);
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

template <int MODE>
static int run(const char* name, float* d, int sms, int iters, double per_instr) {
  const int blocks = sms * 4, threads = 512;
  rate<MODE><<<blocks, threads>>>(d, 16, 0.f);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0);
  rate<MODE><<<blocks, threads>>>(d, iters, 0.f);
  cudaEventRecord(e1);
  if (cudaEventSynchronize(e1) != cudaSuccess) return 1;
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  int khz = 0;
  cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, 0);
  const double results = (double)blocks * threads * iters * 8 * per_instr;
  printf("%-22s %8.3f ms  %6.2f results/clk/SM (at the %d MHz max clock)\n", name, ms,
         results / (ms * 1e-3) / (khz * 1e3) / sms, khz / 1000);
  return 0;
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  float* d = nullptr;
  if (cudaMalloc(&d, sizeof(float) * sms * 4 * 512) != cudaSuccess) return 1;
  int rc = 0;
  rc |= run<0>("ex2.approx.ftz.f32", d, sms, 4096, 1.0);
  rc |= run<1>("ex2.approx.ftz.bf16x2", d, sms, 4096, 2.0);
  rc |= run<2>("packed polynomial", d, sms, 4096, 1.0);
  rc |= run<3>("MUFU:polynomial 1:1", d, sms, 4096, 1.0);
  rc |= run<4>("ex2 + cvt bf16x2 pack", d, sms, 4096, 1.0);
  rc |= run<5>("ex2 + integer pack", d, sms, 4096, 1.0);
  cudaError_t e = cudaDeviceSynchronize();
  printf("status %s\n", cudaGetErrorString(e));
  cudaFree(d);
  return rc || e != cudaSuccess;
}
