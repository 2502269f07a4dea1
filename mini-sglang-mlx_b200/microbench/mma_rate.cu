// tcgen05.mma issue rate for the operand shapes of the extend kernel: one CTA
// per SM, one thread issues 8 x rounds MMAs (K = 16 each) on zero-filled
// shared-memory / TMEM operands, then waits on a commit (bounded). Reports
// clocks per MMA and MACs per clock per SM.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "extend_tc.cuh"

using namespace b2a;

// MODE 0: SS N=128   1: SS N=64   2: SS N=256   3: TS N=128 (A from TMEM)
template <int MODE>
__global__ void __launch_bounds__(256, 1) mma_rate(int rounds, unsigned long long* cyc, int* err) {
  constexpr int N = MODE == 1 ? 64 : (MODE == 2 ? 256 : 128);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 96 * 1024);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + 96 * 1024 + 64);
  const int warp = threadIdx.x >> 5;
  // A: 32 KB at 0, B: up to 64 KB at 32 KB
  for (int i = threadIdx.x; i < 96 * 1024 / 16; i += blockDim.x) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = tc_idesc(false, N);
    const uint32_t sA = smem_u32(smem), sB = smem_u32(smem + 32 * 1024);
    const unsigned long long t0 = clock64();
    for (int r = 0; r < rounds; ++r) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t ad = sw128_desc(sA + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = sw128_desc(sB + (kk >> 2) * (N * 128) + (kk & 3) * 32, 16, 1024);
        if (MODE == 3)
          tc_mma_f16_ts(tmem + (r & 1) * 128, tmem + 256 + kk * 8, bd, idesc, kk > 0 ? 1u : 0u);
        else
          tc_mma_f16(tmem + (MODE == 2 ? 0 : (r & 1) * 128), ad, bd, idesc, kk > 0 ? 1u : 0u);
      }
    }
    tc_commit(bar);
    const bool ok = mbar_wait(bar, 0, kWdExtendBar);
    cyc[blockIdx.x] = clock64() - t0;
    if (!ok) atomicExch(err, 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

template <int MODE>
static void run(const char* name, unsigned long long* d, int* err, int sms, int rounds) {
  constexpr int N = MODE == 1 ? 64 : (MODE == 2 ? 256 : 128);
  auto k = mma_rate<MODE>;
  const int smem = 120 * 1024;  // one CTA per SM, so each owns all 512 TMEM columns
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  k<<<sms, 256, smem>>>(8, d, err);
  k<<<sms, 256, smem>>>(rounds, d, err);
  cudaDeviceSynchronize();
  unsigned long long h[1024];
  cudaMemcpy(h, d, sizeof(unsigned long long) * sms, cudaMemcpyDeviceToHost);
  double avg = 0;
  for (int i = 0; i < sms; ++i) avg += (double)h[i];
  avg /= sms;
  const double macs = 128.0 * N * 16 * 8 * rounds;
  printf("%-12s %6.1f clk per MMA (K=16)  %6.0f MAC/clk/SM\n", name, avg / (8.0 * rounds), macs / avg);
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  if (sms <= 0 || sms > 1024) return 1;
  unsigned long long* d = nullptr;
  int* err = nullptr;
  if (cudaMalloc(&d, sizeof(unsigned long long) * sms) != cudaSuccess || cudaMalloc(&err, sizeof(int)) != cudaSuccess)
    return 1;
  cudaMemset(err, 0, sizeof(int));
  run<0>("SS N=128", d, err, sms, 2000);
  run<1>("SS N=64", d, err, sms, 2000);
  run<2>("SS N=256", d, err, sms, 2000);
  run<3>("TS N=128", d, err, sms, 2000);
  int h = 0;
  cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
  const cudaError_t e = cudaDeviceSynchronize();
  printf("wait timeouts %d, status %s\n", h, cudaGetErrorString(e));
  return (e != cudaSuccess || h) ? 1 : 0;
}
