// Cost of waiting on an mbarrier whose phase has already completed, from
// warps that issue no MMAs (one CTA of 4 warps, 1000 dependent iterations),
// next to a volatile shared-memory poll and a TMEM load. Together with the
// waits between MMA groups in mma_rate.cu this is the fixed cost of each
// hand-off in the extend kernel's S -> softmax -> PV chain.
#include <cstdio>
#include <cstdint>
#include "extend_tc.cuh"
using namespace b2a;
template <int MODE>
__global__ void k(long long* out, int n) {
  __shared__ uint64_t bar[2];
  __shared__ uint32_t slot;
  __shared__ volatile int flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) { mbar_init(&bar[0], 1); fence_mbar_init(); mbar_arrive(&bar[0]); flag = 1; }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&slot)), "r"(32) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = slot;
  long long t0 = clock64();
  int acc = 0;
  for (int i = 0; i < n; ++i) {
    if (MODE == 0) acc += mbar_wait(&bar[0], 0, kWdExtendBar) ? 1 : 0;            // lane-wise try_wait
    if (MODE == 1) acc += __all_sync(0xffffffffu, mbar_wait(&bar[0], 0, kWdExtendBar)) ? 1 : 0;
    if (MODE == 2) acc += flag;                                                   // volatile smem poll
    if (MODE == 3) {                                                              // TMEM load, then wait
      uint32_t u[32];
      tmem_ld32(tmem + ((uint32_t)((warp & 3) * 32) << 16), u);
      tmem_wait_ld();
      acc += (int)(u[0] & 1) + (mbar_wait(&bar[0], 0, kWdExtendBar) ? 1 : 0);
    }
    if (MODE == 4) {                                                              // TMEM load only
      uint32_t u[32];
      tmem_ld32(tmem + ((uint32_t)((warp & 3) * 32) << 16), u);
      tmem_wait_ld();
      acc += (int)(u[0] & 1);
    }
  }
  long long dt = clock64() - t0;
  if (threadIdx.x == 0) out[MODE] = dt / n;
  if (acc == -1) out[7] = acc;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) { tc_fence_after(); asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(32) : "memory"); }
}
int main() {
  long long* d; cudaMalloc(&d, 8 * sizeof(long long)); cudaMemset(d, 0, 8 * sizeof(long long));
  k<0><<<1, 128>>>(d, 1000); k<1><<<1, 128>>>(d, 1000); k<2><<<1, 128>>>(d, 1000); k<3><<<1, 128>>>(d, 1000); k<4><<<1, 128>>>(d, 1000);
  long long h[8]; cudaError_t e = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  printf("ready try_wait %lld clk, __all_sync(try_wait) %lld, volatile smem %lld, tmem ld32+wait %lld, tmem ld32 only %lld (%s)\n",
         h[0], h[1], h[2], h[3], h[4], cudaGetErrorString(e));
  return e != cudaSuccess;
}
