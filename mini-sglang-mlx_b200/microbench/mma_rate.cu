// tcgen05.mma issue rate for the operand shapes of the extend kernel: one CTA
// per SM, one thread issues 8 x rounds MMAs (K = 16 each) on shared-memory /
// TMEM operands that are either zero or random bf16 in +-[1, 2), then waits on
// a commit (bounded). Reports clocks per MMA and MACs per clock per SM.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "extend_tc.cuh"

using namespace b2a;

// MODE 0: SS N=128   1: SS N=64   2: SS N=256   3: TS N=128 (A from TMEM)
//      4: TS N=128 with B MN-major (the PV MMA's V operand)
//      5: the extend kernel's mix: per round 8 SS (S, N=128) then 8 TS B-MN
//         (PV) MMAs into separate TMEM columns
//      6: mode 5 with the kernel's commits (2 after S, 2 after PV)
//      7: SS N=128 with 2 commits after every 8 MMAs
//      8: SS N=128, each group of 8 preceded by a wait on an already
//         completed mbarrier (parity wait that returns at once)
//      9: mode 8 with groups of 4 MMAs
//     10: mode 9 plus tcgen05.fence::after_thread_sync after each wait
//     11: mode 9 polling with mbarrier.test_wait (acquire)
//     12: mode 9 with mbarrier.try_wait.relaxed.cta
//     13: mode 9 polling with mbarrier.test_wait.relaxed.cta
//     14: mode 9 with a volatile shared-memory load instead of the wait
//     15: mode 9 with the wait done by lane 1 of the issuing warp (__syncwarp)
//     16: two issuing warps (lane 0 of warps 0 and 1), SS N=128 into separate
//         TMEM columns, no waits; the time is the later of the two
//     17: mode 16 with a completed-mbarrier wait before every group of 4
template <int MODE>
__global__ void __launch_bounds__(256, 1) mma_rate(int rounds, int random, unsigned long long* cyc, int* err) {
  constexpr int N = MODE == 1 ? 64 : (MODE == 2 ? 256 : 128);
  constexpr bool kMix = MODE == 5 || MODE == 6;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 96 * 1024);
  uint64_t* spare = bar + 2;  // commit targets nobody waits on (modes 6, 7)
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + 96 * 1024 + 64);
  const int warp = threadIdx.x >> 5;
  // A: 32 KB at 0, B: up to 64 KB at 32 KB
  for (int i = threadIdx.x; i < 96 * 1024 / 4; i += blockDim.x) {
    uint32_t v = 0;
    if (random) {
      // two bf16 in +-[1, 2) from an integer hash of the word index
      uint32_t x = (uint32_t)i * 2654435761u + 0x9e3779b9u;
      x ^= x >> 15;
      x *= 0x85ebca6bu;
      x ^= x >> 13;
      v = (0x3f80u | (x & 0x807fu)) | ((0x3f80u | ((x >> 16) & 0x807fu)) << 16);
    }
    reinterpret_cast<uint32_t*>(smem)[i] = v;
  }
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&spare[i], 1);
    fence_mbar_init();
    mbar_arrive(&spare[3]);  // phase 0 of spare[3] completes here: parity-0 waits return at once
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
  if (MODE >= 3 && MODE <= 6) {
    // A operand (64 bf16x2 columns) from the same values, one thread per TMEM lane
    if (warp >= 4) {
      const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
      const uint32_t* src = reinterpret_cast<const uint32_t*>(smem) + (threadIdx.x & 127) * 64;
      for (int c = 0; c < 4; ++c) {
        uint32_t u[16];
        for (int i = 0; i < 16; ++i) u[i] = src[c * 16 + i];
        tmem_st16(tmem + lane_off + 256 + c * 16, u);
      }
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (MODE == 16 || MODE == 17) {
    __syncthreads();  // both issuers start together
    if (threadIdx.x == 0 || threadIdx.x == 32) {
      const int who = threadIdx.x >> 5;
      constexpr uint32_t idesc = tc_idesc(false, 128);
      const uint32_t sA = smem_u32(smem), sB = smem_u32(smem + 32 * 1024);
      const unsigned long long t0 = clock64();
      for (int r = 0; r < rounds; ++r) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          if (MODE == 17 && (kk & 3) == 0 && !mbar_wait(&spare[3], 0, kWdExtendBar)) atomicExch(err, 2);
          const uint64_t ad = sw128_desc(sA + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(sB + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          tc_mma_f16(tmem + who * 256 + (r & 1) * 128, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
      }
      tc_commit(&spare[who]);
      if (!mbar_wait(&spare[who], 0, kWdExtendBar)) atomicExch(err, 1);
      const unsigned long long dt = clock64() - t0;
      atomicMax(&cyc[blockIdx.x], dt);
    }
  } else if (MODE == 15 && threadIdx.x == 1) {
    for (int r = 0; r < rounds; ++r)
      for (int g = 0; g < 2; ++g) {
        if (!mbar_wait(&spare[3], 0, kWdExtendBar)) atomicExch(err, 2);
        __syncwarp(3u);
      }
  }
  if (threadIdx.x == 0 && MODE != 16 && MODE != 17) {
    constexpr uint32_t idesc = tc_idesc(MODE == 4, N);
    const uint32_t sA = smem_u32(smem), sB = smem_u32(smem + 32 * 1024);
    const unsigned long long t0 = clock64();
    for (int r = 0; r < rounds; ++r) {
      if (kMix) {
        constexpr uint32_t idesc_pv = tc_idesc(true, 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sw128_desc(sA + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(sB + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          tc_mma_f16(tmem + 128, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        if (MODE == 6) {
          tc_commit(&spare[0]);
          tc_commit(&spare[1]);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16_ts(tmem + 384, tmem + 256 + kk * 8, sw128_desc(sB + kk * 2048, 16384, 1024), idesc_pv,
                        (r > 0 || kk > 0) ? 1u : 0u);
        if (MODE == 6) {
          tc_commit(&spare[2]);
          tc_commit(&spare[3]);
        }
        continue;
      }
      if (MODE >= 8) {
        constexpr int group = MODE == 8 ? 8 : 4;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          if (kk % group == 0) {
            const uint32_t ba = smem_u32(&spare[3]);
            uint32_t done = 0;
            if (MODE == 8 || MODE == 9 || MODE == 10) {
              done = mbar_wait(&spare[3], 0, kWdExtendBar);
            } else if (MODE == 11) {
              for (int it = 0; it < (1 << 20) && !done; ++it)
                asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                             "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(ba), "r"(0) : "memory");
            } else if (MODE == 12) {
              for (int it = 0; it < (1 << 20) && !done; ++it)
                asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.relaxed.cta.shared::cta.b64 p, [%1], %2;\n\t"
                             "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(ba), "r"(0) : "memory");
            } else if (MODE == 13) {
              for (int it = 0; it < (1 << 20) && !done; ++it)
                asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.relaxed.cta.shared::cta.b64 p, [%1], %2;\n\t"
                             "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(ba), "r"(0) : "memory");
            } else if (MODE == 14) {
              done = *reinterpret_cast<volatile uint32_t*>(&spare[3]) != 0xffffffffu;
            } else {
              __syncwarp(3u);
              done = 1;
            }
            if (!done) atomicExch(err, 2);
            if (MODE == 10) tc_fence_after();
          }
          const uint64_t ad = sw128_desc(sA + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(sB + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          tc_mma_f16(tmem + (r & 1) * 128, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        continue;
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t ad = sw128_desc(sA + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = MODE == 4 ? sw128_desc(sB + kk * 2048, 16384, 1024)
                                      : sw128_desc(sB + (kk >> 2) * (N * 128) + (kk & 3) * 32, 16, 1024);
        if (MODE == 3 || MODE == 4)
          tc_mma_f16_ts(tmem + (r & 1) * 128, tmem + 256 + kk * 8, bd, idesc, kk > 0 ? 1u : 0u);
        else
          tc_mma_f16(tmem + (MODE == 2 ? 0 : (r & 1) * 128), ad, bd, idesc, kk > 0 ? 1u : 0u);
      }
      if (MODE == 7) {
        tc_commit(&spare[0]);
        tc_commit(&spare[1]);
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
static void run(const char* name, unsigned long long* d, int* err, int sms, int rounds, int random) {
  constexpr int N = MODE == 1 ? 64 : (MODE == 2 ? 256 : 128);
  auto k = mma_rate<MODE>;
  const int smem = 120 * 1024;  // one CTA per SM, so each owns all 512 TMEM columns
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  k<<<sms, 256, smem>>>(8, random, d, err);
  cudaMemset(d, 0, sizeof(unsigned long long) * sms);  // modes 16, 17 take the max of two issuers
  k<<<sms, 256, smem>>>(rounds, random, d, err);
  cudaDeviceSynchronize();
  unsigned long long h[1024];
  cudaMemcpy(h, d, sizeof(unsigned long long) * sms, cudaMemcpyDeviceToHost);
  double avg = 0;
  for (int i = 0; i < sms; ++i) avg += (double)h[i];
  avg /= sms;
  const double per_round = (MODE == 5 || MODE == 6 || MODE == 16 || MODE == 17) ? 16.0 : 8.0;
  const double macs = 128.0 * N * 16 * per_round * rounds;
  printf("%-16s %-6s %6.1f clk per MMA (K=16)  %6.0f MAC/clk/SM\n", name, random ? "random" : "zeros",
         avg / (per_round * rounds), macs / avg);
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
  for (int random = 0; random < 2; ++random) {
    run<0>("SS N=128", d, err, sms, 2000, random);
    run<1>("SS N=64", d, err, sms, 2000, random);
    run<2>("SS N=256", d, err, sms, 2000, random);
    run<3>("TS N=128", d, err, sms, 2000, random);
    run<4>("TS N=128 B-MN", d, err, sms, 2000, random);
  }
  run<5>("SS/TS mix", d, err, sms, 2000, 1);
  run<6>("SS/TS mix+commit", d, err, sms, 2000, 1);
  run<7>("SS+commit", d, err, sms, 2000, 1);
  run<8>("SS wait/8", d, err, sms, 2000, 1);
  run<9>("SS wait/4", d, err, sms, 2000, 1);
  run<10>("SS wait+fence/4", d, err, sms, 2000, 1);
  run<11>("SS testwait/4", d, err, sms, 2000, 1);
  run<12>("SS relaxed/4", d, err, sms, 2000, 1);
  run<13>("SS test.rlx/4", d, err, sms, 2000, 1);
  run<14>("SS ld.vol/4", d, err, sms, 2000, 1);
  run<15>("SS lane1wait/4", d, err, sms, 2000, 1);
  run<16>("2 issuers", d, err, sms, 2000, 1);
  run<17>("2 issuers wait/4", d, err, sms, 2000, 1);
  int h = 0;
  cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
  const cudaError_t e = cudaDeviceSynchronize();
  printf("wait timeouts %d, status %s\n", h, cudaGetErrorString(e));
  return (e != cudaSuccess || h) ? 1 : 0;
}
