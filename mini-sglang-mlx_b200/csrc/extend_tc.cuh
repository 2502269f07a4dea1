// Ragged causal extend attention on 5th-generation tensor cores (sm_100a).
//
// Reference: python/minisgl_mlx/attention/base.py:70-105 (per-request SDPA,
// bottom-right causal). Same contract as extend_simt.cuh; this is the
// bf16 / head_dim 128 / page_size % 16 == 0 path.
//
// A 128-row MMA tile packs 128/G query tokens x the G query heads of one kv
// head (row = token * G + g), so a pass over that head's K/V serves the whole
// GQA group. A CTA owns two such tiles of one request (see extend_tc2_kernel)
// and streams the request's K/V once for both: K and V blocks of 128 keys
// are gathered page by page with 16-row SWIZZLE_128B TMA boxes from a 3-D
// tensor map over the pool (keys past the sequence use an out-of-range
// coordinate and arrive as zeros). S and O live in TMEM; the softmax
// threads own one TMEM lane (= tile row) each, so row max and row sum need
// no cross-thread reduction, and write P (bf16) back into TMEM for the
// A-from-TMEM PV MMA. The running max only moves when it grows by more than
// 8 (log2 units); otherwise p = 2^(s - m_stale) <= 256 keeps the fp32
// accumulation exact and O is not rescaled.
// Every mbarrier wait is bounded; a wait that gives up records a watchdog
// code, the roles unwind, in-flight copies and MMAs are drained (bounded) and
// TMEM is released before the CTA exits.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include <string>

#include "common.cuh"

namespace b2a {

constexpr int kTcRows = 128;      // query rows (tokens x GQA heads) per CTA tile
constexpr int kTcKeys = 128;      // keys per K/V block
constexpr int kTcD = 128;         // head_dim handled by this kernel
constexpr uint32_t kTcTileBytes = 128 * 128 * 2;  // one 128x128 bf16 tile (32 KB)
constexpr uint32_t kTcHalfBytes = kTcTileBytes / 2;  // one 64-column SW128 half (16 KB)

struct TcArgs {
  const int32_t* qo_indptr;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* kv_last_page_len;
  const int32_t* work;
  __nv_bfloat16* out;
  int64_t num_slots;
  int64_t stage_slots;  // rows of the staging pool (group-start mode)
  int page_log2;
  int group_starts;     // kv_indices hold each 16-key group's first slot, not page ids
  int Hq, G;
  float qscale;  // scale * log2(e)
};

// ------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

#define B2A_R32(X) \
  "=r"(X[0]), "=r"(X[1]), "=r"(X[2]), "=r"(X[3]), "=r"(X[4]), "=r"(X[5]), "=r"(X[6]), "=r"(X[7]), "=r"(X[8]), \
      "=r"(X[9]), "=r"(X[10]), "=r"(X[11]), "=r"(X[12]), "=r"(X[13]), "=r"(X[14]), "=r"(X[15]), "=r"(X[16]), \
      "=r"(X[17]), "=r"(X[18]), "=r"(X[19]), "=r"(X[20]), "=r"(X[21]), "=r"(X[22]), "=r"(X[23]), "=r"(X[24]), \
      "=r"(X[25]), "=r"(X[26]), "=r"(X[27]), "=r"(X[28]), "=r"(X[29]), "=r"(X[30]), "=r"(X[31])
#define B2A_W32(X) \
  "r"(X[0]), "r"(X[1]), "r"(X[2]), "r"(X[3]), "r"(X[4]), "r"(X[5]), "r"(X[6]), "r"(X[7]), "r"(X[8]), "r"(X[9]), \
      "r"(X[10]), "r"(X[11]), "r"(X[12]), "r"(X[13]), "r"(X[14]), "r"(X[15]), "r"(X[16]), "r"(X[17]), "r"(X[18]), \
      "r"(X[19]), "r"(X[20]), "r"(X[21]), "r"(X[22]), "r"(X[23]), "r"(X[24]), "r"(X[25]), "r"(X[26]), "r"(X[27]), \
      "r"(X[28]), "r"(X[29]), "r"(X[30]), "r"(X[31])

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : B2A_R32(r)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      B2A_W32(r)
      : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, SWIZZLE_128B (sm_100 encoding: version 1 at
// bits 46-47, layout type 2 at bits 61-63). K-major tiles are rows of 128 B,
// 8-row groups 1024 B apart (SBO); MN-major tiles add LBO = distance between
// 64-element column chunks.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> fp32, M=128, N=n.
__host__ __device__ constexpr uint32_t tc_idesc(bool b_mn_major, int n = 128) {
  return (1u << 4)                          // D format fp32
         | (1u << 7)                        // A bf16
         | (1u << 10)                       // B bf16
         | ((b_mn_major ? 1u : 0u) << 16)   // B major
         | ((uint32_t)(n >> 3) << 17)       // N
         | ((uint32_t)(128 >> 4) << 24);    // M
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity, kWdExtendBar)) return true;
  *abort_flag = 1;
  return false;
}

// ------------------------------------------------------------ v2: two Q tiles, P in TMEM
//
// CTA = (work item of up to 2 x 128/G query tokens, kv head h). Tile 0 holds
// the first 128/G tokens, tile 1 the rest; both read the same K/V blocks.
//   warp 0     TMA producer (Q0, Q1 once; K and V blocks through 2-deep rings)
//   warp 1     MMA issuer: S_t = Q_t K^T (SS, M=128 N=128), O_t += P_t V (A = P
//              from TMEM, B = V MN-major from shared memory)
//   warp 2     TMEM allocator: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512);
//              P_t (bf16, 64 columns) is written over the first half of S_t
//   warps 4-7  softmax of tile 0, warps 8-11 softmax of tile 1 (one thread
//              per TMEM lane = tile row)
// MMA issue order per block j: PV0(j), S0(j+1), PV1(j), S1(j+1). tcgen05 MMAs
// of one thread complete in order and a commit covers every earlier MMA, so
// s_full[t] for block j+1 also means PV_t(j) has finished: P_t may be
// overwritten and O_t may be rescaled by the softmax warps of tile t without
// waiting on anything else, and S_t(j+1) never overwrites a P_t still in use.
// The softmax releases P_t(j) in two halves (keys 0-63, then 64-127; one
// mbarrier each), so the first four PV MMAs of the tile can run while it
// finishes the block.
// The single issuing thread is what bounds this kernel: the tensor pipe keeps
// no queue of its MMAs, so every instruction between two MMA groups is idle
// pipe time, and an mbarrier wait costs ~110-240 clk even on a completed phase
// (in-kernel clock stamps: the issuer spends ~3300 clk per block on 24 MMAs
// worth 1536 clk, while the softmax warps idle ~1800 clk per block). Each
// release therefore also bumps a shared-memory count after the arrive; the
// issuer first reads the second half's count with one acquire load (~40 clk)
// and, when both halves are written, issues all eight PV MMAs with no wait.
// Only a P that is not ready yet costs an mbarrier wait (a suspended thread,
// not a spin that would take issue slots from the softmax warps).
constexpr int kTc2Threads = 384;

struct Tc2Smem {
  static constexpr uint32_t Q0 = 0;
  static constexpr uint32_t Q1 = Q0 + kTcTileBytes;
  static constexpr uint32_t K0 = Q1 + kTcTileBytes;
  static constexpr uint32_t V0 = K0 + 2 * kTcTileBytes;
  static constexpr uint32_t BARS = V0 + 2 * kTcTileBytes;
  // q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], (2 spare), mma_done,
  // p_full[2 tiles] x 4 slots (2 halves used): spacing keeps the words the
  // softmax warps arrive on apart from the s_full words they poll (measured ~1%)
  static constexpr int NBARS = 22;
  static constexpr uint32_t TMEM_SLOT = BARS + NBARS * 8;
  static constexpr uint32_t ABORT = TMEM_SLOT + 8;
  static constexpr uint32_t PCNT = ABORT + 8;  // u32 [8]: P releases counted per (tile, half)
  static constexpr uint32_t TOTAL = PCNT + 32;
  static constexpr uint32_t ALLOC = TOTAL + 1024;
};

__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (f2, f2_split, f2_fma, f2_add, in common.cuh) and the
// 3-input max: fewer instructions on the softmax's critical path.
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

__global__ void __launch_bounds__(kTc2Threads, 1)
    extend_tc2_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap kmap2,
                      const __grid_constant__ CUtensorMap vmap2, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Tc2Smem::BARS);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2] per tile
  uint64_t* p_full = bars + 14;   // [tile * 4 + half]: P columns of that half written
  uint64_t* mma_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Tc2Smem::TMEM_SLOT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Tc2Smem::ABORT);
  uint32_t* pcnt = reinterpret_cast<uint32_t*>(smem + Tc2Smem::PCNT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.G;
  const int TT = kTcRows / G;  // tokens per tile
  const int4 w = reinterpret_cast<const int4*>(a.work)[blockIdx.y];
  const int r = w.x, tb = w.y;
  const int nq = min(w.z, 2 * TT);
  if (w.z > nq && threadIdx.x == 0) watchdog_set(kWdTileTooLarge);
  const int nq_t[2] = {min(nq, TT), max(0, nq - TT)};
  const int h = blockIdx.x;
  const int P = 1 << a.page_log2;
  const int q0 = a.qo_indptr[r];
  const int Lq = a.qo_indptr[r + 1] - q0;
  const int pbeg = a.kv_indptr[r];
  const int npages = a.kv_indptr[r + 1] - pbeg;
  const int Lkv = npages > 0 ? ((npages - 1) << a.page_log2) + (a.kv_last_page_len ? a.kv_last_page_len[r] : P) : 0;
  const int prefix = Lkv - Lq;
  // keys visible to the last row of each tile, and the blocks each tile needs
  int nb_t[2];
  for (int t = 0; t < 2; ++t) {
    const int kv_end = nq_t[t] > 0 ? min(Lkv, prefix + tb + t * TT + nq_t[t]) : 0;
    nb_t[t] = (kv_end + kTcKeys - 1) / kTcKeys;
  }
  const int nb = max(nb_t[0], nb_t[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      for (int c = 0; c < 2; ++c) mbar_init(&p_full[i * 4 + c], 4);  // one arrive per softmax warp
    }
    mbar_init(mma_done, 1);
    for (int i = 0; i < 8; ++i) pcnt[i] = 0;
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    int issued_k = 0, issued_v = 0;
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * kTcTileBytes);
      for (int t = 0; t < 2; ++t) {
        // tile 1 rows past the request (or the tensor) load as zeros / stay unused
        tma_load_3d(smem + Tc2Smem::Q0 + t * kTcTileBytes, &qmap, 0, h * G, q0 + tb + t * TT, q_full);
        tma_load_3d(smem + Tc2Smem::Q0 + t * kTcTileBytes + kTcHalfBytes, &qmap, 64, h * G, q0 + tb + t * TT, q_full);
      }
    }
    for (int j = 0; j < nb; ++j) {
      const int st = j & 1;
      const uint32_t ph = (uint32_t)(j >> 1) & 1u;
      int z = (int)a.num_slots;  // out of range -> zero fill
      bool staged = false;       // this lane's group comes from the staging pool
      const int b = lane >> 1, half = lane & 1;
      if (lane < 16) {
        const int key0 = j * kTcKeys + b * 16;
        if (key0 < Lkv) {
          const int64_t e = a.kv_indices[pbeg + (key0 >> a.page_log2)];
          if (a.group_starts) {
            // the group's 16 rows start at slot e of the pool, or at e - num_slots of the
            // staging pool; rows past a pool's end load as zeros (keys past Lkv are masked)
            if (e >= 0 && e < a.num_slots) {
              z = (int)e;
            } else if (e >= a.num_slots && e - a.num_slots < a.stage_slots) {
              z = (int)(e - a.num_slots);
              staged = true;
            } else {
              watchdog_set(kWdBadSlot);
            }
          } else {
            const int64_t slot = e * P + (key0 & (P - 1));
            if (e >= 0 && slot + 16 <= a.num_slots) z = (int)slot;
            else watchdog_set(kWdBadSlot);
          }
        }
      }
      bool ok = __all_sync(0xffffffffu, tc_wait(&k_empty[st], ph ^ 1u, abort_flag));
      if (!ok) break;
      if (lane == 0) mbar_arrive_expect_tx(&k_full[st], kTcTileBytes);
      __syncwarp();
      if (lane < 16)
        tma_load_3d(smem + Tc2Smem::K0 + st * kTcTileBytes + half * kTcHalfBytes + b * 2048, staged ? &kmap2 : &kmap,
                    half * 64, h, z, &k_full[st]);
      ++issued_k;
      ok = __all_sync(0xffffffffu, tc_wait(&v_empty[st], ph ^ 1u, abort_flag));
      if (!ok) break;
      if (lane == 0) mbar_arrive_expect_tx(&v_full[st], kTcTileBytes);
      __syncwarp();
      if (lane < 16)
        tma_load_3d(smem + Tc2Smem::V0 + st * kTcTileBytes + half * kTcHalfBytes + b * 2048, staged ? &vmap2 : &vmap,
                    half * 64, h, z, &v_full[st]);
      ++issued_v;
    }
    if (lane == 0) {
      mbar_wait(q_full, 0, kWdExtendDrain);
      for (int i = max(0, issued_k - 2); i < issued_k; ++i) mbar_wait(&k_full[i & 1], (uint32_t)(i >> 1) & 1u, kWdExtendDrain);
      for (int i = max(0, issued_v - 2); i < issued_v; ++i) mbar_wait(&v_full[i & 1], (uint32_t)(i >> 1) & 1u, kWdExtendDrain);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = tc_idesc(false);
      constexpr uint32_t idesc_pv = tc_idesc(true);
      bool ok = tc_wait(q_full, 0, abort_flag);
      auto issue_s = [&](int t, int j) {
        const uint32_t sQ = smem_u32(smem + Tc2Smem::Q0 + t * kTcTileBytes);
        const uint32_t sK = smem_u32(smem + Tc2Smem::K0 + (j & 1) * kTcTileBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sw128_desc(sQ + (kk >> 2) * kTcHalfBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(sK + (kk >> 2) * kTcHalfBytes + (kk & 3) * 32, 16, 1024);
          tc_mma_f16(tmem + t * 128, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[t]);
      };
      // P(j) of (tile, half) released by all 4 softmax warps: an acquire load of
      // the release count (~40 clk) instead of an mbarrier wait (~160 clk)
      auto p_done = [&](int idx, int j) -> bool {
        uint32_t v;
        asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(&pcnt[idx])) : "memory");
        return v >= 4u * (uint32_t)(j + 1);
      };
      // PV K-steps 4 half .. 4 half + 3 read the P columns of one half
      auto issue_pv = [&](int t, int j, int half) {
        const uint32_t sV = smem_u32(smem + Tc2Smem::V0 + (j & 1) * kTcTileBytes);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int kk = half * 4 + q;
          const uint64_t bd = sw128_desc(sV + kk * 2048, kTcHalfBytes, 1024);
          tc_mma_f16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      if (ok && nb > 0) {
        ok = tc_wait(&k_full[0], 0, abort_flag);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < 2; ++t)
            if (nb_t[t] > 0) issue_s(t, 0);
          tc_commit(&k_empty[0]);
        }
      }
      for (int j = 0; j < nb && ok; ++j) {
        if (!tc_wait(&v_full[j & 1], (uint32_t)(j >> 1) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        const bool more = j + 1 < nb;
        bool k_next = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j < nb_t[t]) {
            if (p_done(t * 4 + 1, j)) {
              tc_fence_after();
              issue_pv(t, j, 0);
              issue_pv(t, j, 1);
            } else {
              for (int half = 0; half < 2 && ok; ++half) {
                if (!p_done(t * 4 + half, j) && !tc_wait(&p_full[t * 4 + half], (uint32_t)j & 1u, abort_flag)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
                issue_pv(t, j, half);
              }
            }
            if (!ok) break;
          }
          if (more && j + 1 < nb_t[t]) {
            if (!k_next) {
              if (!tc_wait(&k_full[(j + 1) & 1], (uint32_t)((j + 1) >> 1) & 1u, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              k_next = true;
            }
            issue_s(t, j + 1);
          }
        }
        if (!ok) break;
        tc_commit(&v_empty[j & 1]);
        if (more) tc_commit(&k_empty[(j + 1) & 1]);
      }
      // every MMA issued above has completed once mma_done fires (also on the abort path)
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, kWdExtendDrain);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- softmax + epilogue
    constexpr unsigned FULL = 0xffffffffu;
    const int t = (warp - 4) >> 2;  // tile of this warpgroup
    const int row = (threadIdx.x - 128) & 127;  // TMEM lane = tile row
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + t * 128 + lane_off;
    const uint32_t tO = tmem + 256 + t * 128 + lane_off;
    const int tok = row / G;
    const int qpos = prefix + tb + t * TT + tok;
    const int lim_abs = min(qpos, Lkv - 1);  // last visible key of this row
    float m = kNegInf, l = 0.f;
    bool ok = true;
    const int my_nb = nb_t[t];
    for (int j = 0; j < my_nb; ++j) {
      ok = __all_sync(FULL, tc_wait(&s_full[t], (uint32_t)j & 1u, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int limit = lim_abs - j * kTcKeys;  // columns 0..limit are visible
      const bool full = limit >= kTcKeys - 1;
      // pass 1: raw row max over the visible columns; two TMEM loads per round
      // trip, 8 independent 3-input max chains
      float mxs[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxs[i] = kNegInf;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t ua[32], ub[32];
        tmem_ld32(tS + half * 64, ua);
        tmem_ld32(tS + half * 64 + 32, ub);
        tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (half * 64 + i > limit) ua[i] = __float_as_uint(kNegInf);
            if (half * 64 + 32 + i > limit) ub[i] = __float_as_uint(kNegInf);
          }
        }
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          mxs[(i >> 2) & 7] = max3f(mxs[(i >> 2) & 7], __uint_as_float(ua[i]), __uint_as_float(ua[i + 1]));
          mxs[(i >> 2) & 7] = max3f(mxs[(i >> 2) & 7], __uint_as_float(ua[i + 2]), __uint_as_float(ua[i + 3]));
          mxs[(i >> 2) & 7] = max3f(mxs[(i >> 2) & 7], __uint_as_float(ub[i]), __uint_as_float(ub[i + 1]));
          mxs[(i >> 2) & 7] = max3f(mxs[(i >> 2) & 7], __uint_as_float(ub[i + 2]), __uint_as_float(ub[i + 3]));
        }
      }
      const float mx = fmaxf(max3f(mxs[0], mxs[1], mxs[2]), fmaxf(max3f(mxs[3], mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
      const float m_blk = mx * a.qscale;  // scale > 0 keeps the order
      float alpha = 1.f;
      if (m == kNegInf) {
        m = m_blk;
      } else if (m_blk - m > 8.f) {
        alpha = ex2_approx(m - m_blk);
        m = m_blk;
      }
      // O_t is stable here: s_full for this block implies PV_t of the previous block finished
      if (j > 0 && __any_sync(FULL, alpha != 1.f)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t u[32];
          tmem_ld32(tO + c * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
          tmem_st32(tO + c * 32, u);
        }
      }
      // pass 2: p = 2^(s*scale - m) (one packed FMA per pair), packed to bf16
      // pairs over the first 64 columns of S; the next chunk's load is in
      // flight while a chunk is processed; 4 independent packed row sums.
      const uint64_t sc2 = f2(a.qscale, a.qscale);
      const uint64_t nm2 = f2(-m, -m);
      uint64_t ps2[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
      uint32_t ua[32], ub[32];
      tmem_ld32(tS, ua);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t(&cur)[32] = (c & 1) ? ub : ua;
        uint32_t(&nxt)[32] = (c & 1) ? ua : ub;
        if (c < 3) tmem_ld32(tS + (c + 1) * 32, nxt);
        uint32_t pk[16];
        float xv[32];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          f2_split(f2_fma(f2(__uint_as_float(cur[2 * i]), __uint_as_float(cur[2 * i + 1])), sc2, nm2), xv[2 * i], xv[2 * i + 1]);
#pragma unroll
        for (int i = 0; i < 32; ++i) xv[i] = ex2_approx(xv[i]);
        if (!full) {
#pragma unroll
          for (int i = 0; i < 32; ++i) xv[i] = (c * 32 + i <= limit) ? xv[i] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          ps2[i & 3] = f2_add(ps2[i & 3], f2(xv[2 * i], xv[2 * i + 1]));
          pk[i] = pack_bf16x2(xv[2 * i], xv[2 * i + 1]);
        }
        // P columns [16c, 16c+16): every S column below 32(c+1) has been read
        tmem_st16(tS + c * 16, pk);
        if (c & 1) {
          // release this half of P to the PV MMA while the rest is computed
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            // the arrive first, then the counted release: a reader that sees the
            // count also sees the barrier phase complete
            mbar_arrive(&p_full[t * 4 + (c >> 1)]);
            asm volatile("red.release.cta.shared::cta.add.u32 [%0], 1;" ::"r"(smem_u32(&pcnt[t * 4 + (c >> 1)])) : "memory");
          }
        }
        if (c < 3) tmem_wait_ld();
      }
      float psum;
      {
        const uint64_t s01 = f2_add(f2_add(ps2[0], ps2[1]), f2_add(ps2[2], ps2[3]));
        float lo, hi;
        f2_split(s01, lo, hi);
        psum = lo + hi;
      }
      l = l * alpha + psum;
    }
    // ---- epilogue: O_t / l -> bf16 rows of the output
    const bool got = __all_sync(FULL, mbar_wait(mma_done, 0, kWdExtendBar));
    tc_fence_after();
    if (ok && got && my_nb > 0) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int g = row - tok * G;
      __nv_bfloat16* dst = a.out + ((size_t)(q0 + tb + t * TT + tok) * a.Hq + h * G + g) * kTcD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t u[32];
        tmem_ld32(tO + c * 32, u);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(__uint_as_float(u[2 * i]) * inv, __uint_as_float(u[2 * i + 1]) * inv);
        if (tok < nq_t[t]) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

// ------------------------------------------------------------ host side
// Query tokens per work item of the tcgen05 path: two 128-row tiles.
inline int extend_tc_tile_tokens(int G) { return 2 * (kTcRows / G); }

inline bool extend_tc_supported(int Hq, int Hkv, int D, int dtype) {
  const int G = Hkv > 0 ? Hq / Hkv : 0;
  return dtype == 1 /* bf16 */ && D == kTcD && (G == 1 || G == 2 || G == 4 || G == 8);
}

// Page sizes the TMA gather handles (16-row boxes inside one page).
inline bool extend_tc_page_ok(int page_log2) { return page_log2 >= 4; }

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder(std::string& err) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn) return fn;
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) {
    err = "cuTensorMapEncodeTiled entry point unavailable";
    return nullptr;
  }
  fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  return fn;
}

inline bool encode_3d(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* map, const void* base, uint64_t d0,
                      uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0,
                      uint32_t b1, uint32_t b2) {
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult rc = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return rc == CUDA_SUCCESS;
}

inline int extend_tc_launch(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
                            const void* k_stage, const void* v_stage, int64_t stage_slots, int group_starts,
                            const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_indices,
                            const int32_t* kv_last_page_len, int page_log2, const int32_t* work, int n_work, int T,
                            int Hq, int Hkv, float scale, void* out, cudaStream_t st, std::string& err) {
  const int G = Hq / Hkv;
  auto enc = tensor_map_encoder(err);
  if (!enc) return 3;
  if (T <= 0 || num_slots <= 0 || num_slots > 0x7fffffffLL - 64) {
    err = "extend_tc: T and num_slots must be in (0, 2^31)";
    return 1;
  }
  CUtensorMap qm, km, vm, km2, vm2;
  const uint64_t row = (uint64_t)kTcD * 2;
  if (!encode_3d(enc, &qm, q, kTcD, (uint64_t)Hq, (uint64_t)T, row, row * Hq, 64, (uint32_t)G,
                 (uint32_t)(kTcRows / G)) ||
      !encode_3d(enc, &km, k_pool, kTcD, (uint64_t)Hkv, (uint64_t)num_slots, row, row * Hkv, 64, 1, 16) ||
      !encode_3d(enc, &vm, v_pool, kTcD, (uint64_t)Hkv, (uint64_t)num_slots, row, row * Hkv, 64, 1, 16)) {
    err = "extend_tc: cuTensorMapEncodeTiled rejected a tensor map";
    return 1;
  }
  km2 = km;
  vm2 = vm;
  if (stage_slots > 0 &&
      (!encode_3d(enc, &km2, k_stage, kTcD, (uint64_t)Hkv, (uint64_t)stage_slots, row, row * Hkv, 64, 1, 16) ||
       !encode_3d(enc, &vm2, v_stage, kTcD, (uint64_t)Hkv, (uint64_t)stage_slots, row, row * Hkv, 64, 1, 16))) {
    err = "extend_tc: cuTensorMapEncodeTiled rejected the staging tensor map";
    return 1;
  }
  TcArgs a;
  a.qo_indptr = qo_indptr;
  a.kv_indptr = kv_indptr;
  a.kv_indices = kv_indices;
  a.kv_last_page_len = kv_last_page_len;
  a.work = work;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.num_slots = num_slots;
  a.stage_slots = stage_slots > 0 ? stage_slots : 0;
  a.page_log2 = page_log2;
  a.group_starts = group_starts;
  a.Hq = Hq;
  a.G = G;
  a.qscale = scale * kLog2e;
  // the caller has raised the kernel's shared-memory limit (once per device).
  // Grid x = kv head, y = work item: the block scheduler hands out the
  // cost-sorted items with all their heads together, so the most expensive
  // tiles start first on every head (measured +6% over head-major order);
  // y is limited to 65535, so longer work lists go out in chunks.
  for (int off = 0; off < n_work; off += 65535) {
    a.work = work + 4 * (size_t)off;
    extend_tc2_kernel<<<dim3(Hkv, std::min(65535, n_work - off)), kTc2Threads, Tc2Smem::ALLOC, st>>>(qm, km, vm, km2,
                                                                                                       vm2, a);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    err = std::string("extend_tc2_kernel: ") + cudaGetErrorString(e);
    return 3;
  }
  err.clear();
  return 0;
}

}  // namespace b2a
