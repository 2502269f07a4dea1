// Paged decode attention on tensor cores (bf16, head_dim 128, page_size >= 16).
//
// Reference: python/minisgl_mlx/attention/metal.py:35-131 and
// attention/naive.py:50-60 (same values as decode.cuh). Same plan, workspace,
// in-launch merge and error handling as decode_kernel; only the stage layout
// and the consumer arithmetic differ.
//
// Why: with G query heads per kv head, the FMA path of decode.cuh spends
// about G*4 FMAs plus a shuffle reduction per (token, head, feature chunk),
// which at G = 4 binds the kernel to its issue rate under the power cap
// instead of HBM. Here one warp per kv head computes, for every stage of 16
// tokens,
//   S^T [16 tokens x 8 head columns] = K [16 x 128] . Q^T      (8 MMAs)
//   O^T [128 x 8]                   += V^T [128 x 16] . P^T    (8 MMAs)
// with mma.sync m16n8k16 (bf16 in, fp32 accumulate), the G query heads as the
// N = 8 columns (zero-padded). The score fragment is turned into the P^T
// operand in registers with movmatrix (an 8x8 transpose), so no score goes
// through shared memory.
//
// Stage layout: the producer loads each (kv head, 64-feature half) of a
// 16-token run as one 3-D TMA box {64, 1, 16} with SWIZZLE_128B, so a head's
// 16 tokens are 16 rows of 128 B whose 16-byte chunks are XOR-permuted by row.
// ldmatrix then reads 8 consecutive tokens at one feature offset from 8
// different bank groups (no conflicts), for K as the A operand of S^T and,
// transposed, for V as the A operand of O^T. A 16-token run never crosses a
// page (page_size >= 16, stages start at multiples of 16 inside a page).
//
// Softmax: scores in the log2 domain (scale * log2 e applied in fp32 after
// the MMA). The reference max of a head column only moves when a score
// exceeds it by more than 8 (p <= 256 keeps bf16 P and fp32 accumulation
// exact); the column max is then reduced across the 8 lanes that share the
// column. Tokens past the segment are masked to p = 0; the rows the box
// loaded for them are pool rows of the same page (finite K/V values).
#pragma once

#include "decode.cuh"
#include "extend_tc.cuh"

namespace b2a {

constexpr int kMmaTok = 16;  // tokens per stage

__host__ __device__ inline uint32_t decode_mma_stage_bytes(int Hkv) {
  return 2u /*K,V*/ * 2u /*feature halves*/ * (uint32_t)Hkv * (uint32_t)(kMmaTok * 128);
}

struct DecodeMmaSmem {
  uint32_t bars, abort_flag, last_flag, total;
};

__host__ __device__ inline DecodeMmaSmem decode_mma_smem_layout(int NSTAGE, int Hkv) {
  DecodeMmaSmem L;
  uint32_t off = (uint32_t)NSTAGE * decode_mma_stage_bytes(Hkv);  // stages are 1024-byte multiples
  L.bars = off;
  off += (uint32_t)NSTAGE * 2u * 8u;
  L.abort_flag = off;
  off += 16;
  L.last_flag = off;
  off += 16;
  L.total = off;
  return L;
}

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
      "{%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// D += A (16x16 bf16, row) . B (16x8 bf16, col), fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose of an 8x8 b16 matrix held one row pair per thread (thread 4r + c
// holds row r, columns 2c and 2c + 1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

// Shared-memory address of token row `row` (0..15), 16-byte chunk `chunk`
// (0..7) of a 16-row SWIZZLE_128B box starting at the 1024-byte aligned `box`.
__device__ __forceinline__ uint32_t sw128_row_chunk(uint32_t box, int row, int chunk) {
  return box + (uint32_t)row * 128u + ((uint32_t)(chunk ^ (row & 7)) << 4);
}

// One stage of one kv head: S^T, online softmax, O^T += V^T P^T.
// kbox[dh] / vbox[dh]: the head's two 64-feature boxes of K and V.
template <int G>
__device__ __forceinline__ void decode_mma_stage(uint32_t kbox0, uint32_t kbox1, uint32_t vbox0, uint32_t vbox1,
                                                 int nt, int lane, float qscale, const uint32_t (&qf)[8][2],
                                                 float (&acc)[8][4], float (&mref)[2], float (&lsum)[2]) {
  constexpr unsigned FULL = 0xffffffffu;
  const int g = lane >> 2;
  const int mi = lane >> 3;          // ldmatrix: the 8x8 matrix this lane addresses
  const int r8 = lane & 7;
  // ---- S^T = K Q^T: A = K [16 tokens x 16 features] per K-step
  float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const int row = r8 + 8 * (mi & 1);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      ldsm_x4(sw128_row_chunk(kbox0, row, 2 * kk + (mi >> 1)), a);
      mma_16816(s0, a, qf[kk][0], qf[kk][1]);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      ldsm_x4(sw128_row_chunk(kbox1, row, 2 * kk + (mi >> 1)), a);
      mma_16816(s1, a, qf[4 + kk][0], qf[4 + kk][1]);
    }
  }
  // x[0]: (token g, column 2c) x[1]: (g, 2c+1) x[2]: (g+8, 2c) x[3]: (g+8, 2c+1)
  float x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = (s0[i] + s1[i]) * qscale;
  if (nt < kMmaTok) {
    if (g >= nt) x[0] = x[1] = kNegInf;
    if (g + 8 >= nt) x[2] = x[3] = kNegInf;
  }
  float cm[2] = {fmaxf(x[0], x[2]), fmaxf(x[1], x[3])};
  const bool grow = cm[0] > mref[0] + 8.f || cm[1] > mref[1] + 8.f;
  if (__any_sync(FULL, grow)) {
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      float v = cm[n];
      v = fmaxf(v, __shfl_xor_sync(FULL, v, 4));
      v = fmaxf(v, __shfl_xor_sync(FULL, v, 8));
      v = fmaxf(v, __shfl_xor_sync(FULL, v, 16));
      if (v > mref[n] + 8.f) {  // the same decision on every lane of the column
        const float alpha = (mref[n] == kNegInf) ? 0.f : exp2f(mref[n] - v);
        mref[n] = v;
        lsum[n] *= alpha;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          acc[mt][n] *= alpha;
          acc[mt][2 + n] *= alpha;
        }
      }
    }
  }
  float p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = (x[i] == kNegInf) ? 0.f : exp2f(x[i] - mref[i & 1]);
  lsum[0] += p[0] + p[2];
  lsum[1] += p[1] + p[3];
  // P^T as the B operand (K = tokens, N = head columns) of O^T += V^T P^T
  const uint32_t pb0 = movmatrix_trans(pack_bf16(p[0], p[1]));  // tokens 0-7
  const uint32_t pb1 = movmatrix_trans(pack_bf16(p[2], p[3]));  // tokens 8-15
  // ---- O^T += V^T P^T: A = V^T [16 features x 16 tokens] per feature tile
  {
    const int row = r8 + 8 * (mi >> 1);
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int chunk = 2 * mt + (mi & 1);  // 16-byte chunk (8 features) of the 128-feature row
      uint32_t a[4];
      ldsm_x4_trans(sw128_row_chunk(chunk < 8 ? vbox0 : vbox1, row, chunk & 7), a);
      mma_16816(acc[mt], a, pb0, pb1);
    }
  }
}

// Launched with Hkv + 1 warps: Hkv consumers (one per kv head) and a producer.
template <int G>
__global__ void __launch_bounds__(17 * 32, 1)
    decode_mma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                      const DecodeArgs a) {
  static_assert(G >= 1 && G <= 8, "the head columns of one MMA hold at most 8 query heads");
  pdl_wait_then_release();
  constexpr int D = 128;
  constexpr unsigned FULL = 0xffffffffu;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int Hkv = a.Hkv;
  const int NCW = a.NCW;  // one consumer warp per kv head
  const uint32_t stage_bytes = decode_mma_stage_bytes(Hkv);
  const DecodeMmaSmem L = decode_mma_smem_layout(a.NSTAGE, Hkv);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + a.NSTAGE;
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L.abort_flag);
  volatile int* s_last = reinterpret_cast<volatile int*>(smem + L.last_flag);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int seg0 = a.cta_indptr[blockIdx.x];
  const int seg1 = a.cta_indptr[blockIdx.x + 1];
  const bool last_first = decode_last_first(a, seg0, seg1);
  const int P = 1 << a.page_log2;
  // stage s: K boxes at [s][0][dh][head], V boxes at [s][1][dh][head] (2 KB each)
  auto box = [&](int st, int kind, int dh, int head) -> uint32_t {
    return smem_u32(smem) + (uint32_t)st * stage_bytes + (uint32_t)kind * (stage_bytes / 2u) +
           (uint32_t)(dh * Hkv + head) * (uint32_t)(kMmaTok * 128);
  };

  if (warp == NCW) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = l2_evict_first_policy();
    int ctr = 0;
    bool ok = true;
    for (int i = 0; i < seg1 - seg0 && ok; ++i) {
      const int si = decode_seg_at(a, seg0, seg1, last_first, i);
      int b, pbeg, ntok, slot;
      decode_get_seg(a, si, b, pbeg, ntok, slot);
      if (!decode_seg_ok(a, b, slot)) continue;  // the consumers skip it too (and report it)
      for (int tok = 0; tok < ntok; tok += kMmaTok) {
        if (!__all_sync(FULL, *s_abort == 0)) {
          ok = false;
          break;
        }
        const int st = ctr % a.NSTAGE;
        const uint32_t ph = (uint32_t)(ctr / a.NSTAGE) & 1u;
        if (!__all_sync(FULL, mbar_wait(&empty[st], ph ^ 1u, kWdDecodeEmpty))) {
          *s_abort = 1;
          ok = false;
          break;
        }
        int64_t src = -1;
        if (lane == 0) {
          const int64_t page = a.kv_indices[pbeg + (tok >> a.page_log2)];
          const int64_t s0 = page * P + (tok & (P - 1));
          src = (page >= 0 && s0 + kMmaTok <= a.num_slots) ? s0 : -1;
        }
        src = __shfl_sync(FULL, src, 0);
        // Bad page ids never reach the copy engine: record the error and let the
        // consumers run this stage on stale data.
        if (lane == 0) {
          if (src >= 0) {
            mbar_arrive_expect_tx(&full[st], stage_bytes);
          } else {
            watchdog_set(kWdBadSlot);
            mbar_arrive(&full[st]);
          }
        }
        __syncwarp();
        if (src >= 0) {
          // lane = head * 4 + kind * 2 + feature half: one 16-row box each
          for (int l = lane; l < 4 * Hkv; l += 32) {
            const int head = l >> 2, kind = (l >> 1) & 1, dh = l & 1;
            tma_load_3d_hint(smem + (box(st, kind, dh, head) - smem_u32(smem)), kind ? &vmap : &kmap, dh * 64, head,
                             (int)src, &full[st], pol);
          }
        }
        __syncwarp();
        ++ctr;
      }
    }
    // Never leave while our own copies may still be landing.
    const int first = ctr > a.NSTAGE ? ctr - a.NSTAGE : 0;
    for (int i = first; i < ctr; ++i) mbar_wait(&full[i % a.NSTAGE], (uint32_t)(i / a.NSTAGE) & 1u, kWdDecodeDrain);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int h = warp;  // kv head
  const int g = lane >> 2, c = lane & 3;
  const __nv_bfloat16* qbase = reinterpret_cast<const __nv_bfloat16*>(a.q);
  int ctr = 0;
  for (int i = 0; i < seg1 - seg0; ++i) {
    const int si = decode_seg_at(a, seg0, seg1, last_first, i);
    int b, pbeg, ntok, slot;
    decode_get_seg(a, si, b, pbeg, ntok, slot);
    if (!decode_seg_ok(a, b, slot)) {
      if (threadIdx.x == 0) watchdog_set(kWdBadPlan);
      continue;
    }
    // B operand of S^T = K Q^T (K = features, N = head columns): column g is query
    // head h*G + g (zero for g >= G); K-step kk holds features 16kk + 2c, +1, +8, +9
    uint32_t qf[8][2];
    {
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qbase + ((size_t)b * a.Hq + h * G + (g < G ? g : 0)) * D);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qf[kk][0] = g < G ? qrow[8 * kk + c] : 0u;
        qf[kk][1] = g < G ? qrow[8 * kk + 4 + c] : 0u;
      }
    }
    float acc[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
    float mref[2] = {kNegInf, kNegInf}, lsum[2] = {0.f, 0.f};
    for (int tok = 0; tok < ntok; tok += kMmaTok) {
      const int nt = min(kMmaTok, ntok - tok);
      const int st = ctr % a.NSTAGE;
      const uint32_t ph = (uint32_t)(ctr / a.NSTAGE) & 1u;
      bool ok = __all_sync(FULL, *s_abort == 0);
      if (ok) ok = __all_sync(FULL, mbar_wait(&full[st], ph, kWdDecodeFull));
      if (!ok) *s_abort = 1;
      if (ok)
        decode_mma_stage<G>(box(st, 0, 0, h), box(st, 0, 1, h), box(st, 1, 0, h), box(st, 1, 1, h), nt, lane,
                            a.qscale, qf, acc, mref, lsum);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      ++ctr;
    }
    // ---- finalize: row sums over the 8 lanes of each head column
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      lsum[n] += __shfl_xor_sync(FULL, lsum[n], 4);
      lsum[n] += __shfl_xor_sync(FULL, lsum[n], 8);
      lsum[n] += __shfl_xor_sync(FULL, lsum[n], 16);
    }
    // thread (g, c) holds features 16mt + g and 16mt + g + 8 of head columns 2c, 2c + 1
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const int gq = 2 * c + n;  // head column
      if (gq < G) {
        const size_t row = (size_t)h * G + gq;
        if (slot < 0) {
          const float inv = lsum[n] > 0.f ? 1.f / lsum[n] : 0.f;
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + ((size_t)b * a.Hq + row) * D;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[16 * mt + g] = __float2bfloat16_rn(acc[mt][n] * inv);
            o[16 * mt + g + 8] = __float2bfloat16_rn(acc[mt][2 + n] * inv);
          }
        } else {
          float* o = a.ws_acc + ((size_t)slot * a.Hq + row) * D;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[16 * mt + g] = acc[mt][n];
            o[16 * mt + g + 8] = acc[mt][2 + n];
          }
          if (g == 0) {
            a.ws_ml[((size_t)slot * a.Hq + row) * 2 + 0] = mref[n];
            a.ws_ml[((size_t)slot * a.Hq + row) * 2 + 1] = lsum[n];
          }
        }
      }
    }
    if (slot >= 0) {
      __threadfence();  // publish this warp's partial rows at GPU scope before the ticket
      // Merge ticket of request b, as in decode_kernel.
      named_bar_sync(1, NCW * 32);
      const int p0 = a.merge_indptr[b], p1 = a.merge_indptr[b + 1];
      if (threadIdx.x == 0) {
        const int prev = atomicAdd(&a.tickets[p0], 1);
        const bool last = prev == p1 - p0 - 1;
        if (last) a.tickets[p0] = 0;  // every partial has arrived: re-arm for the next call
        *s_last = last ? 1 : 0;
      }
      named_bar_sync(1, NCW * 32);
      if (*s_last) {
        __threadfence();
        decode_merge_request<__nv_bfloat16, D>(a, b, p0, p1, warp, lane);
      }
    }
  }
}

// ------------------------------------------------------------ host side
// Shapes this kernel serves. G = 2 stays on decode_kernel: measured on config 2
// (16q/8kv, page 16, B = 128, L ~ U[100, 2048]) this kernel ran a call in
// 0.112 ms against 0.099 ms for the FMA path, whose G = 2 arithmetic is light
// enough to hide under the stream; at G = 4 (config 5) it is the other way
// round (0.93 against 0.78 of the HBM peak).
inline bool decode_mma_supported(int Hq, int Hkv, int D, int dtype, int page_log2) {
  const int G = Hkv > 0 ? Hq / Hkv : 0;
  // Hkv 4 or 8: two stages of 16 tokens (64 KB each at Hkv 8) fit in shared memory; Hkv 16 would
  // need 128 KB stages and stays on decode_kernel
  return dtype == 1 /* bf16 */ && D == 128 && page_log2 >= 4 && (Hkv == 4 || Hkv == 8) && (G == 4 || G == 8);
}

// Ring depth: as many 16-token stages as fit (at most 6) next to the barriers
// and the 1024-byte alignment slack.
inline int decode_mma_nstage(int Hkv, size_t smem_limit) {
  int ns = 6;
  while (ns > 2 && decode_mma_smem_layout(ns, Hkv).total + 1024 > smem_limit) --ns;
  return ns;
}

}  // namespace b2a
