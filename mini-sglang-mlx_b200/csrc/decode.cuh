// Paged decode attention (one query row per request) for sm_100a.
//
// Reference: python/minisgl_mlx/attention/metal.py:35-131 (Metal kernel: one
// threadgroup per (request, kv head), online softmax, fp32 accumulation) and
// attention/naive.py:50-60 (gather + masked SDPA, same values).
//
// B200 design (not a translation of the Metal kernel):
//   * The pool row of one slot holds all Hkv heads ([Hkv, D], 2 KB for
//     8x128 bf16), and a page is page_size consecutive rows. A CTA therefore
//     works on ALL kv heads of a request at once and moves whole page runs
//     with single cp.async.bulk (TMA) copies into a NSTAGE-deep shared-memory
//     ring, completion tracked by mbarriers (one producer warp).
//   * Grid = persistent CTAs, each owning a contiguous, equal share of the
//     concatenated page stream of the batch (host plan). A request cut by a
//     share boundary produces partial (m, l, acc) rows; requests inside a
//     share are written directly. Each split request has a merge ticket (an
//     int32 counter in the workspace): a CTA that has written one of its
//     partials takes a ticket, and the CTA that takes the last one merges all
//     of that request's partials and re-arms the counter to zero. No CTA ever
//     waits for another, and no separate merge launch follows.
//   * NCW consumer warps (16 when shared memory allows, else 8); warp w
//     serves kv head w / WPH and every WPH-th group of TG tokens of a stage,
//     so two or more groups are in flight per head. Lane = D/32 features. The
//     G query heads of the group share every K/V row read. The TG*G partial
//     dot products of a group are reduced with a transpose-butterfly (about
//     one shuffle per sum), leaving each lane with one (token, head) score;
//     softmax statistics are per lane and the probabilities go through a
//     32-float smem slot to the PV loop. Warps of one head combine their
//     (m, l, acc) through shared memory at the end of a segment.
//   * Scores are kept in the log2 domain (q pre-scaled by scale*log2 e).
#pragma once
#include <type_traits>

#include "common.cuh"

namespace b2a {

struct DecodeArgs {
  const void* q;
  const void* k_pool;
  const void* v_pool;
  const int32_t* kv_indices;  // page ids
  const int32_t* kv_indptr;   // direct mode: token CSR (page_size 1)
  const int32_t* cta_indptr;  // plan mode: CSR over segs; NULL = direct mode
  const int32_t* segs;        // int4 {request, first page idx, n_tokens, out_slot}
  const int32_t* merge_indptr;  // [B + 1] CSR over partial slots (plan mode)
  float* ws_acc;              // [n_partials, Hq, D]
  float* ws_ml;               // [n_partials, Hq, 2]
  int32_t* tickets;           // [n_partials] merge counters, indexed by a request's first partial slot
  void* out;                  // [B, Hq, D]
  int64_t num_slots;
  int B;           // requests (bounds of the plan's request ids)
  int n_partials;  // partial slots the workspace holds (bounds of the plan's slots)
  int page_log2;
  int Hq, Hkv;
  float qscale;  // softmax scale * log2(e)
  int TS;        // tokens per stage
  int NSTAGE;
  int WPH;  // consumer warps per kv head
  int NCW;  // consumer warps
  uint32_t row_bytes;
  uint32_t stage_bytes;  // bytes of ONE of K/V in a stage (TS * row_bytes)
};

struct DecodeSmem {
  // byte offsets inside the dynamic shared memory block
  uint32_t bars, pbuf, cbuf, abort_flag, last_flag, total;
};

__host__ __device__ inline DecodeSmem decode_smem_layout(int NSTAGE, uint32_t stage_bytes, int NCW, int WPH,
                                                         int G, int D) {
  DecodeSmem L;
  uint32_t off = (uint32_t)NSTAGE * 2u * stage_bytes;
  off = (off + 127u) & ~127u;
  L.bars = off;
  off += (uint32_t)NSTAGE * 2u * 8u;
  off = (off + 15u) & ~15u;
  L.pbuf = off;
  off += (uint32_t)NCW * 32u * 4u;
  L.cbuf = off;
  if (WPH > 1) off += (uint32_t)NCW * (uint32_t)G * (uint32_t)(D + 2) * 4u;
  L.abort_flag = off;
  off += 16;
  L.last_flag = off;
  off += 16;
  L.total = off;
  return L;
}

__device__ __forceinline__ void decode_get_seg(const DecodeArgs& a, int idx, int& b, int& page_begin, int& ntok,
                                               int& slot) {
  if (a.cta_indptr != nullptr) {
    const int4 s = reinterpret_cast<const int4*>(a.segs)[idx];
    b = s.x;
    page_begin = s.y;
    ntok = s.z;
    slot = s.w;
  } else {
    b = blockIdx.x;
    page_begin = a.kv_indptr[b];
    ntok = a.kv_indptr[b + 1] - page_begin;
    slot = -1;
  }
}

// Visit order of a CTA's segments [seg0, seg1). The plan lists them in page
// order, so a CTA's last segment is usually the head of a request whose tail the
// next CTA streams first; visited last, its merge would fall at the very end of
// every CTA. When the last segment writes a partial it is visited first instead
// (then the others in page order), so both pieces of such a request finish early
// and the CTA that merges it does so while other CTAs are still streaming.
__device__ __forceinline__ int decode_seg_at(const DecodeArgs& a, int seg0, int seg1, bool last_first, int i) {
  if (!last_first) return seg0 + i;
  return i == 0 ? seg1 - 1 : seg0 + i - 1;
}

__device__ __forceinline__ bool decode_last_first(const DecodeArgs& a, int seg0, int seg1) {
  if (a.cta_indptr == nullptr || seg1 - seg0 < 2) return false;
  return reinterpret_cast<const int4*>(a.segs)[seg1 - 1].w >= 0;
}

// A segment is used only if its request id is in [0, B) and, when it writes a
// partial, its slot lies in its request's merge range inside the workspace.
// Producer and consumers decide identically, so a rejected segment is skipped
// by both (no stage is issued or awaited for it) and reported as kWdBadPlan.
__device__ __forceinline__ bool decode_seg_ok(const DecodeArgs& a, int b, int slot) {
  if (b < 0 || b >= a.B) return false;
  if (slot < 0) return true;
  const int p0 = a.merge_indptr[b], p1 = a.merge_indptr[b + 1];
  return p0 >= 0 && p0 <= slot && slot < p1 && p1 <= a.n_partials;
}

template <int G>
__device__ __forceinline__ void load_p(const float* pb, int i, float (&pg)[G]) {
  if constexpr (G == 1) {
    pg[0] = pb[i];
  } else if constexpr (G == 2) {
    const float2 t = reinterpret_cast<const float2*>(pb)[i];
    pg[0] = t.x;
    pg[1] = t.y;
  } else {
#pragma unroll
    for (int j = 0; j < G / 4; ++j) {
      const float4 t = reinterpret_cast<const float4*>(pb + i * G)[j];
      pg[4 * j + 0] = t.x;
      pg[4 * j + 1] = t.y;
      pg[4 * j + 2] = t.z;
      pg[4 * j + 3] = t.w;
    }
  }
}

// Tokens per reduction group: V = TG * G partial dot products per group,
// V <= 32 so one lane ends up owning one (token, query head) score.
template <int G>
__host__ __device__ constexpr int decode_tg() {
  return G <= 4 ? 8 : 32 / G;
}

constexpr int ilog2c(int x) { return x <= 1 ? 0 : 1 + ilog2c(x >> 1); }

// Partial dot products of TG tokens x G query heads for one kv head. q and the
// accumulators are packed feature pairs (fma.rn.f32x2): a lane's EPT features
// give EPT/2 packed FMAs per head, the two halves are added at the end.
template <typename T, int D, int G, int TG, bool CHECK>
__device__ __forceinline__ void decode_qk(const T* __restrict__ kh, int row_elems, int nvalid,
                                          const uint64_t (&qv2)[G][D / 64], float (&v)[TG * G]) {
  constexpr int EPT = D / 32;
#pragma unroll
  for (int i = 0; i < TG; ++i) {
    if (!CHECK || i < nvalid) {
      float kf[EPT];
      load_vec<T, EPT>(kh + i * row_elems, kf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        uint64_t s2 = f2(0.f, 0.f);
#pragma unroll
        for (int e = 0; e < EPT / 2; ++e) s2 = f2_fma(qv2[g][e], f2(kf[2 * e], kf[2 * e + 1]), s2);
        float lo, hi;
        f2_split(s2, lo, hi);
        v[i * G + g] = lo + hi;
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) v[i * G + g] = 0.f;
    }
  }
}

template <typename T, int D, int G, int TG, bool CHECK>
__device__ __forceinline__ void decode_pv(const T* __restrict__ vh, int row_elems, int nvalid, const float* pb,
                                          uint64_t (&acc2)[G][D / 64]) {
  constexpr int EPT = D / 32;
#pragma unroll
  for (int i = 0; i < TG; ++i) {
    if (!CHECK || i < nvalid) {
      float vf[EPT];
      load_vec<T, EPT>(vh + i * row_elems, vf);
      float pg[G];
      load_p<G>(pb, i, pg);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint64_t p2 = f2(pg[g], pg[g]);
#pragma unroll
        for (int e = 0; e < EPT / 2; ++e) acc2[g][e] = f2_fma(p2, f2(vf[2 * e], vf[2 * e + 1]), acc2[g][e]);
      }
    }
  }
}

// One group of TG tokens (nvalid of them real) for one kv head.
//
// The V = TG*G partial sums (each lane holds D/32 features of every one) are
// reduced with log2(V) transposing butterfly steps -- at each step a lane
// keeps the half of its remaining values selected by its lane bit and adds
// the partner's copy of that half -- followed by 5 - log2(V) plain xor steps.
// Lane l then holds the full score of value j = l >> REM, i.e. of token
// j / G and query head j % G (lanes differing only in the low REM bits hold
// the same value). Softmax statistics stay per lane; the probabilities go to
// a per-warp shared slot for the PV loop.
template <typename T, int D, int G, int TG>
__device__ __forceinline__ void decode_group(const T* __restrict__ kh, const T* __restrict__ vh, int row_elems,
                                             int nvalid, int lane, const uint64_t (&qv)[G][D / 64],
                                             uint64_t (&acc)[G][D / 64], float& m_mine, float& l_mine, float* pb) {
  constexpr int EPT = D / 32;
  constexpr int V = TG * G;
  static_assert(V <= 32 && (V & (V - 1)) == 0, "group must hold at most 32 power-of-two values");
  constexpr int K = ilog2c(V);
  constexpr int REM = 5 - K;
  constexpr int LG = ilog2c(G);
  constexpr unsigned FULL = 0xffffffffu;
  (void)EPT;
  float v[V];
  if (nvalid == TG) decode_qk<T, D, G, TG, false>(kh, row_elems, nvalid, qv, v);
  else decode_qk<T, D, G, TG, true>(kh, row_elems, nvalid, qv, v);
#pragma unroll
  for (int st = 0; st < K; ++st) {
    const int off = 16 >> st;
    const int half = V >> (st + 1);
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float lo = v[j], hi = v[j + half];
      const float send = upper ? lo : hi;
      const float keep = upper ? hi : lo;
      v[j] = keep + __shfl_xor_sync(FULL, send, off);
    }
  }
#pragma unroll
  for (int off = (1 << REM) >> 1; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(FULL, v[0], off);
  const int my_tok = lane >> (REM + LG);
  const float s = (my_tok < nvalid) ? v[0] : kNegInf;
  float mt = s;
#pragma unroll
  for (int off = 1 << (REM + LG); off < 32; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(FULL, mt, off));
  const float m_new = fmaxf(m_mine, mt);
  const float alpha = (m_mine == m_new) ? 1.f : exp2f(m_mine - m_new);
  const float p = (s == kNegInf) ? 0.f : exp2f(s - m_new);
  l_mine = l_mine * alpha + p;
  m_mine = m_new;
  if ((lane & ((1 << REM) - 1)) == 0) pb[lane >> REM] = p;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float ag = __shfl_sync(FULL, alpha, g << REM);
    if (ag != 1.f) {
      const uint64_t a2 = f2(ag, ag);
#pragma unroll
      for (int e = 0; e < EPT / 2; ++e) acc[g][e] = f2_mul(acc[g][e], a2);
    }
  }
  __syncwarp();
  if (nvalid == TG) decode_pv<T, D, G, TG, false>(vh, row_elems, nvalid, pb, acc);
  else decode_pv<T, D, G, TG, true>(vh, row_elems, nvalid, pb, acc);
  __syncwarp();
}

// Combine the partial rows of request b (slots [p0, p1)), written by this and
// other CTAs of the same launch: consumer warp w takes query heads w, w + NCW, ...
// The rows are read through L2 (ld.global.cg): another SM wrote them, and this
// SM's L1 may still hold lines of the same workspace from an earlier launch.
// Up to eight partials are fetched at once and folded into a running (M, l, acc)
// (the same online rescaling as the kernel's softmax), so a merge costs one L2
// round trip per eight partials instead of a dependent load chain per partial.
template <typename T, int D>
__device__ __forceinline__ void decode_merge_request(const DecodeArgs& a, int b, int p0, int p1, int warp,
                                                     int lane) {
  constexpr int EPT = D / 32;
  constexpr int U = 8;  // partials fetched together: one L2 round trip per U partials
  const int Hq = a.Hq;
  for (int qh = warp; qh < Hq; qh += a.NCW) {
    float M = kNegInf, Lsum = 0.f, acc[EPT];
#pragma unroll
    for (int e = 0; e < EPT; ++e) acc[e] = 0.f;
    for (int base = p0; base < p1; base += U) {
      float m[U], l[U], o[U][EPT];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int p = base + u;
        if (p < p1) {
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.ws_ml + ((size_t)p * Hq + qh) * 2));
          m[u] = ml.x;
          l[u] = ml.y;
          const float* src = a.ws_acc + ((size_t)p * Hq + qh) * D + lane * EPT;
#pragma unroll
          for (int e = 0; e < EPT; e += 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(src + e));
            o[u][e] = v.x;
            o[u][e + 1] = v.y;
            o[u][e + 2] = v.z;
            o[u][e + 3] = v.w;
          }
        } else {
          m[u] = kNegInf;
          l[u] = 0.f;
#pragma unroll
          for (int e = 0; e < EPT; ++e) o[u][e] = 0.f;
        }
      }
      float Mn = M;
#pragma unroll
      for (int u = 0; u < U; ++u) Mn = fmaxf(Mn, m[u]);
      const float keep = (M == kNegInf) ? 0.f : exp2f(M - Mn);
      Lsum *= keep;
#pragma unroll
      for (int e = 0; e < EPT; ++e) acc[e] *= keep;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float w = (m[u] == kNegInf) ? 0.f : exp2f(m[u] - Mn);
        Lsum += l[u] * w;
#pragma unroll
        for (int e = 0; e < EPT; ++e) acc[e] = fmaf(w, o[u][e], acc[e]);
      }
      M = Mn;
    }
    const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
#pragma unroll
    for (int e = 0; e < EPT; ++e) acc[e] *= inv;
    store_vec<T, EPT>(reinterpret_cast<T*>(a.out) + ((size_t)b * Hq + qh) * D + lane * EPT, acc);
  }
}

template <typename T, int D, int G, int NCW>
__global__ void __launch_bounds__((NCW + 1) * 32, 1) decode_kernel(const DecodeArgs a) {
  // Programmatic dependent launch: the next kernel may become resident now; this one
  // sets up its barriers and reads its plan and the first stage's page ids while the
  // previous kernel still runs, and waits for it (griddepcontrol.wait) only before
  // touching what that kernel may have written: q, the KV rows, the workspace, out.
  // The plan arrays are written before the previous kernel of the stream starts.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int EPT = D / 32;
  constexpr int TG = decode_tg<G>();
  constexpr int REM = 5 - ilog2c(TG * G);
  constexpr int LG = ilog2c(G);
  constexpr unsigned FULL = 0xffffffffu;
  extern __shared__ __align__(128) uint8_t smem[];
  const int G_ = G;
  const DecodeSmem L = decode_smem_layout(a.NSTAGE, a.stage_bytes, a.NCW, a.WPH, G_, D);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + a.NSTAGE;
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L.abort_flag);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], a.NCW);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  int seg0, seg1;
  if (a.cta_indptr != nullptr) {
    seg0 = a.cta_indptr[blockIdx.x];
    seg1 = a.cta_indptr[blockIdx.x + 1];
  } else {
    seg0 = 0;
    seg1 = 1;
  }
  const int P = 1 << a.page_log2;
  const int TS = a.TS;

  if (warp == a.NCW) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = l2_evict_first_policy();
    const uint8_t* kp = reinterpret_cast<const uint8_t*>(a.k_pool);
    const uint8_t* vp = reinterpret_cast<const uint8_t*>(a.v_pool);
    const size_t rowB = a.row_bytes;
    int ctr = 0;
    bool ok = true;
    bool waited = false;  // griddepcontrol.wait done (before the first copy)
    const bool last_first = decode_last_first(a, seg0, seg1);
    for (int i = 0; i < seg1 - seg0 && ok; ++i) {
      const int si = decode_seg_at(a, seg0, seg1, last_first, i);
      int b, pbeg, ntok, slot;
      decode_get_seg(a, si, b, pbeg, ntok, slot);
      if (!decode_seg_ok(a, b, slot)) continue;  // the consumers skip it too (and report it)
      for (int tok = 0; tok < ntok; tok += TS) {
        if (!__all_sync(FULL, *s_abort == 0)) {
          ok = false;
          break;
        }
        const int nt = min(TS, ntok - tok);
        const int st = ctr % a.NSTAGE;
        const uint32_t ph = (uint32_t)(ctr / a.NSTAGE) & 1u;
        const bool got = __all_sync(FULL, mbar_wait(&empty[st], ph ^ 1u, kWdDecodeEmpty));
        if (!got) {
          *s_abort = 1;
          ok = false;
          break;
        }
        uint8_t* kdst = smem + (size_t)st * 2u * a.stage_bytes;
        uint8_t* vdst = kdst + a.stage_bytes;
        // A stage is either a run inside one page (P >= TS) or whole pages
        // (P < TS, stages start on page boundaries); lane j owns copy j.
        const bool one_run = P >= TS;
        const int ncopies = one_run ? 1 : ((nt + P - 1) >> a.page_log2);
        int64_t src_slot[2] = {0, 0};
        int rows_of[2] = {0, 0};
        int64_t pg[2] = {-2, -2};
        bool in_range = true;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int j = lane + 32 * u;
          if (j < ncopies) {
            const int64_t page = a.kv_indices[pbeg + (tok >> a.page_log2) + j];
            pg[u] = page;
            src_slot[u] = one_run ? page * P + (tok & (P - 1)) : page * P;
            rows_of[u] = one_run ? nt : min(P, nt - j * P);
            in_range = in_range && page >= 0 && src_slot[u] + rows_of[u] <= a.num_slots;
          }
        }
        // Consecutive page ids are consecutive slots: a run of them becomes ONE
        // bulk copy issued by the run's first copy, so small pages (page_size 1
        // from a fresh allocator) do not pay the copy engine's per-copy cost per
        // page. Only the stage's last page can be partial, so a run's rows are
        // min(end * P, nt) - j * P. Bytes and the expect_tx count are unchanged.
        int run_rows[2] = {0, 0};
        {
          const int64_t prev0 = __shfl_up_sync(FULL, pg[0], 1);
          const int64_t last0 = __shfl_sync(FULL, pg[0], 31);
          const int64_t prev1 = __shfl_up_sync(FULL, pg[1], 1);
          const bool h0 = lane < ncopies && (lane == 0 || pg[0] != prev0 + 1);
          const bool h1 = lane + 32 < ncopies && pg[1] != (lane == 0 ? last0 : prev1) + 1;
          const uint64_t heads = (uint64_t)__ballot_sync(FULL, h0) | ((uint64_t)__ballot_sync(FULL, h1) << 32);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int j = lane + 32 * u;
            if (u == 0 ? h0 : h1) {
              const uint64_t above = j >= 63 ? 0ull : (heads >> (j + 1)) << (j + 1);
              const int end = above ? __ffsll((long long)above) - 1 : ncopies;
              run_rows[u] = min(end * P, nt) - j * P;
            }
          }
        }
        // Bad page ids never reach the copy engine: record the error, skip the
        // copies of this stage and let the consumers run on stale data.
        const bool all_ok = __all_sync(FULL, in_range);
        if (!all_ok && lane == 0) watchdog_set(kWdBadSlot);
        if (lane == 0) {
          if (all_ok) mbar_arrive_expect_tx(&full[st], (uint32_t)(2u * (uint32_t)nt * a.row_bytes));
          else mbar_arrive(&full[st]);
        }
        __syncwarp();
        if (!waited) {
          asm volatile("griddepcontrol.wait;" ::: "memory");  // the KV rows of the previous kernel
          waited = true;
        }
        if (all_ok) {
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int j = lane + 32 * u;
            if (run_rows[u] > 0) {
              const uint32_t bytes = (uint32_t)run_rows[u] * a.row_bytes;
              const size_t doff = (size_t)j * P * rowB;
              bulk_g2s(kdst + doff, kp + src_slot[u] * rowB, bytes, &full[st], pol);
              bulk_g2s(vdst + doff, vp + src_slot[u] * rowB, bytes, &full[st], pol);
            }
          }
        }
        __syncwarp();
        ++ctr;
      }
    }
    // Never leave while our own bulk copies may still be landing.
    const int first = ctr > a.NSTAGE ? ctr - a.NSTAGE : 0;
    for (int i = first; i < ctr; ++i)
      mbar_wait(&full[i % a.NSTAGE], (uint32_t)(i / a.NSTAGE) & 1u, kWdDecodeDrain);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int h = warp / a.WPH;
  const int sub = warp - h * a.WPH;
  float* pb = reinterpret_cast<float*>(smem + L.pbuf) + warp * 32;
  float* cbuf = reinterpret_cast<float*>(smem + L.cbuf);
  volatile int* s_last = reinterpret_cast<volatile int*>(smem + L.last_flag);
  const T* qbase = reinterpret_cast<const T*>(a.q);
  int ctr = 0;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // q, the workspace and out follow the previous kernel
  const bool last_first = decode_last_first(a, seg0, seg1);
  for (int i = 0; i < seg1 - seg0; ++i) {
    const int si = decode_seg_at(a, seg0, seg1, last_first, i);
    int b, pbeg, ntok, slot;
    decode_get_seg(a, si, b, pbeg, ntok, slot);
    if (!decode_seg_ok(a, b, slot)) {
      if (threadIdx.x == 0) watchdog_set(kWdBadPlan);
      continue;
    }
    uint64_t qv2[G][EPT / 2], acc2[G][EPT / 2];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float qf[EPT];
      load_vec<T, EPT>(qbase + ((size_t)b * a.Hq + h * G + g) * D + lane * EPT, qf);
#pragma unroll
      for (int e = 0; e < EPT / 2; ++e) {
        qv2[g][e] = f2(qf[2 * e] * a.qscale, qf[2 * e + 1] * a.qscale);
        acc2[g][e] = f2(0.f, 0.f);
      }
    }
    float m_mine = kNegInf, l_mine = 0.f;
    for (int tok = 0; tok < ntok; tok += TS) {
      const int nt = min(TS, ntok - tok);
      const int st = ctr % a.NSTAGE;
      const uint32_t ph = (uint32_t)(ctr / a.NSTAGE) & 1u;
      bool ok = __all_sync(FULL, *s_abort == 0);
      if (ok) ok = __all_sync(FULL, mbar_wait(&full[st], ph, kWdDecodeFull));
      if (!ok) *s_abort = 1;
      if (ok) {
        const T* Ks = reinterpret_cast<const T*>(smem + (size_t)st * 2u * a.stage_bytes);
        const T* Vs = reinterpret_cast<const T*>(smem + (size_t)st * 2u * a.stage_bytes + a.stage_bytes);
        const int row_elems = a.Hkv * D;
        for (int t0 = sub * TG; t0 < nt; t0 += a.WPH * TG) {
          const size_t off = ((size_t)t0 * a.Hkv + h) * D + lane * EPT;
          decode_group<T, D, G, TG>(Ks + off, Vs + off, row_elems, min(TG, nt - t0), lane, qv2, acc2, m_mine,
                                    l_mine, pb);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      ++ctr;
    }
    // ---- finalize this segment
    float acc[G][EPT];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < EPT / 2; ++e) f2_split(acc2[g][e], acc[g][2 * e], acc[g][2 * e + 1]);
    float l_red = l_mine;
#pragma unroll
    for (int off = 1 << (REM + LG); off < 32; off <<= 1) l_red += __shfl_xor_sync(FULL, l_red, off);
    float mg[G], lg[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      mg[g] = __shfl_sync(FULL, m_mine, g << REM);
      lg[g] = __shfl_sync(FULL, l_red, g << REM);
    }
    if (a.WPH > 1) {
      float* mine = cbuf + (size_t)warp * G * (D + 2);
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e = 0; e < EPT; ++e) mine[g * (D + 2) + lane * EPT + e] = acc[g][e];
        if (lane == 0) {
          mine[g * (D + 2) + D] = mg[g];
          mine[g * (D + 2) + D + 1] = lg[g];
        }
      }
      named_bar_sync(1, a.NCW * 32);
      if (sub == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float M = kNegInf;
          for (int s2 = 0; s2 < a.WPH; ++s2) M = fmaxf(M, cbuf[(size_t)(warp + s2) * G * (D + 2) + g * (D + 2) + D]);
          float Lsum = 0.f;
#pragma unroll
          for (int e = 0; e < EPT; ++e) acc[g][e] = 0.f;
          for (int s2 = 0; s2 < a.WPH; ++s2) {
            const float* o = cbuf + (size_t)(warp + s2) * G * (D + 2) + g * (D + 2);
            const float w = (o[D] == kNegInf) ? 0.f : exp2f(o[D] - M);
            Lsum += o[D + 1] * w;
#pragma unroll
            for (int e = 0; e < EPT; ++e) acc[g][e] = fmaf(w, o[lane * EPT + e], acc[g][e]);
          }
          mg[g] = M;
          lg[g] = Lsum;
        }
      }
    }
    if (sub == 0) {
      if (slot < 0) {
        T* o = reinterpret_cast<T*>(a.out) + ((size_t)b * a.Hq + h * G) * D + lane * EPT;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float inv = lg[g] > 0.f ? 1.f / lg[g] : 0.f;
          float r[EPT];
#pragma unroll
          for (int e = 0; e < EPT; ++e) r[e] = acc[g][e] * inv;
          store_vec<T, EPT>(o + (size_t)g * D, r);
        }
      } else {
        float* o = a.ws_acc + ((size_t)slot * a.Hq + h * G) * D + lane * EPT;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          store_vec<float, EPT>(o + (size_t)g * D, acc[g]);
          if (lane == 0) {
            a.ws_ml[((size_t)slot * a.Hq + h * G + g) * 2 + 0] = mg[g];
            a.ws_ml[((size_t)slot * a.Hq + h * G + g) * 2 + 1] = lg[g];
          }
        }
        __threadfence();  // publish this warp's partial rows at GPU scope before the ticket
      }
    }
    if (slot >= 0) {
      // Merge ticket of request b (every consumer warp sees the same slot). An
      // aborted CTA still gets here for each of its segments, so a counter
      // always reaches its request's partial count and is re-armed.
      named_bar_sync(1, a.NCW * 32);
      const int p0 = a.merge_indptr[b], p1 = a.merge_indptr[b + 1];
      if (threadIdx.x == 0) {
        const int prev = atomicAdd(&a.tickets[p0], 1);
        const bool last = prev == p1 - p0 - 1;
        if (last) a.tickets[p0] = 0;  // every partial has arrived: re-arm for the next call
        *s_last = last ? 1 : 0;
      }
      named_bar_sync(1, a.NCW * 32);
      if (*s_last) {
        __threadfence();
        decode_merge_request<T, D>(a, b, p0, p1, warp, lane);
      }
    } else if (a.WPH > 1) {
      named_bar_sync(1, a.NCW * 32);
    }
  }
}

}  // namespace b2a
