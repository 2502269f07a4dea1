// Decode metadata built on the device from a device page table.
//
// Reference: the per-step host work of python/minisgl_mlx/attention/metal.py:145-152
// (kv_indptr = [0, cumsum(L)], kv_indices = the valid page-table entries in
// row-major order) and scheduler/scheduler.py:155-158 (the page-table rows of
// the batch). Here the page CSR, the last-page lengths and the split-KV plan
// of b2a_decode_plan are produced by two kernels on the caller's stream, so a
// decode step needs only the batch's rows and lengths on the device and can
// be captured in a CUDA graph together with the forward pass.
//
//   decode_plan_kernel   one CTA: npages scan -> kv_indptr, last_page_len;
//                        pieces of every request (cuts at multiples of
//                        decode_share_pages(total, num_ctas) pages, the last
//                        CTA takes the rest) -> segs, merge_indptr; segment histogram per
//                        CTA -> cta_indptr. Same arithmetic as
//                        b2a_decode_plan, so the outputs are identical.
//   decode_indices_kernel  kv_indices[kv_indptr[b] + p] = page_table[row_b, p * P] / P.
//   page_table_scatter_kernel  page_table[rows[i], cols[i]] = values[i]: keeps a
//                        device copy of the host page table current with the
//                        slots a step allocates.
// Entries that would fall outside a buffer are skipped and reported through
// the device watchdog (kWdBadSlot, kWdMetaOverflow).
#pragma once
#include "common.cuh"

namespace b2a {

constexpr int kPlanThreads = 1024;
constexpr int kPlanMaxCtas = 1024;

// Pages of one CTA's share of a decode batch: the batch's pages over the CTAs, but never
// fewer than 64 tokens' worth. A tiny batch then runs on fewer CTAs with fewer split
// partials to merge (the merge reads them in a handful of L2 round trips), instead of one
// partial per page across the whole grid. Host and device plans use this one formula.
constexpr int kDecodeMinShareTokens = 64;

__host__ __device__ inline int64_t decode_share_pages(int64_t total, int num_ctas, int page_log2) {
  const int64_t floor_pages = page_log2 >= 6 ? 1 : (int64_t)(kDecodeMinShareTokens >> page_log2);
  const int64_t even = (total + num_ctas - 1) / num_ctas;
  return even > floor_pages ? even : floor_pages;
}

struct DecodeMetaArgs {
  const int32_t* page_table;
  int64_t stride;      // int32 entries per page-table row
  int64_t table_rows;  // rows in the page table
  const int32_t* rows;
  const int32_t* lens;
  int B;
  int page_log2;
  int num_ctas;
  int64_t idx_capacity;  // entries of kv_indices
  int seg_capacity;      // segments (rows of segs)
  int32_t* kv_indptr;        // [B + 1]
  int32_t* kv_indices;       // [idx_capacity]
  int32_t* last_page_len;    // [B]
  int32_t* cta_indptr;       // [num_ctas + 1]
  int32_t* segs;             // [seg_capacity, 4]
  int32_t* merge_indptr;     // [B + 1]
  int32_t* counts;           // [2]: segments, split partials
};

// Exclusive block scan of one int per thread (kPlanThreads threads); returns
// the thread's exclusive prefix and writes the block total to *total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (kPlanThreads >> 5) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive prefix of warp totals
  }
  __syncthreads();
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  const int tot = warp_sums[(kPlanThreads >> 5) - 1];
  __syncthreads();  // warp_sums is reused by the next scan
  *total = tot;
  return before;
}

__global__ void __launch_bounds__(kPlanThreads, 1) decode_plan_kernel(const DecodeMetaArgs a) {
  __shared__ int warp_sums[32];
  __shared__ int hist[kPlanMaxCtas];
  const int P = 1 << a.page_log2;
  const int C = a.num_ctas;
  for (int c = threadIdx.x; c < C; c += blockDim.x) hist[c] = 0;
  // ---- page CSR: kv_indptr, last_page_len
  int carry = 0;
  for (int base = 0; base < a.B; base += kPlanThreads) {
    const int b = base + threadIdx.x;
    int L = 0;
    if (b < a.B) {
      L = a.lens[b];
      if (L < 0 || (int64_t)L > a.stride) {
        watchdog_set(kWdMetaOverflow);
        L = L < 0 ? 0 : (int)a.stride;
      }
    }
    const int np = (L + P - 1) >> a.page_log2;
    int tot;
    const int ex = block_exclusive_scan(np, warp_sums, &tot);
    if (b < a.B) {
      a.kv_indptr[b] = carry + ex;
      a.last_page_len[b] = np > 0 ? L - ((np - 1) << a.page_log2) : 0;
    }
    carry += tot;
  }
  if (threadIdx.x == 0) a.kv_indptr[a.B] = carry;
  __syncthreads();
  const int64_t total = carry;
  const int64_t per = decode_share_pages(total, C, a.page_log2);
  // ---- pieces, segments, merge ranges
  int seg_carry = 0, part_carry = 0;
  if (threadIdx.x == 0) a.merge_indptr[0] = 0;
  for (int base = 0; base < a.B; base += kPlanThreads) {
    const int b = base + threadIdx.x;
    int64_t p0 = 0, p1 = 0;
    int c0 = 0, pieces = 0;
    if (b < a.B) {
      p0 = a.kv_indptr[b];
      p1 = a.kv_indptr[b + 1];
      c0 = (int)min(p0 / per, (int64_t)C - 1);
      const int c1 = p1 > p0 ? (int)min((p1 - 1) / per, (int64_t)C - 1) : c0;
      pieces = c1 - c0 + 1;
    }
    const bool split = pieces > 1;
    int seg_tot, part_tot;
    const int seg0 = seg_carry + block_exclusive_scan(pieces, warp_sums, &seg_tot);
    const int part0 = part_carry + block_exclusive_scan(split ? pieces : 0, warp_sums, &part_tot);
    if (b < a.B) {
      const int last = p1 > p0 ? a.last_page_len[b] : 0;
      for (int k = 0; k < pieces; ++k) {
        const int cta = c0 + k;
        const int64_t s = k == 0 ? p0 : (int64_t)cta * per;
        const int64_t cut = cta == C - 1 ? p1 : min(p1, (int64_t)(cta + 1) * per);
        int64_t ntok = (cut - s) << a.page_log2;
        if (cut == p1 && p1 > p0) ntok -= P - last;
        const int seg = seg0 + k;
        if (seg < a.seg_capacity) {
          int4 v = make_int4(b, (int)s, (int)ntok, split ? part0 + k : -1);
          reinterpret_cast<int4*>(a.segs)[seg] = v;
          atomicAdd(&hist[cta], 1);
        } else {
          watchdog_set(kWdMetaOverflow);
        }
      }
      a.merge_indptr[b + 1] = part0 + (split ? pieces : 0);
    }
    seg_carry += seg_tot;
    part_carry += part_tot;
  }
  __syncthreads();
  // ---- cta_indptr: exclusive scan of the per-CTA segment counts
  int run = 0;
  for (int base = 0; base < C; base += kPlanThreads) {
    const int c = base + threadIdx.x;
    const int h = c < C ? hist[c] : 0;
    int tot;
    const int ex = block_exclusive_scan(h, warp_sums, &tot);
    if (c < C) a.cta_indptr[c] = run + ex;
    run += tot;
  }
  if (threadIdx.x == 0) {
    a.cta_indptr[C] = run;
    a.counts[0] = seg_carry;
    a.counts[1] = part_carry;
  }
}

// One CTA per request (grid-strided): page ids of its first lens[b] tokens.
__global__ void __launch_bounds__(256) decode_indices_kernel(const DecodeMetaArgs a) {
  for (int b = blockIdx.x; b < a.B; b += gridDim.x) {
    const int64_t row = a.rows[b];
    const int64_t p0 = a.kv_indptr[b];
    const int np = a.kv_indptr[b + 1] - (int)p0;
    if (row < 0 || row >= a.table_rows) {
      if (threadIdx.x == 0) watchdog_set(kWdMetaOverflow);
      continue;
    }
    const int32_t* src = a.page_table + row * a.stride;
    for (int p = threadIdx.x; p < np; p += blockDim.x) {
      if (p0 + p >= a.idx_capacity) {
        watchdog_set(kWdMetaOverflow);
        break;
      }
      const int32_t e = src[(int64_t)p << a.page_log2];
      if (e < 0 || (e & ((1 << a.page_log2) - 1))) watchdog_set(kWdBadSlot);
      a.kv_indices[p0 + p] = e >> a.page_log2;
    }
  }
}

__global__ void page_table_scatter_kernel(int32_t* page_table, int64_t stride, int64_t table_rows,
                                          const int32_t* rows, const int32_t* cols, const int32_t* values, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = rows[i], c = cols[i];
    if (r < 0 || r >= table_rows || c < 0 || c >= stride) {
      watchdog_set(kWdMetaOverflow);
      continue;
    }
    page_table[r * stride + c] = values[i];
  }
}

}  // namespace b2a
