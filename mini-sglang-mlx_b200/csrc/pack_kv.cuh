// Pack the KV rows of a batch of requests into pages of 16 contiguous slots.
//
// The tcgen05 extend kernel gathers keys with 16-row TMA boxes, so it needs
// page_size % 16 == 0. With the reference's default page_size 1 (or any
// smaller page) the backend first copies every request's Lkv rows -- its
// cached prefix and the rows just stored -- into a staging pool where request
// b starts at slot out_page_indptr[b] * 16 and its rows are consecutive, then
// runs the tcgen05 kernel on that pool with identity page ids. One warp per
// token row (all kv heads: Hkv * D * sizeof(T) bytes) copies K and V with
// 16-byte vector loads; the copy is byte-exact.
// Row-list form (tok_indptr == NULL): row g < total copies slot kv_indices[g]
// of the pool to staging row g -- the 16-key groups of extend_groups that are
// not one run of consecutive slots, each padded to 16 rows by its caller.
#pragma once
#include "common.cuh"

namespace b2a {

constexpr int kPackPage = 16;

struct PackArgs {
  const uint8_t* k_pool;
  const uint8_t* v_pool;
  int64_t num_slots;
  const int32_t* kv_indptr;   // [B+1] page CSR of the source pool
  const int32_t* kv_indices;  // page ids
  int page_log2;
  const int32_t* tok_indptr;       // [B+1] token CSR: request b owns rows [tok_indptr[b], tok_indptr[b+1])
  const int32_t* out_page_indptr;  // [B+1] first staging page of each request
  int B;
  int64_t total;  // tok_indptr[B]
  int row_vec;    // 16-byte vectors per token row
  uint8_t* k_out;
  uint8_t* v_out;
  int64_t out_slots;
};

__global__ void __launch_bounds__(256) pack_kv_kernel(PackArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t g = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (g >= a.total) return;
  int64_t page, src, dst;
  if (a.tok_indptr == nullptr) {  // row list
    page = a.kv_indices[g];
    src = page;
    dst = g;
  } else {
    // request of row g: last b with tok_indptr[b] <= g
    int lo = 0, hi = a.B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.tok_indptr[mid] <= g) lo = mid;
      else hi = mid - 1;
    }
    const int b = lo;
    const int64_t p = g - a.tok_indptr[b];
    const int P = 1 << a.page_log2;
    page = a.kv_indices[a.kv_indptr[b] + (p >> a.page_log2)];
    src = page * P + (p & (P - 1));
    dst = (int64_t)a.out_page_indptr[b] * kPackPage + p;
  }
  if (page < 0 || src >= a.num_slots || dst >= a.out_slots) {
    if (lane == 0) watchdog_set(kWdBadSlot);
    return;
  }
  const size_t rb = (size_t)a.row_vec * 16;
  const uint4* ks = reinterpret_cast<const uint4*>(a.k_pool + (size_t)src * rb);
  const uint4* vs = reinterpret_cast<const uint4*>(a.v_pool + (size_t)src * rb);
  uint4* kd = reinterpret_cast<uint4*>(a.k_out + (size_t)dst * rb);
  uint4* vd = reinterpret_cast<uint4*>(a.v_out + (size_t)dst * rb);
  for (int i = lane; i < a.row_vec; i += 32) {
    const uint4 kv = ks[i], vv = vs[i];
    kd[i] = kv;
    vd[i] = vv;
  }
}

}  // namespace b2a
