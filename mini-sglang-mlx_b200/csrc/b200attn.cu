// C ABI of the B200 attention backend: argument validation, host-side plans,
// kernel configuration and dispatch. Declarations and contracts live in
// include/b200attn.h; each kernel file names the reference code it replaces.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "b200attn.h"
#include "common.cuh"
#include "decode.cuh"
#include "decode_mma.cuh"
#include "extend_simt.cuh"
#include "extend_tc.cuh"
#include "pack_kv.cuh"
#include "proj.cuh"
#include "metadata.cuh"
#include "rmsnorm.cuh"
#include "rope_store.cuh"
#include "swiglu.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int ok() {
  g_err.clear();
  return B2A_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B2A_ERR_CUDA, "%s: CUDA error %s", what, cudaGetErrorString(e));
  return ok();
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int ilog2_exact(int x) {
  if (x <= 0 || (x & (x - 1)) != 0) return -1;
  int l = 0;
  while ((1 << l) < x) ++l;
  return l;
}

size_t dtype_size(int dtype) {
  switch (dtype) {
    case B2A_DTYPE_F32:
      return 4;
    case B2A_DTYPE_BF16:
    case B2A_DTYPE_F16:
      return 2;
    default:
      return 0;
  }
}

// Calls f(T{}) for the element type of `dtype`; f returns an int status.
template <bool AllowF16, typename F>
int with_dtype(int dtype, F&& f) {
  switch (dtype) {
    case B2A_DTYPE_F32:
      return f(float{});
    case B2A_DTYPE_BF16:
      return f(__nv_bfloat16{});
    case B2A_DTYPE_F16:
      if constexpr (AllowF16) return f(__half{});
      return fail(B2A_ERR_UNSUPPORTED, "fp16 is supported by the store/rope kernels only");
    default:
      return fail(B2A_ERR_INVALID, "unknown dtype code %d", dtype);
  }
}

template <int D, typename F>
int with_g(int G, F&& f) {
  switch (G) {
    case 1:
      return f(std::integral_constant<int, 1>{});
    case 2:
      return f(std::integral_constant<int, 2>{});
    case 4:
      return f(std::integral_constant<int, 4>{});
    case 8:
      return f(std::integral_constant<int, 8>{});
    default:
      return fail(B2A_ERR_UNSUPPORTED, "GQA group size %d not compiled (1, 2, 4, 8)", G);
  }
}

template <typename F>
int with_d(int D, F&& f) {
  switch (D) {
    case 64:
      return f(std::integral_constant<int, 64>{});
    case 128:
      return f(std::integral_constant<int, 128>{});
    case 256:
      return f(std::integral_constant<int, 256>{});
    default:
      return fail(B2A_ERR_UNSUPPORTED, "head_dim %d not compiled (64, 128, 256)", D);
  }
}

int check_heads(int Hq, int Hkv, int D) {
  if (Hq <= 0 || Hkv <= 0 || D <= 0) return fail(B2A_ERR_INVALID, "head counts and head_dim must be > 0");
  if (Hq % Hkv != 0) return fail(B2A_ERR_INVALID, "Hq (%d) must be a multiple of Hkv (%d)", Hq, Hkv);
  if (D % 32 != 0) return fail(B2A_ERR_INVALID, "head_dim %d must be a multiple of 32", D);
  return B2A_OK;
}

// ------------------------------------------------------------ decode config
struct DecodeCfg {
  int TS, NSTAGE, WPH, NCW;
  uint32_t row_bytes, stage_bytes;
  size_t smem;
};

constexpr size_t kSmemLimit = 232448;  // opt-in dynamic shared memory per block (sm_100)

int decode_config(int Hq, int Hkv, int D, size_t es, DecodeCfg& c) {
  if (Hkv > 16 || 16 % Hkv != 0)
    return fail(B2A_ERR_UNSUPPORTED, "decode supports Hkv in {1, 2, 4, 8, 16}, got %d", Hkv);
  const int G = Hq / Hkv;
  const int TG = G <= 4 ? 8 : 32 / G;
  c.row_bytes = (uint32_t)(Hkv * D * es);
  int TS = 64;
  while (TS > 1 && 2ull * TS * c.row_bytes > 65536ull) TS >>= 1;
  // Prefer 16 consumer warps (two groups per head in flight); fall back to 8
  // when a stage cannot feed them or the combine buffer does not fit.
  for (int ncw : {16, 8}) {
    if (ncw % Hkv != 0) continue;
    const int wph = ncw / Hkv;
    // 16 warps leave 96 registers a thread: only the shapes that fit them
    if (ncw == 16 && (TS < wph * TG || D > 128 || G > 4)) continue;
    const b2a::DecodeSmem fixed = b2a::decode_smem_layout(0, 0, ncw, wph, G, D);
    const uint32_t stage = (uint32_t)TS * c.row_bytes;
    const size_t avail = kSmemLimit - fixed.total - 256;
    const int ns = (int)std::min<size_t>(4, avail / (2ull * stage));
    if (ns < 2) continue;
    c.NCW = ncw;
    c.WPH = wph;
    c.TS = TS;
    c.NSTAGE = ns;
    c.stage_bytes = stage;
    c.smem = b2a::decode_smem_layout(ns, stage, ncw, wph, G, D).total;
    return B2A_OK;
  }
  return fail(B2A_ERR_UNSUPPORTED, "decode config (Hq %d, Hkv %d, D %d) does not fit in shared memory", Hq, Hkv, D);
}

// Launch with programmatic stream serialization: the kernel may become resident
// while the previous kernel of the stream finishes (it waits in
// pdl_wait_then_release before touching memory), which hides the launch gap
// between the back-to-back kernels of a layer inside CUDA graphs.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Raises a kernel's dynamic shared-memory limit once per (kernel, device), so
// steady-state launches (and launches inside CUDA graph capture) make no
// attribute calls.
int ensure_smem(const void* kern, size_t smem, const char* what) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(B2A_ERR_CUDA, "%s: no current device", what);
  std::lock_guard<std::mutex> lock(mu);
  size_t& have = done[{kern, dev}];
  if (have >= smem) return B2A_OK;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return fail(B2A_ERR_CUDA, "%s: set smem attribute: %s", what, cudaGetErrorString(e));
  have = smem;
  return B2A_OK;
}

template <typename T, int D, int G, int NCW>
int decode_launch(const b2a::DecodeArgs& a, const DecodeCfg& c, int grid, cudaStream_t st) {
  auto kern = b2a::decode_kernel<T, D, G, NCW>;
  if (int rc = ensure_smem((const void*)kern, c.smem, "decode")) return rc;
  launch_pdl(kern, dim3(grid), dim3((c.NCW + 1) * 32), c.smem, st, a);
  return check_launch("decode_kernel");
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return n;
}

}  // namespace

// =================================================================== C ABI
extern "C" {

const char* b2a_last_error(void) { return g_err.c_str(); }

int b2a_abi_version(void) { return B2A_ABI_VERSION; }

int b2a_device_error(void* stream, int* code_out) {
  if (!code_out) return fail(B2A_ERR_INVALID, "code_out is NULL");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int code = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&code, b2a::g_watchdog, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(b2a::g_watchdog, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(B2A_ERR_CUDA, "device_error: %s", cudaGetErrorString(e));
  *code_out = code;
  return ok();
}

// ------------------------------------------------------------------ store
int b2a_rope_store(void* q, int64_t q_row_stride, void* k, int64_t k_row_stride, const void* v,
                   int64_t v_row_stride, const int32_t* positions, const int32_t* out_loc, void* k_pool,
                   void* v_pool, int64_t num_slots, const float* inv_freq, float rope_scale, int rot_dim, int T,
                   int Hq, int Hkv, int D, int dtype, void* stream) {
  return b2a_qknorm_rope_store(q, q_row_stride, nullptr, k, k_row_stride, v, v_row_stride, nullptr, nullptr, 0.f,
                               positions, out_loc, k_pool, v_pool, num_slots, inv_freq, rope_scale, rot_dim, T, Hq,
                               Hkv, D, dtype, stream);
}

int b2a_qknorm_rope_store(void* q, int64_t q_row_stride, void* q_out, void* k, int64_t k_row_stride, const void* v,
                          int64_t v_row_stride, const void* q_norm_w, const void* k_norm_w, float norm_eps,
                          const int32_t* positions, const int32_t* out_loc, void* k_pool, void* v_pool,
                          int64_t num_slots, const float* inv_freq, float rope_scale, int rot_dim, int T, int Hq,
                          int Hkv, int D, int dtype, void* stream) {
  if (T < 0) return fail(B2A_ERR_INVALID, "T must be >= 0");
  const size_t es = dtype_size(dtype);
  if ((q_norm_w || k_norm_w) && !(norm_eps >= 0.f)) return fail(B2A_ERR_INVALID, "norm_eps must be >= 0");
  if ((q_norm_w || q_out) && Hq > 0 && !q) return fail(B2A_ERR_INVALID, "q_norm_w / q_out given without q");
  if (es && ((q_norm_w && !aligned(q_norm_w, es)) || (k_norm_w && !aligned(k_norm_w, es)) ||
             (q_out && !aligned(q_out, es))))
    return fail(B2A_ERR_INVALID, "norm weights and q_out must be aligned to their element size");
  if (T == 0) return ok();
  if (Hq < 0 || Hkv <= 0 || D <= 0) return fail(B2A_ERR_INVALID, "bad head shape");
  if (rot_dim < 0 || rot_dim > D || (rot_dim & 1)) return fail(B2A_ERR_INVALID, "rot_dim %d invalid for D %d", rot_dim, D);
  const bool rotate = rot_dim > 0;
  const bool store = k_pool != nullptr || v_pool != nullptr;
  if (store && (!k_pool || !v_pool || !out_loc || !v)) return fail(B2A_ERR_INVALID, "store needs k_pool, v_pool, v, out_loc");
  if (store && num_slots <= 0) return fail(B2A_ERR_INVALID, "num_slots must be > 0");
  if (rotate && (!positions || !inv_freq)) return fail(B2A_ERR_INVALID, "rope needs positions and inv_freq");
  if (!k || ((rotate || q_norm_w) && Hq > 0 && !q)) return fail(B2A_ERR_INVALID, "q/k pointers are NULL");
  if (q_row_stride < (int64_t)Hq * D || k_row_stride < (int64_t)Hkv * D || (store && v_row_stride < (int64_t)Hkv * D))
    return fail(B2A_ERR_INVALID, "row strides smaller than a token row");
  b2a::RopeStoreArgs a;
  a.q = q;
  a.q_stride = q_row_stride;
  a.q_out = q_out;
  a.k = k;
  a.k_stride = k_row_stride;
  a.v = v;
  a.v_stride = v_row_stride;
  a.positions = positions;
  a.out_loc = out_loc;
  a.k_pool = store ? k_pool : nullptr;
  a.v_pool = store ? v_pool : nullptr;
  a.inv_freq = inv_freq;
  a.q_norm_w = q_norm_w;
  a.k_norm_w = k_norm_w;
  a.norm_eps = norm_eps;
  a.rope_scale = rope_scale;
  a.rot_dim = rot_dim;
  a.num_slots = num_slots;
  a.T = T;
  a.Hq = (rotate || q_norm_w || q_out) ? Hq : 0;  // q rows matter when rotated, normalised or moved
  a.Hkv = Hkv;
  a.D = D;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // token-major fast path: 16-bit rows, D = rot_dim = 128, every row and pointer on
  // 16 bytes (bit-identical rotation; see rope_store_tok_kernel)
  const bool tok_path = (dtype == B2A_DTYPE_BF16 || dtype == B2A_DTYPE_F16) && D == 128 && rot_dim == 128 &&
                        aligned(k, 16) && k_row_stride % 8 == 0 && (a.Hq == 0 || (aligned(q, 16) && q_row_stride % 8 == 0)) &&
                        (!q_out || aligned(q_out, 16)) && aligned(inv_freq, 16) &&
                        (!q_norm_w || aligned(q_norm_w, 16)) && (!k_norm_w || aligned(k_norm_w, 16)) &&
                        (!store || (aligned(v, 16) && v_row_stride % 8 == 0 && aligned(k_pool, 16) && aligned(v_pool, 16)));
  if (tok_path) {
    const int ng = (a.Hq + Hkv + 3) / 4;
    // warps per token: enough warps for 148 SMs at small T, one per token at large T
    const int W = (int)std::max<int64_t>(1, std::min<int64_t>({8, (int64_t)ng, (2368 + T - 1) / T}));
    const int64_t tblocks = ((int64_t)T * W + 7) / 8;
    if (tblocks > 0x7fffffff) return fail(B2A_ERR_INVALID, "too many tokens");
    if (dtype == B2A_DTYPE_BF16)
      launch_pdl(b2a::rope_store_tok_kernel<__nv_bfloat16>, dim3((unsigned)tblocks), dim3(256), 0, st, a, W);
    else
      launch_pdl(b2a::rope_store_tok_kernel<__half>, dim3((unsigned)tblocks), dim3(256), 0, st, a, W);
    return check_launch("rope_store_tok_kernel");
  }
  const int64_t rows = (int64_t)T * (a.Hq + 2 * Hkv);
  const int64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffff) return fail(B2A_ERR_INVALID, "too many rows");
  return with_dtype<true>(dtype, [&](auto tag) {
    using Tt = decltype(tag);
    launch_pdl(b2a::rope_store_kernel<Tt>, dim3((unsigned)blocks), dim3(256), 0, st, a);
    return check_launch("rope_store_kernel");
  });
}

int b2a_store_kv(const void* k, int64_t k_row_stride, const void* v, int64_t v_row_stride, const int32_t* out_loc,
                 void* k_pool, void* v_pool, int64_t num_slots, int T, int Hkv, int D, int dtype, void* stream) {
  if (!k_pool || !v_pool) return fail(B2A_ERR_INVALID, "k_pool/v_pool are NULL");
  return b2a_rope_store(nullptr, 0, const_cast<void*>(k), k_row_stride, v, v_row_stride, nullptr, out_loc, k_pool,
                        v_pool, num_slots, nullptr, 1.0f, 0, T, 0, Hkv, D, dtype, stream);
}

// ------------------------------------------------------------------ decode
int b2a_decode_plan(const int32_t* kv_indptr, const int32_t* kv_last_page_len, int B, int page_size, int num_ctas,
                    int32_t* cta_indptr, int32_t* segs, int seg_capacity, int32_t* merge_indptr, int* n_segs,
                    int* n_partials) {
  if (B < 0 || num_ctas <= 0) return fail(B2A_ERR_INVALID, "B must be >= 0 and num_ctas > 0");
  if (!kv_indptr || !cta_indptr || !segs || !merge_indptr || !n_segs || !n_partials)
    return fail(B2A_ERR_INVALID, "NULL plan argument");
  if (ilog2_exact(page_size) < 0) return fail(B2A_ERR_INVALID, "page_size %d must be a power of two", page_size);
  if (kv_indptr[0] != 0) return fail(B2A_ERR_INVALID, "kv_indptr[0] must be 0");
  for (int b = 0; b < B; ++b) {
    if (kv_indptr[b + 1] < kv_indptr[b]) return fail(B2A_ERR_INVALID, "kv_indptr not monotonic at %d", b);
    if (kv_last_page_len && kv_indptr[b + 1] > kv_indptr[b] &&
        (kv_last_page_len[b] < 1 || kv_last_page_len[b] > page_size))
      return fail(B2A_ERR_INVALID, "kv_last_page_len[%d]=%d out of [1, %d]", b, kv_last_page_len[b], page_size);
  }
  const int64_t total = kv_indptr[B];
  const int64_t per = b2a::decode_share_pages(total, num_ctas, ilog2_exact(page_size));
  int ns = 0, np = 0;
  std::fill(cta_indptr, cta_indptr + num_ctas + 1, 0);
  std::vector<int> seg_cta;
  seg_cta.reserve(B + num_ctas);
  merge_indptr[0] = 0;
  for (int b = 0; b < B; ++b) {
    const int64_t p0 = kv_indptr[b], p1 = kv_indptr[b + 1];
    const int last = (p1 > p0) ? (kv_last_page_len ? kv_last_page_len[b] : page_size) : 0;
    // pieces: page ranges cut at multiples of `per`
    int pieces = 0;
    int64_t s = p0;
    do {
      const int64_t cta = std::min<int64_t>(s / per, num_ctas - 1);
      const int64_t cut = (cta == num_ctas - 1) ? p1 : std::min<int64_t>(p1, (cta + 1) * per);
      ++pieces;
      s = cut;
    } while (s < p1);
    const bool split = pieces > 1;
    s = p0;
    do {
      const int64_t cta = std::min<int64_t>(s / per, num_ctas - 1);
      const int64_t cut = (cta == num_ctas - 1) ? p1 : std::min<int64_t>(p1, (cta + 1) * per);
      if (ns >= seg_capacity) return fail(B2A_ERR_WORKSPACE, "seg_capacity %d too small", seg_capacity);
      int64_t ntok = (cut - s) * page_size;
      if (cut == p1 && p1 > p0) ntok -= (page_size - last);
      segs[4 * ns + 0] = b;
      segs[4 * ns + 1] = (int32_t)s;
      segs[4 * ns + 2] = (int32_t)ntok;
      segs[4 * ns + 3] = split ? np++ : -1;
      seg_cta.push_back((int)cta);
      ++ns;
      s = cut;
    } while (s < p1);
    merge_indptr[b + 1] = np;
  }
  // Segments were emitted in page order, so their CTA ids are non-decreasing.
  for (int i = 0; i < ns; ++i) cta_indptr[seg_cta[i] + 1]++;
  for (int c = 0; c < num_ctas; ++c) cta_indptr[c + 1] += cta_indptr[c];
  *n_segs = ns;
  *n_partials = np;
  return ok();
}

int b2a_decode_metadata(const int32_t* page_table, int64_t table_rows, int64_t table_stride, const int32_t* rows,
                        const int32_t* lens, int B, int page_size, int num_ctas, int32_t* kv_indptr,
                        int32_t* kv_indices, int64_t idx_capacity, int32_t* kv_last_page_len, int32_t* cta_indptr,
                        int32_t* segs, int seg_capacity, int32_t* merge_indptr, int32_t* counts, void* stream) {
  if (B < 0) return fail(B2A_ERR_INVALID, "B must be >= 0");
  if (num_ctas <= 0 || num_ctas > b2a::kPlanMaxCtas)
    return fail(B2A_ERR_INVALID, "num_ctas %d out of [1, %d]", num_ctas, b2a::kPlanMaxCtas);
  const int plog = ilog2_exact(page_size);
  if (plog < 0) return fail(B2A_ERR_INVALID, "page_size %d must be a power of two", page_size);
  if (table_rows <= 0 || table_stride <= 0) return fail(B2A_ERR_INVALID, "empty page table");
  if (!page_table || !kv_indptr || !kv_indices || !kv_last_page_len || !cta_indptr || !segs || !merge_indptr ||
      !counts || (B > 0 && (!rows || !lens)))
    return fail(B2A_ERR_INVALID, "NULL metadata argument");
  if (!aligned(segs, 16)) return fail(B2A_ERR_INVALID, "segs must be 16-byte aligned (written as int4)");
  if ((int64_t)seg_capacity < (int64_t)B + num_ctas)
    return fail(B2A_ERR_WORKSPACE, "seg_capacity %d < B + num_ctas = %lld", seg_capacity, (long long)B + num_ctas);
  b2a::DecodeMetaArgs a;
  a.page_table = page_table;
  a.stride = table_stride;
  a.table_rows = table_rows;
  a.rows = rows;
  a.lens = lens;
  a.B = B;
  a.page_log2 = plog;
  a.num_ctas = num_ctas;
  a.idx_capacity = idx_capacity;
  a.seg_capacity = seg_capacity;
  a.kv_indptr = kv_indptr;
  a.kv_indices = kv_indices;
  a.last_page_len = kv_last_page_len;
  a.cta_indptr = cta_indptr;
  a.segs = segs;
  a.merge_indptr = merge_indptr;
  a.counts = counts;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  b2a::decode_plan_kernel<<<1, b2a::kPlanThreads, 0, st>>>(a);
  if (int rc = check_launch("decode_plan_kernel")) return rc;
  if (B == 0) return ok();
  b2a::decode_indices_kernel<<<std::min(B, 65535), 256, 0, st>>>(a);
  return check_launch("decode_indices_kernel");
}

int b2a_page_table_scatter(int32_t* page_table, int64_t table_rows, int64_t table_stride, const int32_t* rows,
                           const int32_t* cols, const int32_t* values, int64_t n, void* stream) {
  if (n < 0) return fail(B2A_ERR_INVALID, "n must be >= 0");
  if (n == 0) return ok();
  if (!page_table || !rows || !cols || !values) return fail(B2A_ERR_INVALID, "NULL scatter argument");
  if (table_rows <= 0 || table_stride <= 0) return fail(B2A_ERR_INVALID, "empty page table");
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 4096);
  b2a::page_table_scatter_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      page_table, table_stride, table_rows, rows, cols, values, n);
  return check_launch("page_table_scatter_kernel");
}

int b2a_decode_num_ctas(int Hq, int Hkv, int D, int dtype, int* num_ctas) {
  if (!num_ctas) return fail(B2A_ERR_INVALID, "num_ctas is NULL");
  if (int rc = check_heads(Hq, Hkv, D)) return rc;
  const size_t es = dtype_size(dtype);
  if (es == 0 || dtype == B2A_DTYPE_F16) return fail(B2A_ERR_UNSUPPORTED, "decode dtype %d", dtype);
  DecodeCfg c;
  if (int rc = decode_config(Hq, Hkv, D, es, c)) return rc;
  const int sms = num_sms();
  if (sms <= 0) return fail(B2A_ERR_CUDA, "no CUDA device");
  // One CTA per SM: the kernel is sized to own an SM's shared memory.
  const int per_sm = std::max<int>(1, (int)(kSmemLimit / (c.smem + 1024)));
  *num_ctas = sms * per_sm;
  return ok();
}

}  // extern "C"

namespace {
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Split-partial rows of a decode call: acc [n, Hq, D] then (m, l) [n, Hq, 2], fp32.
size_t decode_partial_bytes(int n_partials, int Hq, int D) {
  return align256((size_t)n_partials * Hq * D * sizeof(float)) + (size_t)n_partials * Hq * 2 * sizeof(float);
}

// Workspace layout: the merge counters (int32 [n_partials]) at its START, the
// partial rows at its END (256-byte aligned). With every call's counters at
// the front and partials at the back, no call's partials ever overlap the
// counters of another call made with a different n_partials on the same
// buffer, so counters only ever hold counts (zero between calls).
struct DecodeWs {
  int32_t* tickets;
  float* acc;
  float* ml;
};
DecodeWs decode_ws_layout(void* ws, size_t ws_bytes, int n_partials, int Hq, int D) {
  DecodeWs w;
  uint8_t* base = reinterpret_cast<uint8_t*>(ws);
  const size_t part = decode_partial_bytes(n_partials, Hq, D);
  const size_t acc_off = (ws_bytes - part) & ~(size_t)255;
  w.tickets = reinterpret_cast<int32_t*>(base);
  w.acc = reinterpret_cast<float*>(base + acc_off);
  w.ml = reinterpret_cast<float*>(base + acc_off + align256((size_t)n_partials * Hq * D * sizeof(float)));
  return w;
}
}  // namespace

extern "C" {

size_t b2a_decode_workspace_bytes(int n_partials, int Hq, int D) {
  if (n_partials <= 0) return 0;
  return align256((size_t)n_partials * sizeof(int32_t)) + decode_partial_bytes(n_partials, Hq, D);
}

static int decode_common(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
                         const int32_t* kv_indices,
                         const int32_t* kv_indptr, int page_size, const int32_t* cta_indptr, const int32_t* segs,
                         int grid, const int32_t* merge_indptr, int n_partials, int B, int Hq, int Hkv, int D,
                         float scale, void* workspace, size_t workspace_bytes, void* out, int dtype, void* stream) {
  if (B < 0) return fail(B2A_ERR_INVALID, "B must be >= 0");
  if (B == 0) return ok();
  if (int rc = check_heads(Hq, Hkv, D)) return rc;
  if (!q || !k_pool || !v_pool || !kv_indices || !out) return fail(B2A_ERR_INVALID, "NULL tensor pointer");
  if (num_slots <= 0) return fail(B2A_ERR_INVALID, "num_slots must be > 0");
  if (!aligned(q, 16) || !aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(out, 16))
    return fail(B2A_ERR_INVALID, "q/k_pool/v_pool/out must be 16-byte aligned");
  const int plog = ilog2_exact(page_size);
  if (plog < 0 || page_size > 4096) return fail(B2A_ERR_INVALID, "page_size %d must be a power of two <= 4096", page_size);
  const size_t es = dtype_size(dtype);
  if (es == 0 || dtype == B2A_DTYPE_F16) return fail(B2A_ERR_UNSUPPORTED, "decode dtype %d", dtype);
  DecodeCfg c;
  if (int rc = decode_config(Hq, Hkv, D, es, c)) return rc;
  if (n_partials < 0) return fail(B2A_ERR_INVALID, "n_partials must be >= 0");
  const size_t need = b2a_decode_workspace_bytes(n_partials, Hq, D);
  if (n_partials > 0 && (!workspace || workspace_bytes < need || !merge_indptr))
    return fail(B2A_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (workspace && !aligned(workspace, 256)) return fail(B2A_ERR_INVALID, "workspace must be 256-byte aligned");
  b2a::DecodeArgs a;
  a.q = q;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.kv_indices = kv_indices;
  a.num_slots = num_slots;
  a.kv_indptr = kv_indptr;
  a.cta_indptr = cta_indptr;
  a.segs = segs;
  a.merge_indptr = merge_indptr;
  if (n_partials > 0) {
    const DecodeWs w = decode_ws_layout(workspace, workspace_bytes, n_partials, Hq, D);
    a.tickets = w.tickets;
    a.ws_acc = w.acc;
    a.ws_ml = w.ml;
  } else {
    a.tickets = nullptr;
    a.ws_acc = a.ws_ml = nullptr;
  }
  a.B = B;
  a.n_partials = n_partials;
  a.out = out;
  a.page_log2 = plog;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.qscale = scale * b2a::kLog2e;
  a.TS = c.TS;
  a.NSTAGE = c.NSTAGE;
  a.WPH = c.WPH;
  a.NCW = c.NCW;
  a.row_bytes = c.row_bytes;
  a.stage_bytes = c.stage_bytes;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int G = Hq / Hkv;
  if (cta_indptr != nullptr && b2a::decode_mma_supported(Hq, Hkv, D, dtype, plog)) {
    // tensor-core decode: TMA boxes {64 features, 1 head, 16 tokens} per page run
    if (num_slots > 0x7fffffffLL - 64) return fail(B2A_ERR_INVALID, "decode: num_slots must be < 2^31");
    auto enc = b2a::tensor_map_encoder(g_err);
    if (!enc) return fail(B2A_ERR_CUDA, "decode: %s", g_err.c_str());
    CUtensorMap km, vm;
    const uint64_t row = (uint64_t)D * 2;
    if (!b2a::encode_3d(enc, &km, k_pool, (uint64_t)D, (uint64_t)Hkv, (uint64_t)num_slots, row, row * Hkv, 64, 1,
                        b2a::kMmaTok) ||
        !b2a::encode_3d(enc, &vm, v_pool, (uint64_t)D, (uint64_t)Hkv, (uint64_t)num_slots, row, row * Hkv, 64, 1,
                        b2a::kMmaTok))
      return fail(B2A_ERR_INVALID, "decode: cuTensorMapEncodeTiled rejected the pool tensor map");
    a.NCW = Hkv;
    a.WPH = 1;
    a.NSTAGE = b2a::decode_mma_nstage(Hkv, kSmemLimit);
    a.TS = b2a::kMmaTok;
    const size_t smem = b2a::decode_mma_smem_layout(a.NSTAGE, Hkv).total + 1024;
    auto launch = [&](auto kern) -> int {
      if (int rc = ensure_smem((const void*)kern, smem, "decode_mma")) return rc;
      launch_pdl(kern, dim3(grid), dim3((Hkv + 1) * 32), smem, st, km, vm, a);
      return check_launch("decode_mma_kernel");
    };
    switch (G) {
      case 4:
        return launch(b2a::decode_mma_kernel<4>);
      default:
        return launch(b2a::decode_mma_kernel<8>);
    }
  }
  int rc = with_dtype<false>(dtype, [&](auto tag) {
    using Tt = decltype(tag);
    return with_d(D, [&](auto dc) {
      constexpr int Dc = decltype(dc)::value;
      return with_g<Dc>(G, [&](auto gc) {
        constexpr int Gc = decltype(gc)::value;
        // split requests are merged inside the decode launch (merge tickets)
        if constexpr (Dc <= 128 && Gc <= 4) {
          return c.NCW == 16 ? decode_launch<Tt, Dc, Gc, 16>(a, c, grid, st) : decode_launch<Tt, Dc, Gc, 8>(a, c, grid, st);
        } else {
          return decode_launch<Tt, Dc, Gc, 8>(a, c, grid, st);
        }
      });
    });
  });
  return rc;
}

int b2a_paged_decode(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
                     const int32_t* kv_indptr, const int32_t* kv_indices, int B, int Hq, int Hkv, int D, float scale,
                     void* out, int dtype, void* stream) {
  if (!kv_indptr) return fail(B2A_ERR_INVALID, "kv_indptr is NULL");
  return decode_common(q, k_pool, v_pool, num_slots, kv_indices, kv_indptr, 1, nullptr, nullptr, B, nullptr, 0, B, Hq, Hkv,
                       D, scale, nullptr, 0, out, dtype, stream);
}

int b2a_decode(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots, const int32_t* kv_indices,
               int page_size,
               const int32_t* cta_indptr, const int32_t* segs, int num_ctas, const int32_t* merge_indptr,
               int n_partials, int B, int Hq, int Hkv, int D, float scale, void* workspace, size_t workspace_bytes,
               void* out, int dtype, void* stream) {
  if (!cta_indptr || !segs || num_ctas <= 0) return fail(B2A_ERR_INVALID, "decode plan missing (cta_indptr/segs)");
  if (!aligned(segs, 16)) return fail(B2A_ERR_INVALID, "segs must be 16-byte aligned (read as int4)");
  return decode_common(q, k_pool, v_pool, num_slots, kv_indices, nullptr, page_size, cta_indptr, segs, num_ctas, merge_indptr,
                       n_partials, B, Hq, Hkv, D, scale, workspace, workspace_bytes, out, dtype, stream);
}

}  // extern "C"

// ------------------------------------------------------------------ decode without allocation
// Some callers cannot allocate device memory at the point where they run
// decode: an engine whose memory planner has handed the whole device to the
// KV pool, or a host that is only allowed to pass pointers it already owns
// (pre-registered buffers, a foreign framework's tensors). For them the
// split-KV partials and merge counters live in this file-scope device array
// instead of a caller-provided workspace. The array is part of the library
// image, so every GPU that loads the library keeps it until the process exits.
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;  // 8 MiB of split partials per device
__device__ __align__(256) uint8_t g_decode_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
// Device address of g_decode_scratch, per device ordinal. Written and read
// atomically, so first calls from several host threads are well defined (they
// all store the same address). It is refreshed by every call made outside
// stream capture: after cudaDeviceReset, or with another context current, the
// module is loaded again and the array may move, so a cached address is only
// trusted while a capture is in progress (capture cannot follow a reset
// without a non-captured call, which refreshes it).
std::atomic<void*> g_decode_scratch_addr[kMaxDevices];

}  // namespace

extern "C" int b2a_decode_noalloc(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
                                  const int32_t* kv_indices, int page_size, const int32_t* cta_indptr,
                                  const int32_t* segs, int num_ctas, const int32_t* merge_indptr, int n_partials,
                                  int B, int Hq, int Hkv, int D, float scale, void* out, int dtype, void* stream) {
  if (!cta_indptr || !segs || num_ctas <= 0) return fail(B2A_ERR_INVALID, "decode plan missing (cta_indptr/segs)");
  if (!aligned(segs, 16)) return fail(B2A_ERR_INVALID, "segs must be 16-byte aligned (read as int4)");
  if (n_partials < 0) return fail(B2A_ERR_INVALID, "n_partials must be >= 0");
  const size_t need = b2a_decode_workspace_bytes(n_partials, Hq, D);
  if (need > kNoAllocScratchBytes)
    return fail(B2A_ERR_WORKSPACE,
                "b2a_decode_noalloc: %d split partials need %zu bytes, above the %zu-byte static scratch; "
                "use b2a_decode with a workspace or a plan with fewer CTAs",
                n_partials, need, kNoAllocScratchBytes);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(B2A_ERR_CUDA, "b2a_decode_noalloc: no usable current device (%s)", cudaGetErrorString(e));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(st, &cap);
  if (e != cudaSuccess) return fail(B2A_ERR_CUDA, "b2a_decode_noalloc: %s", cudaGetErrorString(e));
  void* scratch = nullptr;
  if (cap == cudaStreamCaptureStatusNone) {
    // Set-up on this device, with the device current: the host-side symbol is
    // only a stand-in, the kernel needs the array's device address.
    e = cudaGetSymbolAddress(&scratch, g_decode_scratch);
    if (e != cudaSuccess || !scratch)
      return fail(B2A_ERR_CUDA, "b2a_decode_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_decode_scratch_addr[dev].store(scratch, std::memory_order_release);
  } else {
    scratch = g_decode_scratch_addr[dev].load(std::memory_order_acquire);
    if (!scratch)
      return fail(B2A_ERR_INVALID,
                  "b2a_decode_noalloc: the first call on a device must come before any stream capture");
  }
  // The array keeps the last call's contents. The merge counters at its start
  // must be zero: a completed call leaves them so, but a call cut short by a
  // device error may not, so they are cleared here (a memset, no allocation).
  // Partial rows need no clearing: each is written before it is read.
  if (n_partials > 0) {
    e = cudaMemsetAsync(scratch, 0, (size_t)n_partials * sizeof(int32_t), st);
    if (e != cudaSuccess) return fail(B2A_ERR_CUDA, "b2a_decode_noalloc: clear counters: %s", cudaGetErrorString(e));
  }
  return decode_common(q, k_pool, v_pool, num_slots, kv_indices, nullptr, page_size, cta_indptr, segs, num_ctas,
                       merge_indptr, n_partials, B, Hq, Hkv, D, scale, scratch, kNoAllocScratchBytes, out, dtype,
                       stream);
}

extern "C" {

// ------------------------------------------------------------------ extend
static bool extend_uses_tc(int Hq, int Hkv, int D, int dtype, int page_log2) {
  return b2a::extend_tc_supported(Hq, Hkv, D, dtype) && b2a::extend_tc_page_ok(page_log2);
}

int b2a_extend_tile_q(int Hq, int Hkv, int D, int dtype, int page_size, int* tile_q) {
  if (!tile_q) return fail(B2A_ERR_INVALID, "tile_q is NULL");
  if (int rc = check_heads(Hq, Hkv, D)) return rc;
  const int plog = ilog2_exact(page_size);
  if (plog < 0) return fail(B2A_ERR_INVALID, "page_size %d must be a power of two", page_size);
  const int G = Hq / Hkv;
  if (extend_uses_tc(Hq, Hkv, D, dtype, plog)) {
    *tile_q = b2a::extend_tc_tile_tokens(G);
  } else {
    if (G > b2a::kSimtRows) return fail(B2A_ERR_UNSUPPORTED, "GQA group %d too large", G);
    *tile_q = b2a::kSimtRows / G;
  }
  return ok();
}

int b2a_pack_kv(const void* k_pool, const void* v_pool, int64_t num_slots, const int32_t* kv_indptr,
                const int32_t* kv_indices, int page_size, const int32_t* tok_indptr, const int32_t* out_page_indptr,
                int B, int64_t total_tokens, int Hkv, int D, int dtype, void* k_out, void* v_out, int64_t out_slots,
                void* stream) {
  if (B < 0 || total_tokens < 0) return fail(B2A_ERR_INVALID, "negative size");
  if (B == 0 || total_tokens == 0) return ok();
  const bool row_list = tok_indptr == nullptr;
  if (row_list && (kv_indptr || out_page_indptr || page_size != 1))
    return fail(B2A_ERR_INVALID, "row-list pack: kv_indptr and out_page_indptr NULL, page_size 1");
  if (row_list && total_tokens > out_slots) return fail(B2A_ERR_INVALID, "row-list pack: total_tokens > out_slots");
  const size_t es = dtype_size(dtype);
  if (es == 0) return fail(B2A_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (Hkv <= 0 || D <= 0) return fail(B2A_ERR_INVALID, "bad head shape");
  const size_t row = (size_t)Hkv * D * es;
  if (row % 16) return fail(B2A_ERR_INVALID, "token rows of %zu bytes are not a multiple of 16", row);
  if (!k_pool || !v_pool || !kv_indices || !k_out || !v_out || (!row_list && (!kv_indptr || !out_page_indptr)))
    return fail(B2A_ERR_INVALID, "NULL pointer argument");
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(k_out, 16) || !aligned(v_out, 16))
    return fail(B2A_ERR_INVALID, "pools must be 16-byte aligned");
  const int plog = ilog2_exact(page_size);
  if (plog < 0) return fail(B2A_ERR_INVALID, "page_size %d must be a power of two", page_size);
  if (num_slots <= 0 || out_slots <= 0) return fail(B2A_ERR_INVALID, "num_slots/out_slots must be > 0");
  b2a::PackArgs a;
  a.k_pool = reinterpret_cast<const uint8_t*>(k_pool);
  a.v_pool = reinterpret_cast<const uint8_t*>(v_pool);
  a.num_slots = num_slots;
  a.kv_indptr = kv_indptr;
  a.kv_indices = kv_indices;
  a.page_log2 = plog;
  a.tok_indptr = tok_indptr;
  a.out_page_indptr = out_page_indptr;
  a.B = B;
  a.total = total_tokens;
  a.row_vec = (int)(row / 16);
  a.k_out = reinterpret_cast<uint8_t*>(k_out);
  a.v_out = reinterpret_cast<uint8_t*>(v_out);
  a.out_slots = out_slots;
  const int64_t blocks = (total_tokens + 7) / 8;
  if (blocks > 0x7fffffff) return fail(B2A_ERR_INVALID, "too many rows");
  b2a::pack_kv_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("pack_kv_kernel");
}

int b2a_swiglu(const void* gate_up, int64_t row_stride, void* out, int64_t rows, int F, int dtype, void* stream) {
  if (rows < 0 || F < 0) return fail(B2A_ERR_INVALID, "negative size");
  if (rows == 0 || F == 0) return ok();
  if (F % 2) return fail(B2A_ERR_INVALID, "F = %d must be even", F);
  if (row_stride < 2 * (int64_t)F) return fail(B2A_ERR_INVALID, "row_stride %lld < 2F", (long long)row_stride);
  if (!gate_up || !out) return fail(B2A_ERR_INVALID, "NULL pointer argument");
  const int64_t n = rows * (F / 2);
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return with_dtype<true>(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    b2a::swiglu_kernel<T><<<blocks, 256, 0, st>>>(reinterpret_cast<const T*>(gate_up), row_stride,
                                                   reinterpret_cast<T*>(out), rows, F);
    return check_launch("swiglu_kernel");
  });
}

int b2a_rmsnorm(const void* x, int64_t x_row_stride, int64_t x_rows, const int32_t* rows, int64_t n_rows,
                const void* w, float eps, int H, void* y, int dtype, void* stream) {
  if (n_rows < 0 || x_rows < 0) return fail(B2A_ERR_INVALID, "negative row count");
  if (n_rows == 0) return ok();
  if (!x || !w || !y) return fail(B2A_ERR_INVALID, "NULL pointer argument");
  if (!rows && n_rows > x_rows) return fail(B2A_ERR_INVALID, "n_rows %lld > x_rows %lld without a gather",
                                           (long long)n_rows, (long long)x_rows);
  if (!(eps >= 0.f)) return fail(B2A_ERR_INVALID, "eps must be >= 0");
  const size_t es = dtype_size(dtype);
  if (es == 0) return fail(B2A_ERR_UNSUPPORTED, "dtype %d", dtype);
  const int ev = (int)(16 / es);
  if (H <= 0 || H % (32 * ev)) return fail(B2A_ERR_UNSUPPORTED, "H = %d must be a multiple of %d", H, 32 * ev);
  const int vpl = H / (32 * ev);
  if (x_row_stride < H || (x_row_stride * (int64_t)es) % 16)
    return fail(B2A_ERR_INVALID, "x_row_stride %lld: >= H and 16-byte multiple rows needed", (long long)x_row_stride);
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(w, 16)) return fail(B2A_ERR_INVALID, "x/y/w must be 16-byte aligned");
  if ((n_rows + 7) / 8 > 0x7fffffff) return fail(B2A_ERR_INVALID, "too many rows");
  b2a::RmsNormArgs a;
  a.x = x;
  a.x_stride = x_row_stride;
  a.rows = rows;
  a.x_rows = x_rows;
  a.y = y;
  a.w = w;
  a.n_rows = n_rows;
  a.H = H;
  a.eps = eps;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((n_rows + 7) / 8));
  return with_dtype<true>(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    switch (vpl) {
      case 1:
        launch_pdl(b2a::rmsnorm_kernel<T, 1>, grid, dim3(256), 0, st, a);
        break;
      case 2:
        launch_pdl(b2a::rmsnorm_kernel<T, 2>, grid, dim3(256), 0, st, a);
        break;
      case 4:
        launch_pdl(b2a::rmsnorm_kernel<T, 4>, grid, dim3(256), 0, st, a);
        break;
      case 8:
        launch_pdl(b2a::rmsnorm_kernel<T, 8>, grid, dim3(256), 0, st, a);
        break;
      case 16:
        launch_pdl(b2a::rmsnorm_kernel<T, 16>, grid, dim3(256), 0, st, a);
        break;
      default:
        return fail(B2A_ERR_UNSUPPORTED, "H = %d: %d vectors per lane not compiled (1, 2, 4, 8, 16)", H, vpl);
    }
    return check_launch("rmsnorm_kernel");
  });
}

int b2a_extend_plan(const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_last_page_len, int B,
                    int page_size, int tile_q, int32_t* work, int work_capacity, int* n_work) {
  if (!qo_indptr || !kv_indptr || !work || !n_work) return fail(B2A_ERR_INVALID, "NULL plan argument");
  if (B < 0 || tile_q <= 0) return fail(B2A_ERR_INVALID, "B must be >= 0, tile_q > 0");
  if (ilog2_exact(page_size) < 0) return fail(B2A_ERR_INVALID, "page_size %d must be a power of two", page_size);
  struct Item {
    int r, tb, nq;
    int64_t cost;
  };
  std::vector<Item> items;
  for (int r = 0; r < B; ++r) {
    const int Lq = qo_indptr[r + 1] - qo_indptr[r];
    const int np = kv_indptr[r + 1] - kv_indptr[r];
    if (Lq < 0 || np < 0) return fail(B2A_ERR_INVALID, "indptr not monotonic at request %d", r);
    const int last = np > 0 ? (kv_last_page_len ? kv_last_page_len[r] : page_size) : 0;
    if (np > 0 && (last < 1 || last > page_size))
      return fail(B2A_ERR_INVALID, "kv_last_page_len[%d]=%d out of [1, %d]", r, last, page_size);
    const int64_t Lkv = np > 0 ? (int64_t)(np - 1) * page_size + last : 0;
    if (Lkv < Lq) return fail(B2A_ERR_INVALID, "request %d: kv length %lld < query length %d", r, (long long)Lkv, Lq);
    const int64_t prefix = Lkv - Lq;
    for (int tb = 0; tb < Lq; tb += tile_q) {
      const int nq = std::min(tile_q, Lq - tb);
      items.push_back({r, tb, nq, (int64_t)nq * (prefix + tb + nq)});
    }
  }
  if ((int)items.size() > work_capacity) return fail(B2A_ERR_WORKSPACE, "work_capacity %d < %zu tiles", work_capacity, items.size());
  std::stable_sort(items.begin(), items.end(), [](const Item& x, const Item& y) { return x.cost > y.cost; });
  for (size_t i = 0; i < items.size(); ++i) {
    work[4 * i + 0] = items[i].r;
    work[4 * i + 1] = items[i].tb;
    work[4 * i + 2] = items[i].nq;
    work[4 * i + 3] = 0;
  }
  *n_work = (int)items.size();
  return ok();
}

int b2a_extend(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots, const int32_t* qo_indptr,
               const int32_t* kv_indptr, const int32_t* kv_indices, const int32_t* kv_last_page_len, int page_size,
               const int32_t* work, int n_work, int T, int B, int Hq, int Hkv, int D, float scale, void* out,
               int dtype, void* stream) {
  if (n_work < 0 || B < 0 || T < 0) return fail(B2A_ERR_INVALID, "negative size");
  if (n_work == 0) return ok();
  if (int rc = check_heads(Hq, Hkv, D)) return rc;
  if (!q || !k_pool || !v_pool || !qo_indptr || !kv_indptr || !kv_indices || !work || !out)
    return fail(B2A_ERR_INVALID, "NULL pointer argument");
  if (!aligned(work, 16)) return fail(B2A_ERR_INVALID, "work must be 16-byte aligned (read as int4)");
  if (!aligned(q, 16) || !aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(out, 16))
    return fail(B2A_ERR_INVALID, "q/k_pool/v_pool/out must be 16-byte aligned");
  const int plog = ilog2_exact(page_size);
  if (plog < 0) return fail(B2A_ERR_INVALID, "page_size %d must be a power of two", page_size);
  if (num_slots <= 0) return fail(B2A_ERR_INVALID, "num_slots must be > 0");
  if (dtype == B2A_DTYPE_F16 || dtype_size(dtype) == 0) return fail(B2A_ERR_UNSUPPORTED, "extend dtype %d", dtype);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int G = Hq / Hkv;
  if (extend_uses_tc(Hq, Hkv, D, dtype, plog)) {
    if (int rc = ensure_smem((const void*)b2a::extend_tc2_kernel, b2a::Tc2Smem::ALLOC, "extend_tc")) return rc;
    return b2a::extend_tc_launch(q, k_pool, v_pool, num_slots, nullptr, nullptr, 0, 0, qo_indptr, kv_indptr,
                                 kv_indices, kv_last_page_len, plog, work, n_work, T, Hq, Hkv, scale, out, st, g_err);
  }
  if (G > b2a::kSimtRows) return fail(B2A_ERR_UNSUPPORTED, "GQA group %d too large", G);
  b2a::ExtendArgs a;
  a.q = q;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.qo_indptr = qo_indptr;
  a.kv_indptr = kv_indptr;
  a.kv_indices = kv_indices;
  a.kv_last_page_len = kv_last_page_len;
  a.work = work;
  a.out = out;
  a.num_slots = num_slots;
  a.page_log2 = plog;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.qscale = scale * b2a::kLog2e;
  return with_dtype<false>(dtype, [&](auto tag) {
    using Tt = decltype(tag);
    return with_d(D, [&](auto dc) {
      constexpr int Dc = decltype(dc)::value;
      return with_g<Dc>(G, [&](auto gc) {
        constexpr int Gc = decltype(gc)::value;
        auto kern = b2a::extend_simt_kernel<Tt, Dc, Gc>;
        const size_t smem = b2a::extend_simt_smem(Dc);
        if (int rc = ensure_smem((const void*)kern, smem, "extend")) return rc;
        kern<<<dim3(n_work, Hkv), b2a::kSimtThreads, smem, st>>>(a);
        return check_launch("extend_simt_kernel");
      });
    });
  });
}

int b2a_extend_groups(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots, const void* k_stage,
                      const void* v_stage, int64_t stage_slots, const int32_t* qo_indptr, const int32_t* group_indptr,
                      const int32_t* group_starts, const int32_t* kv_last_len, const int32_t* work, int n_work, int T,
                      int B, int Hq, int Hkv, int D, float scale, void* out, int dtype, void* stream) {
  if (n_work < 0 || B < 0 || T < 0 || stage_slots < 0) return fail(B2A_ERR_INVALID, "negative size");
  if (n_work == 0) return ok();
  if (int rc = check_heads(Hq, Hkv, D)) return rc;
  if (!extend_uses_tc(Hq, Hkv, D, dtype, 4))
    return fail(B2A_ERR_UNSUPPORTED, "extend_groups: the tcgen05 path only (bf16, D 128, GQA group 1/2/4/8)");
  if (!q || !k_pool || !v_pool || !qo_indptr || !group_indptr || !group_starts || !work || !out ||
      (stage_slots > 0 && (!k_stage || !v_stage)))
    return fail(B2A_ERR_INVALID, "NULL pointer argument");
  if (!aligned(work, 16)) return fail(B2A_ERR_INVALID, "work must be 16-byte aligned (read as int4)");
  if (!aligned(q, 16) || !aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(out, 16) ||
      (stage_slots > 0 && (!aligned(k_stage, 16) || !aligned(v_stage, 16))))
    return fail(B2A_ERR_INVALID, "q/pools/out must be 16-byte aligned");
  if (num_slots <= 0 || num_slots + stage_slots > 0x7fffffffLL - 64)
    return fail(B2A_ERR_INVALID, "num_slots + stage_slots must be in (0, 2^31)");
  if (int rc = ensure_smem((const void*)b2a::extend_tc2_kernel, b2a::Tc2Smem::ALLOC, "extend_tc")) return rc;
  return b2a::extend_tc_launch(q, k_pool, v_pool, num_slots, k_stage, v_stage, stage_slots, 1, qo_indptr,
                               group_indptr, group_starts, kv_last_len, 4, work, n_work, T, Hq, Hkv, scale, out,
                               reinterpret_cast<cudaStream_t>(stream), g_err);
}

}  // extern "C"

namespace {

// Projection launch shape: CTAs of `warps` warps, each warp `kpw` 128-wide k
// slices. The widest split (most warps) whose grid is resident in one wave is
// taken, so the whole weight stream is in flight at once; residency is the
// occupancy calculator's, cached per (kernel, warps).
template <int NB, int A, int MODE, bool NORM>
int proj_launch(const b2a::ProjArgs& a0, int grid, cudaStream_t st) {
  // 512-thread CTAs cap a thread at 128 registers: too few for 64 token rows, for the
  // paired SwiGLU tiles and for the normalised operand batches; those take 8 warps
  constexpr int MAXW = (NB == 8 || A == 2 || NORM) ? 8 : 16;
  auto kern = b2a::proj_kernel<NB, A, MODE, NORM, MAXW>;
  using S = b2a::ProjSmem<NB, A>;
  const int kc = a0.K / 128;
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, int> resident;  // (device, warps, K) -> CTAs per SM
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(B2A_ERR_CUDA, "proj: no current device");
  const int sms = num_sms();
  int warps = 0;
  for (int wc = std::min(MAXW, kc); wc >= 1; --wc) {
    if (kc % wc) continue;
    const size_t smem = S::bytes(a0.K, wc);
    if (smem > 227 * 1024) continue;
    if (int rc = ensure_smem((const void*)kern, smem, "proj")) return rc;
    int per_sm = 0;
    {
      std::lock_guard<std::mutex> lock(mu);
      auto it = resident.find({dev, wc, a0.K});
      if (it != resident.end()) {
        per_sm = it->second;
      } else {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, wc * 32, smem) != cudaSuccess)
          return fail(B2A_ERR_CUDA, "proj: occupancy query failed");
        resident[{dev, wc, a0.K}] = per_sm;
      }
    }
    if (warps == 0 && per_sm > 0) warps = wc;  // the widest split that runs at all
    if (per_sm > 0 && (int64_t)per_sm * sms >= grid) {
      warps = wc;
      break;
    }
  }
  if (warps == 0) return fail(B2A_ERR_UNSUPPORTED, "proj: no launchable warp count for K = %d", a0.K);
  b2a::ProjArgs a = a0;
  a.kpw = kc / warps;
  launch_pdl(kern, dim3((unsigned)grid), dim3(warps * 32), S::bytes(a0.K, warps), st, a);
  return check_launch("proj_kernel");
}

template <int NB>
int proj_tiles(const b2a::ProjArgs& a, int mode, bool norm, int grid, cudaStream_t st) {
  switch (mode) {
    case b2a::kProjPlain:
      return norm ? proj_launch<NB, 1, b2a::kProjPlain, true>(a, grid, st)
                  : proj_launch<NB, 1, b2a::kProjPlain, false>(a, grid, st);
    case b2a::kProjResidual:
      return norm ? proj_launch<NB, 1, b2a::kProjResidual, true>(a, grid, st)
                  : proj_launch<NB, 1, b2a::kProjResidual, false>(a, grid, st);
    default:
      return norm ? proj_launch<NB, 2, b2a::kProjSwiglu, true>(a, grid, st)
                  : proj_launch<NB, 2, b2a::kProjSwiglu, false>(a, grid, st);
  }
}

}  // namespace

extern "C" int b2a_proj(const void* x, int64_t x_row_stride, int M, int K, const void* w, int N,
                        const void* norm_w, float eps, const void* res, int64_t res_row_stride, void* out,
                        int64_t out_row_stride, int mode, int dtype, void* stream) {
  if (M < 0 || K < 0 || N < 0) return fail(B2A_ERR_INVALID, "negative size");
  if (mode < b2a::kProjPlain || mode > b2a::kProjSwiglu) return fail(B2A_ERR_INVALID, "unknown proj mode %d", mode);
  if (dtype != B2A_DTYPE_BF16) return fail(B2A_ERR_UNSUPPORTED, "proj: bf16 only (dtype %d)", dtype);
  if (M == 0 || N == 0) return ok();
  if (M > 64) return fail(B2A_ERR_UNSUPPORTED, "proj: M = %d token rows (at most 64)", M);
  if (K == 0 || K % 128) return fail(B2A_ERR_UNSUPPORTED, "proj: K = %d must be a positive multiple of 128", K);
  const int n_out = mode == b2a::kProjSwiglu ? N / 2 : N;
  if (mode == b2a::kProjSwiglu ? N % 32 : N % 16)
    return fail(B2A_ERR_UNSUPPORTED, "proj: N = %d must be a multiple of %d", N, mode == b2a::kProjSwiglu ? 32 : 16);
  if (!x || !w || !out || (mode == b2a::kProjResidual && !res)) return fail(B2A_ERR_INVALID, "NULL pointer argument");
  if (!aligned(x, 16) || !aligned(w, 16) || (norm_w && !aligned(norm_w, 16)))
    return fail(B2A_ERR_INVALID, "proj: x, w and norm_w must be 16-byte aligned");
  if (!aligned(out, 2) || (res && !aligned(res, 2))) return fail(B2A_ERR_INVALID, "proj: out/res misaligned");
  if (x_row_stride < K || x_row_stride % 8) return fail(B2A_ERR_INVALID, "proj: x_row_stride %lld (>= K, multiple of 8)",
                                                       (long long)x_row_stride);
  if (out_row_stride < n_out) return fail(B2A_ERR_INVALID, "proj: out_row_stride %lld < %d", (long long)out_row_stride, n_out);
  if (mode == b2a::kProjResidual && res_row_stride < N)
    return fail(B2A_ERR_INVALID, "proj: res_row_stride %lld < N", (long long)res_row_stride);
  if (!(eps >= 0.f)) return fail(B2A_ERR_INVALID, "eps must be >= 0");
  b2a::ProjArgs a;
  a.x = reinterpret_cast<const __nv_bfloat16*>(x);
  a.w = reinterpret_cast<const __nv_bfloat16*>(w);
  a.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w);
  a.res = reinterpret_cast<const __nv_bfloat16*>(res);
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ldx = x_row_stride;
  a.ldr = res_row_stride;
  a.ldo = out_row_stride;
  a.M = M;
  a.K = K;
  a.F = N / 2;
  a.kpw = 0;
  a.eps = eps;
  // a CTA holds 16 weight rows (a 16-row gate tile and a 16-row up tile for swiglu)
  const int A = mode == b2a::kProjSwiglu ? 2 : 1;
  const int grid = N / (16 * A);
  if ((size_t)16 * A * (2 * (size_t)K + 64) + 16 > 227 * 1024)
    return fail(B2A_ERR_UNSUPPORTED, "proj: K = %d: the %d-row weight slab does not fit in shared memory", K, 16 * A);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool norm = norm_w != nullptr;
  if (M <= 8) return proj_tiles<1>(a, mode, norm, grid, st);
  if (M <= 16) return proj_tiles<2>(a, mode, norm, grid, st);
  if (M <= 32) return proj_tiles<4>(a, mode, norm, grid, st);
  return proj_tiles<8>(a, mode, norm, grid, st);
}
