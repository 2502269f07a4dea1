/*
 * b200attn.h - C ABI of the B200 attention backend for mini-sglang-mlx.
 *
 * The library (libb200attn.so) replaces the reference's attention hot path:
 * the KV-pool store, the rotary embedding applied in AttentionLayer, the
 * shared prefill/extend attention and the paged decode attention. Every entry
 * point takes plain device pointers, sizes and a CUDA stream (cudaStream_t
 * passed as void*); nothing here knows about torch, MLX or Python objects.
 *
 * Conventions
 *   - Status: every int-returning call returns B2A_OK (0) or a nonzero
 *     B2A_ERR_* code; b2a_last_error() returns the message of the last failing
 *     call made on this host thread.
 *   - dtype: B2A_DTYPE_F32 or B2A_DTYPE_BF16 (B2A_DTYPE_F16 is accepted by the
 *     store/rope kernels only). All activations and pools share one dtype.
 *   - Layouts (row-major, innermost last):
 *       q, out           [T, Hq, D]   (decode: T = B, one query row per request)
 *       k, v (new rows)  [T, Hkv, D]  with an explicit token-row stride
 *       k_pool, v_pool   [num_slots, Hkv, D] for ONE layer
 *   - Paging: a page is page_size consecutive pool slots starting at a
 *     multiple of page_size. kv_indptr[B+1] is a CSR over pages,
 *     kv_indices[] holds page ids (slot / page_size) and kv_last_page_len[B]
 *     the number of valid slots in each request's last page (NULL means every
 *     last page is full). With
 *     page_size == 1 this is exactly the token CSR of the reference's Metal
 *     backend (kv_indptr = [0, cumsum(L)], kv_indices = slots).
 *   - Bounds: every page id / slot is checked on the device against
 *     num_slots; an out-of-range index skips the access and sets the watchdog
 *     word (b2a_device_error) instead of faulting.
 *   - Allocation: no entry point allocates device memory. Scratch comes from
 *     a caller-provided workspace sized by the *_workspace_bytes queries.
 *   - Threading: calls are re-entrant across streams; the host-side error
 *     string is thread-local. Plans are pure host functions.
 */
#ifndef B200ATTN_H
#define B200ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2A_ABI_VERSION 1

#define B2A_DTYPE_F32 0
#define B2A_DTYPE_BF16 1
#define B2A_DTYPE_F16 2

#define B2A_OK 0
#define B2A_ERR_INVALID 1     /* bad argument (shape, pointer, alignment) */
#define B2A_ERR_UNSUPPORTED 2 /* valid but not compiled (e.g. head_dim 96) */
#define B2A_ERR_CUDA 3        /* CUDA launch/runtime error                 */
#define B2A_ERR_WORKSPACE 4   /* workspace or plan capacity too small      */

/* Message of the last failing call on this host thread ("" if none). */
const char* b2a_last_error(void);

/* B2A_ABI_VERSION of the loaded library. */
int b2a_abi_version(void);

/* Reads and clears the device-side watchdog word that bounded spin-waits
 * set when they give up (0 = no error). Synchronises `stream`. */
int b2a_device_error(void* stream, int* code_out);

/* ------------------------------------------------------------------------
 * KV-pool store.
 * Replaces MHAKVCache.store_kv (python/minisgl_mlx/kvcache/pool.py:47-50):
 *   k_pool[out_loc[t]] = k[t];  v_pool[out_loc[t]] = v[t]   for t < T.
 * Byte-exact copy. out_loc entries must be unique and < num_slots.
 * ------------------------------------------------------------------------ */
int b2a_store_kv(const void* k, int64_t k_row_stride, const void* v, int64_t v_row_stride,
                 const int32_t* out_loc, void* k_pool, void* v_pool, int64_t num_slots, int T,
                 int Hkv, int D, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Fused rotary embedding + KV store.
 * Replaces the first three lines of AttentionLayer.__call__
 * (python/minisgl_mlx/layers.py:107-109): RotaryEmbedding (layers.py:45-56,
 * mx.fast.rope with traditional=False) on q and k, then store_kv of the
 * rotated k and the untouched v (kvcache/pool.py:47-50).
 *   angle(t, i) = fl32(fl32(positions[t] * rope_scale) * inv_freq[i]),
 *   i < rot_dim/2; pairs (i, i + rot_dim/2) are rotated, features >= rot_dim
 *   pass through. q and k are rotated IN PLACE (row strides in elements).
 * inv_freq: device float32[rot_dim/2] (base^(-2i/rot_dim), or 1/freqs for
 * llama3 scaling). rot_dim == 0 disables the rotation (pure store);
 * k_pool == v_pool == NULL disables the store (pure rope).
 * ------------------------------------------------------------------------ */
int b2a_rope_store(void* q, int64_t q_row_stride, void* k, int64_t k_row_stride, const void* v,
                   int64_t v_row_stride, const int32_t* positions, const int32_t* out_loc,
                   void* k_pool, void* v_pool, int64_t num_slots, const float* inv_freq,
                   float rope_scale, int rot_dim, int T, int Hq, int Hkv, int D, int dtype,
                   void* stream);

/* ------------------------------------------------------------------------
 * b2a_rope_store with the per-head q/k RMSNorm of Qwen3 fused in front.
 * No single reference function: it merges the q_norm / k_norm calls of
 * Attention.__call__ (python/minisgl_mlx/models/transformer.py:54-56, MLX
 * nn.RMSNorm over head_dim) into the call b2a_rope_store replaces.
 * Each q (k) head row x of D elements becomes
 *   y = x * 1 / sqrt(mean(x^2) + norm_eps) * w,  w = q_norm_w (k_norm_w),
 * rounded to `dtype`, then rotated and stored exactly as b2a_rope_store.
 * q_norm_w / k_norm_w: device arrays of D elements of `dtype`; either may be
 * NULL (that kind is not normalised). q_out: NULL (q is normalised and
 * rotated in place), or a contiguous [T, Hq, D] destination for the final q
 * rows, in which case q's rows are scratch (e.g. q is a strided view of a
 * fused qkv projection and q_out feeds the attention call directly).
 * With q_out, q_norm_w and k_norm_w all NULL this is b2a_rope_store.
 * ------------------------------------------------------------------------ */
int b2a_qknorm_rope_store(void* q, int64_t q_row_stride, void* q_out, void* k, int64_t k_row_stride, const void* v,
                          int64_t v_row_stride, const void* q_norm_w, const void* k_norm_w,
                          float norm_eps, const int32_t* positions, const int32_t* out_loc,
                          void* k_pool, void* v_pool, int64_t num_slots, const float* inv_freq,
                          float rope_scale, int rot_dim, int T, int Hq, int Hkv, int D, int dtype,
                          void* stream);

/* ------------------------------------------------------------------------
 * Paged decode attention, drop-in form.
 * Same inputs and meaning as paged_decode_attention
 * (python/minisgl_mlx/attention/metal.py:112-131): one query row per request,
 * kv_indptr[B+1] token CSR, kv_indices[] pool slots (page_size 1),
 *   out[b, h] = softmax(scale * q[b,h] . K[idx]^T) . V[idx],
 *   idx = kv_indices[kv_indptr[b] : kv_indptr[b+1]], kv head = h / (Hq/Hkv).
 * One CTA per request, no split, no workspace. fp32 accumulation.
 * ------------------------------------------------------------------------ */
int b2a_paged_decode(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
                     const int32_t* kv_indptr, const int32_t* kv_indices, int B, int Hq, int Hkv,
                     int D, float scale, void* out, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Paged split-KV decode attention, production form.
 * Replaces MetalAttnBackend.prepare_decode/forward_decode
 * (python/minisgl_mlx/attention/metal.py:145-162) and the naive backend's
 * forward_decode (attention/naive.py:50-60), which computes the same values.
 *
 * b2a_decode_plan (host only, no GPU): cuts the concatenated page stream of
 * all requests into `num_ctas` near-equal contiguous ranges of at least 64
 * tokens' worth of pages each (a small batch leaves the last CTAs without
 * work rather than splitting every page into its own partial). Each range is a
 * list of segments {request, first page index into kv_indices, n_tokens,
 * out_slot}; out_slot == -1 writes the final output directly, otherwise the
 * segment writes a partial (m, l, acc) that b2a_decode merges per request.
 *   kv_indptr, kv_last_page_len : HOST int32 [B+1], [B] (NULL = full pages)
 *   cta_indptr (out)            : int32 [num_ctas + 1] CSR over segments
 *   segs (out)                  : int32 [seg_capacity * 4]
 *   merge_indptr (out)          : int32 [B + 1] CSR over partial slots
 * b2a_decode_num_ctas returns the persistent grid size the kernel wants on
 * the current device for this head shape (SM count x resident CTAs).
 *
 * b2a_decode runs the plan in ONE launch: the CTA that writes the last
 * partial of a split request (found with a per-request int32 merge counter,
 * an atomic count, never a wait) merges that request's partials.
 * Workspace (b2a_decode_workspace_bytes(n_partials, Hq, D) bytes or more,
 * 256-byte aligned): the merge counters (int32 [n_partials]) sit at its start
 * and the fp32 partial rows at its end. Zero-fill a workspace once when it is
 * allocated; every completed call leaves the counters at zero again, so a
 * buffer can be reused by any number of calls with any n_partials (for one
 * head shape). A segment whose request id is outside [0, B) or whose partial
 * slot is outside its request's merge range (or past n_partials) is skipped
 * and reported as device error 35 (b2a_device_error); such a call can leave
 * counters set, so zero the workspace again before the next call.
 * Launched with programmatic stream serialization: the kernel reads the plan
 * (cta_indptr, segs, merge_indptr) and the page ids before it waits for the
 * previous kernel of the stream, and q, the pools, the workspace and out only
 * after. Write the plan and the page ids with a copy or a kernel ordered
 * before that previous kernel, or with a kernel that does not trigger its
 * dependents early (griddepcontrol.launch_dependents), such as
 * b2a_decode_metadata.
 * ------------------------------------------------------------------------ */
int b2a_decode_plan(const int32_t* kv_indptr, const int32_t* kv_last_page_len, int B,
                    int page_size, int num_ctas, int32_t* cta_indptr, int32_t* segs,
                    int seg_capacity, int32_t* merge_indptr, int* n_segs, int* n_partials);
int b2a_decode_num_ctas(int Hq, int Hkv, int D, int dtype, int* num_ctas);
size_t b2a_decode_workspace_bytes(int n_partials, int Hq, int D);
int b2a_decode(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
               const int32_t* kv_indices, int page_size, const int32_t* cta_indptr, const int32_t* segs, int num_ctas,
               const int32_t* merge_indptr, int n_partials, int B, int Hq, int Hkv, int D,
               float scale, void* workspace, size_t workspace_bytes, void* out, int dtype,
               void* stream);

/* ------------------------------------------------------------------------
 * Decode metadata built on the device (stream-ordered, no host work).
 * Replaces the per-step host build of MetalAttnBackend.prepare_decode
 * (python/minisgl_mlx/attention/metal.py:145-152) together with the page-table
 * row lookup of scheduler/scheduler.py:155-158, and b2a_decode_plan: from a
 * DEVICE copy of the page table and the batch's rows and lengths it writes
 * everything b2a_decode reads, so a decode step, metadata included, can be
 * captured in one CUDA graph.
 *   page_table      : device int32 [table_rows, table_stride], token-granular
 *                     (entry p * page_size of a row = first slot of page p)
 *   rows, lens      : device int32 [B] page-table row and token count
 *   kv_indptr       : out int32 [B + 1]      page CSR
 *   kv_indices      : out int32 [idx_capacity] page ids (slot / page_size)
 *   kv_last_page_len: out int32 [B]
 *   cta_indptr, segs, merge_indptr: out, as from b2a_decode_plan for the same
 *                     CSR and num_ctas (identical values); seg_capacity must
 *                     be >= B + num_ctas (the plan's upper bound), segs
 *                     16-byte aligned
 *   counts          : out int32 [2] = {segments, split partials}; pass
 *                     n_partials = B + num_ctas to b2a_decode with a workspace
 *                     of that capacity (the merge reads merge_indptr on the
 *                     device)
 * num_ctas <= 1024. Lengths above table_stride, rows outside the table and
 * page ids past idx_capacity are skipped and recorded as device error 34
 * (b2a_device_error); negative or unaligned entries as 32.
 *
 * b2a_page_table_scatter writes page_table[rows[i], cols[i]] = values[i] for
 * i < n (device arrays): the slots a step allocates on the host, applied to
 * the device copy. Out-of-range (row, col) pairs are skipped (error 34).
 * ------------------------------------------------------------------------ */
int b2a_decode_metadata(const int32_t* page_table, int64_t table_rows, int64_t table_stride,
                        const int32_t* rows, const int32_t* lens, int B, int page_size, int num_ctas,
                        int32_t* kv_indptr, int32_t* kv_indices, int64_t idx_capacity,
                        int32_t* kv_last_page_len, int32_t* cta_indptr, int32_t* segs, int seg_capacity,
                        int32_t* merge_indptr, int32_t* counts, void* stream);
int b2a_page_table_scatter(int32_t* page_table, int64_t table_rows, int64_t table_stride,
                           const int32_t* rows, const int32_t* cols, const int32_t* values, int64_t n,
                           void* stream);

/* ------------------------------------------------------------------------
 * Paged split-KV decode that allocates nothing and takes no workspace.
 * No counterpart in the reference: it is an extra entry point of this
 * library. It is for callers that cannot allocate device memory when decode
 * runs, for example an engine whose memory planner has given the device to
 * the KV pool, or a host that may only pass buffers it already owns.
 * Same arguments and results as b2a_decode without workspace/workspace_bytes.
 * The split partials and merge counters live in an 8 MiB file-scope device
 * array inside the library, held by every GPU that loads it until the process
 * exits; a plan whose b2a_decode_workspace_bytes(n_partials, Hq, D) exceeds
 * 8 MiB is rejected with B2A_ERR_WORKSPACE. Every call made outside stream
 * capture looks up that array's device address (cudaGetSymbolAddress) with
 * its device current, so a reset device or another current context is
 * followed; a call made during capture reuses the address the last such call
 * found, so make the first call on a device before any stream capture. All
 * calls share the array and it keeps the last call's contents, so calls that
 * overlap on the GPU (other streams, other host threads) race; serialise
 * them. Each call clears the merge counters with a stream-ordered memset
 * before its kernel; the partial rows are written before they are read.
 * ------------------------------------------------------------------------ */
int b2a_decode_noalloc(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
                       const int32_t* kv_indices, int page_size, const int32_t* cta_indptr,
                       const int32_t* segs, int num_ctas, const int32_t* merge_indptr,
                       int n_partials, int B, int Hq, int Hkv, int D, float scale, void* out,
                       int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Ragged causal extend (prefill) attention over a paged prefix.
 * Replaces BaseAttnBackend._prepare_prefill/_forward_prefill
 * (python/minisgl_mlx/attention/base.py:70-105): request r owns query rows
 * [qo_indptr[r], qo_indptr[r+1]) (Lq rows) and Lkv pool tokens described by
 * its pages (the cached prefix followed by the rows just stored). Row i of r
 * attends keys j <= Lkv - Lq + i (bottom-right causal, mx.fast SDPA
 * mask="causal"; for Lq == 1 this is "no mask").
 * b2a_extend_plan (host only) tiles every request into query tiles of
 * b2a_extend_tile_q() rows and orders them longest-first:
 *   work (out) : int32 [work_capacity * 4] = {request, q_tile_begin, q_tile_rows, 0}
 * The kernel is chosen by (dtype, D, Hq/Hkv, page_size): bf16 with D == 128,
 * GQA group 1/2/4/8 and page_size a multiple of 16 runs on tcgen05 tensor
 * cores (TMEM accumulators, TMA-fed tiles, 128/G query tokens per tile);
 * every other supported shape runs a SIMT fp32-accumulating kernel (64/G
 * tokens per tile). `work` must come from b2a_extend_plan with the tile size
 * b2a_extend_tile_q returns for the same arguments; a larger tile is clamped
 * and flagged through the watchdog word.
 * ------------------------------------------------------------------------ */
int b2a_extend_tile_q(int Hq, int Hkv, int D, int dtype, int page_size, int* tile_q);

/* ------------------------------------------------------------------------
 * Extend attention over 16-key groups that start at any slot (pools with
 * page_size < 16, e.g. the reference's default page_size 1).
 * Same attention as b2a_extend (attention/base.py:70-105), with the keys of
 * request b given as groups of 16: group j covers keys [16j, 16j + 16) and
 * its rows are 16 consecutive slots starting at
 *   e = group_starts[group_indptr[b] + j]:
 *   e < num_slots                    -> k_pool / v_pool rows e .. e + 15
 *   num_slots <= e < num_slots + stage_slots
 *                                    -> k_stage / v_stage rows e - num_slots ..
 * Lkv_b = 16 * (groups_b - 1) + kv_last_len[b]; rows of a group past Lkv_b
 * (or past a pool's end) are never attended. A caller reads runs of
 * contiguous slots in place and copies only the other groups to the staging
 * pool (b2a_pack_kv with one 16-row page per group). work comes from
 * b2a_extend_plan(qo_indptr, group_indptr, kv_last_len, B, 16, tile_q, ...).
 * bf16, D 128, GQA group 1/2/4/8 (the tcgen05 kernel) only. A start outside
 * both pools zero-fills its group and records device error 32.
 * ------------------------------------------------------------------------ */
int b2a_extend_groups(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
                      const void* k_stage, const void* v_stage, int64_t stage_slots,
                      const int32_t* qo_indptr, const int32_t* group_indptr, const int32_t* group_starts,
                      const int32_t* kv_last_len, const int32_t* work, int n_work, int T, int B, int Hq,
                      int Hkv, int D, float scale, void* out, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Pack requests' KV rows into pages of 16 contiguous slots (no reference
 * counterpart: it lets b2a_extend run its tcgen05 path for pools whose page
 * size is below 16, e.g. the reference's default page_size 1).
 * For request b < B and position p < tok_indptr[b+1] - tok_indptr[b]:
 *   src = kv_indices[kv_indptr[b] + p / page_size] * page_size + p % page_size
 *   k_out[out_page_indptr[b] * 16 + p] = k_pool[src]   (whole Hkv x D rows, bytes)
 *   v_out[...]                        = v_pool[src]
 * total_tokens = tok_indptr[B]; k_out / v_out hold out_slots rows.
 * Row-list form: tok_indptr, kv_indptr and out_page_indptr NULL, page_size 1:
 *   k_out[g] = k_pool[kv_indices[g]], v_out[g] = v_pool[kv_indices[g]],  g < total_tokens
 * (the groups b2a_extend_groups reads from its staging pool; B is ignored but > 0).
 * A source outside the pool is skipped and recorded as device error 32.
 * ------------------------------------------------------------------------ */
int b2a_pack_kv(const void* k_pool, const void* v_pool, int64_t num_slots, const int32_t* kv_indptr,
                const int32_t* kv_indices, int page_size, const int32_t* tok_indptr,
                const int32_t* out_page_indptr, int B, int64_t total_tokens, int Hkv, int D, int dtype,
                void* k_out, void* v_out, int64_t out_slots, void* stream);
int b2a_extend_plan(const int32_t* qo_indptr, const int32_t* kv_indptr,
                    const int32_t* kv_last_page_len, int B, int page_size, int tile_q,
                    int32_t* work, int work_capacity, int* n_work);
int b2a_extend(const void* q, const void* k_pool, const void* v_pool, int64_t num_slots,
               const int32_t* qo_indptr, const int32_t* kv_indptr, const int32_t* kv_indices,
               const int32_t* kv_last_page_len, int page_size, const int32_t* work, int n_work,
               int T, int B, int Hq, int Hkv, int D, float scale, void* out, int dtype,
               void* stream);

/* ------------------------------------------------------------------------
 * SwiGLU activation of the engine harness's MLP.
 * Replaces `swiglu(gate, up)` (python/minisgl_mlx/models/transformer.py:26-30,
 * fused by mx.compile) called from MLP.__call__ (:67-69). Row r of gate_up
 * holds [gate (F) | up (F)] starting at gate_up + r * row_stride elements;
 *   out[r * F + i] = silu(gate[i]) * up[i]
 * in fp32 with silu(gate) rounded to the storage type before the product, as
 * the unfused `silu(gate) * up` does. F must be even; dtype f32, bf16 or f16.
 * ------------------------------------------------------------------------ */
int b2a_swiglu(const void* gate_up, int64_t row_stride, void* out, int64_t rows, int F, int dtype,
               void* stream);

/* ------------------------------------------------------------------------
 * RMSNorm of hidden rows with an optional row gather (engine harness).
 * Replaces nn.RMSNorm (python/minisgl_mlx/models/transformer.py:77-82, the
 * two norms of every decoder layer) and, with `rows`, the last-token gather
 * plus final norm of CausalLM.__call__ (:109-113) in one launch:
 *   y[i] = x[r] / sqrt(mean(x[r]^2) + eps) * w,  r = rows ? rows[i] : i,
 * in fp32, rounded once to `dtype`. x: x_rows rows of H elements, row i at
 * x + i * x_row_stride; y: contiguous [n_rows, H]; w: [H]. All 16-byte
 * aligned; H a multiple of 32 * (16 / element size), at most 16 vectors per
 * lane. A gather index outside [0, x_rows) skips that row and records device
 * error 32.
 * ------------------------------------------------------------------------ */
int b2a_rmsnorm(const void* x, int64_t x_row_stride, int64_t x_rows, const int32_t* rows, int64_t n_rows,
                const void* w, float eps, int H, void* y, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Decode-batch projection with its neighbours fused (engine harness).
 * Replaces, for a step of at most 64 token rows, the projections of a decoder
 * layer together with the norm in front and the add or activation behind
 * (python/minisgl_mlx/models/transformer.py: qkv_proj / o_proj :41-42,
 * gate_up_proj / down_proj :64-65, DecoderLayer.__call__ :80-82, swiglu
 * :26-30 and :67-69). With W = w [N, K] (row-major, K contiguous) and
 * xn = x when norm_w is NULL, else the RMSNorm of each x row
 * (x / sqrt(mean(x^2) + eps) * norm_w):
 *   mode 0 (plain)     out[M, N]   = xn W^T
 *   mode 1 (residual)  out[M, N]   = res + xn W^T   (out may be res: in place)
 *   mode 2 (swiglu)    out[M, N/2] = silu(g) * u,  [g | u] = xn W^T
 *                      (gate rows 0..N/2-1 of w, up rows N/2..N-1)
 * bf16 only, fp32 accumulation, one rounding to bf16 per stored value (the
 * swiglu form rounds g, u and silu(g) like the unfused 16-bit form; the norm's
 * per-row scale multiplies the fp32 product, so its operand is x * norm_w
 * rounded once). M <= 64; K a positive multiple of 128; N a multiple of 16
 * (32 for swiglu). x, w, norm_w 16-byte aligned, x_row_stride a multiple of 8
 * elements. Launched with programmatic stream serialization: the weight reads
 * start before the previous kernel of the stream has finished.
 * ------------------------------------------------------------------------ */
#define B2A_PROJ_PLAIN 0
#define B2A_PROJ_RESIDUAL 1
#define B2A_PROJ_SWIGLU 2
int b2a_proj(const void* x, int64_t x_row_stride, int M, int K, const void* w, int N, const void* norm_w,
             float eps, const void* res, int64_t res_row_stride, void* out, int64_t out_row_stride, int mode,
             int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200ATTN_H */
