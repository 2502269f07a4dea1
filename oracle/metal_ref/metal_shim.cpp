// Runs the reference's own Metal paged-decode kernel body on the CPU.
// TEST INFRASTRUCTURE ONLY: it pins the oracle (and the golden vectors) to the
// reference's kernel code; the product never links it.
//
// The kernel body is NOT in this repository. oracle/metal_ref/build.py reads it
// from the reference (the _PAGED_DECODE_SOURCE string of
// python/minisgl_mlx/attention/metal.py:35-95) into oracle/_ref/ and compiles
// this file with it. The body is written per thread with Metal's SIMT
// builtins; here every thread of a threadgroup is a cooperative fiber
// (ucontext) and the builtins are rendezvous points:
//   simd_sum(x)            all 32 lanes of the simdgroup deposit, the last one
//                          adds them in lane order, everyone gets the sum
//   threadgroup_barrier()  all threads of the threadgroup arrive
//   threadgroup T a[...]   one array shared by the threadgroup (a function
//                          static; threadgroups run one after another)
//   fast::exp              std::exp (float)
// The grid is (NSG*32, Hkv, B) with one threadgroup per (request, kv head),
// NSG = 32 if D <= 128 else 16, exactly as paged_decode_attention launches it
// (metal.py:123-130).
#include <ucontext.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace metal_emul {

using uint = unsigned int;
struct uint3 {
  uint x, y, z;
};
enum class mem_flags { mem_threadgroup };

// bfloat16 storage with round-to-nearest-even conversion from float.
struct bfloat16_t {
  uint16_t bits;
  bfloat16_t() = default;
  bfloat16_t(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
      bits = (uint16_t)((u >> 16) | 0x40);
    } else {
      const uint32_t lsb = (u >> 16) & 1u;
      bits = (uint16_t)((u + 0x7fffu + lsb) >> 16);
    }
  }
  operator float() const {
    uint32_t u = (uint32_t)bits << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  }
};

namespace fast {
inline float exp(float x) { return std::exp(x); }
}  // namespace fast
using std::max;

// ---------------------------------------------------------------- fibers
struct Sched {
  int nthreads = 0;
  int current = 0;
  ucontext_t main_ctx;
  std::vector<ucontext_t> ctx;
  std::vector<std::vector<char>> stacks;
  std::vector<int> done;
  std::vector<float> simd_vals, simd_result;
  std::vector<int> simd_count, simd_gen;
  int bar_count = 0, bar_gen = 0;
};
static Sched* S = nullptr;

static void yield_now() { swapcontext(&S->ctx[S->current], &S->main_ctx); }

inline float simd_sum(float v) {
  const int t = S->current;
  const int sg = t / 32;
  S->simd_vals[t] = v;
  const int gen = S->simd_gen[sg];
  if (++S->simd_count[sg] == 32) {
    float s = 0.f;
    for (int i = 0; i < 32; ++i) s += S->simd_vals[sg * 32 + i];
    S->simd_result[sg] = s;
    S->simd_count[sg] = 0;
    S->simd_gen[sg]++;
  } else {
    while (S->simd_gen[sg] == gen) yield_now();
  }
  return S->simd_result[sg];
}

inline void threadgroup_barrier(mem_flags) {
  const int gen = S->bar_gen;
  if (++S->bar_count == S->nthreads) {
    S->bar_count = 0;
    S->bar_gen++;
  } else {
    while (S->bar_gen == gen) yield_now();
  }
}

// ---------------------------------------------------------------- the kernel
template <typename T, int G, int D, int NSG>
struct Kernel {
  struct Args {
    const T* q;
    const T* k_pool;
    const T* v_pool;
    const int32_t* kv_indptr;
    const int32_t* kv_indices;
    const float* scale;
    T* out;
    int q_shape[3];
    int k_pool_shape[3];
    uint3 tg;
  };
  static Args* A;

  static void body(const T* q, const T* k_pool, const T* v_pool, const int32_t* kv_indptr,
                   const int32_t* kv_indices, const float* scale, T* out, const int* q_shape,
                   const int* k_pool_shape, uint3 threadgroup_position_in_grid, uint simdgroup_index_in_threadgroup,
                   uint thread_index_in_simdgroup, uint thread_index_in_threadgroup) {
#define device
#define threadgroup static
#include "paged_decode_body.inc"
#undef threadgroup
#undef device
  }

  static void entry(int tid) {
    body(A->q, A->k_pool, A->v_pool, A->kv_indptr, A->kv_indices, A->scale, A->out, A->q_shape, A->k_pool_shape,
         A->tg, (uint)(tid / 32), (uint)(tid % 32), (uint)tid);
    S->done[tid] = 1;
  }

  static void run(const T* q, const T* k, const T* v, const int32_t* indptr, const int32_t* indices, float scale,
                  int B, int Hq, int Hkv, int N, T* out) {
    Args a;
    a.q = q;
    a.k_pool = k;
    a.v_pool = v;
    a.kv_indptr = indptr;
    a.kv_indices = indices;
    a.scale = &scale;
    a.out = out;
    a.q_shape[0] = B;
    a.q_shape[1] = Hq;
    a.q_shape[2] = D;
    a.k_pool_shape[0] = N;
    a.k_pool_shape[1] = Hkv;
    a.k_pool_shape[2] = D;
    A = &a;
    Sched sched;
    S = &sched;
    const int nt = NSG * 32;
    sched.nthreads = nt;
    sched.ctx.resize(nt);
    sched.stacks.assign(nt, std::vector<char>(64 * 1024));
    sched.done.assign(nt, 0);
    sched.simd_vals.assign(nt, 0.f);
    sched.simd_result.assign(NSG, 0.f);
    sched.simd_count.assign(NSG, 0);
    sched.simd_gen.assign(NSG, 0);
    for (int b = 0; b < B; ++b) {
      for (int kvh = 0; kvh < Hkv; ++kvh) {
        a.tg = uint3{0u, (uint)kvh, (uint)b};
        std::fill(sched.done.begin(), sched.done.end(), 0);
        sched.bar_count = 0;
        for (int t = 0; t < nt; ++t) {
          getcontext(&sched.ctx[t]);
          sched.ctx[t].uc_stack.ss_sp = sched.stacks[t].data();
          sched.ctx[t].uc_stack.ss_size = sched.stacks[t].size();
          sched.ctx[t].uc_link = &sched.main_ctx;
          makecontext(&sched.ctx[t], (void (*)())entry, 1, t);
        }
        int alive = nt;
        while (alive > 0) {
          alive = 0;
          for (int t = 0; t < nt; ++t) {
            if (sched.done[t]) continue;
            sched.current = t;
            swapcontext(&sched.main_ctx, &sched.ctx[t]);
            if (!sched.done[t]) ++alive;
          }
        }
      }
    }
    S = nullptr;
  }
};
template <typename T, int G, int D, int NSG>
typename Kernel<T, G, D, NSG>::Args* Kernel<T, G, D, NSG>::A = nullptr;

template <typename T, int G, int D>
int run_d(const void* q, const void* k, const void* v, const int32_t* indptr, const int32_t* indices, float scale,
          int B, int Hq, int Hkv, int N, void* out) {
  constexpr int NSG = D <= 128 ? 32 : 16;  // metal.py:123
  Kernel<T, G, D, NSG>::run((const T*)q, (const T*)k, (const T*)v, indptr, indices, scale, B, Hq, Hkv, N, (T*)out);
  return 0;
}

template <typename T, int G>
int run_g(int D, const void* q, const void* k, const void* v, const int32_t* indptr, const int32_t* indices,
          float scale, int B, int Hq, int Hkv, int N, void* out) {
  switch (D) {
    case 64:
      return run_d<T, G, 64>(q, k, v, indptr, indices, scale, B, Hq, Hkv, N, out);
    case 128:
      return run_d<T, G, 128>(q, k, v, indptr, indices, scale, B, Hq, Hkv, N, out);
    case 256:
      return run_d<T, G, 256>(q, k, v, indptr, indices, scale, B, Hq, Hkv, N, out);
  }
  return 2;
}

template <typename T>
int run_t(int G, int D, const void* q, const void* k, const void* v, const int32_t* indptr,
          const int32_t* indices, float scale, int B, int Hq, int Hkv, int N, void* out) {
  switch (G) {
    case 1:
      return run_g<T, 1>(D, q, k, v, indptr, indices, scale, B, Hq, Hkv, N, out);
    case 2:
      return run_g<T, 2>(D, q, k, v, indptr, indices, scale, B, Hq, Hkv, N, out);
    case 4:
      return run_g<T, 4>(D, q, k, v, indptr, indices, scale, B, Hq, Hkv, N, out);
    case 8:
      return run_g<T, 8>(D, q, k, v, indptr, indices, scale, B, Hq, Hkv, N, out);
  }
  return 2;
}

}  // namespace metal_emul

// dtype 0 = float32, 1 = bfloat16 (uint16 storage). Returns 0 on success.
extern "C" int metal_ref_paged_decode(const void* q, const void* k_pool, const void* v_pool, const int32_t* kv_indptr,
                                      const int32_t* kv_indices, float scale, int B, int Hq, int Hkv, int N, int D,
                                      int dtype, void* out) {
  if (Hkv <= 0 || Hq % Hkv != 0 || D % 32 != 0) return 1;  // the assert of metal.py:122
  const int G = Hq / Hkv;
  if (dtype == 0) return metal_emul::run_t<float>(G, D, q, k_pool, v_pool, kv_indptr, kv_indices, scale, B, Hq, Hkv, N, out);
  if (dtype == 1)
    return metal_emul::run_t<metal_emul::bfloat16_t>(G, D, q, k_pool, v_pool, kv_indptr, kv_indices, scale, B, Hq, Hkv,
                                                     N, out);
  return 2;
}
