// Ragged causal extend attention on tcgen05 tensor cores (bf16, head_dim 128).
#pragma once
#include <string>

#include "common.cuh"

namespace b2a {

constexpr int kTcRows = 128;  // query rows (tokens x GQA heads) per CTA tile

inline bool extend_tc_supported(int Hq, int Hkv, int D, int dtype) {
  (void)Hq;
  (void)Hkv;
  (void)D;
  (void)dtype;
  return false;
}

inline int extend_tc_launch(const void*, const void*, const void*, int64_t, const int32_t*, const int32_t*,
                            const int32_t*, const int32_t*, int, const int32_t*, int, int, int, int, float, void*,
                            cudaStream_t, std::string& err) {
  err = "tcgen05 extend kernel not built";
  return 2;
}

}  // namespace b2a
