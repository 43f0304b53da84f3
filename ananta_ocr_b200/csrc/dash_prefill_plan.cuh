// dash_prefill_plan.cuh -- what plan_kernel leaves for the prefill attention
// kernels (the tcgen05 bf16/fp16 kernel and the fp32 CUDA-core kernel), and
// the sequence-layout helpers they share.
#pragma once
#include <cstdint>
#include "../../include/dash_b200.h"

namespace dash {

struct PrefillPlan {
  const int32_t* cidx;     // canonical lists [nih][n_rows][K]
  const float* cbias;
  const uint32_t* tmask;   // per-tile unions [nih][n_tiles][nwords]
  const float* rowmax;     // largest kept bias per row [nih][n_rows] (-inf: none)
  int64_t n_rows;
  int32_t nwords;
  int32_t tiles_per_seq;
  int32_t G;               // query heads per kv head
  int32_t TT;              // tokens per tile (= 128 / G)
  int32_t paged;
  int32_t nblk_cap;
};

__device__ __forceinline__ int kv_len_of(const DashSeqs& q, int s) {
  return q.kv_len ? q.kv_len[s] : q.kv_len_fixed;
}
__device__ __forceinline__ int q_len_of(const DashSeqs& q, int s) {
  return q.q_start ? q.q_start[s + 1] - q.q_start[s] : q.q_len_fixed;
}
__device__ __forceinline__ int pos0_of(const DashSeqs& q, int s) {
  return q.pos0 ? q.pos0[s] : kv_len_of(q, s) - q_len_of(q, s);
}
__device__ __forceinline__ int64_t row_base(const DashSeqs& q, int s) {
  return q.q_start ? (int64_t)q.q_start[s] : (int64_t)s * q.q_len_fixed;
}

// Launches the fp32 CUDA-core kernel over plan_kernel's canonical lists.
int launch_prefill_f32(const DashPrefillArgs& a, const PrefillPlan& p, cudaStream_t st);

}  // namespace dash
