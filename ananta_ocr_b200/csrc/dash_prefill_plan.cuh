// dash_prefill_plan.cuh -- what plan_kernel leaves for the prefill attention
// kernels (the tcgen05 bf16/fp16 kernel and the fp32 CUDA-core kernel), and
// the sequence-layout helpers they share.
#pragma once
#include <cstdint>
#include <cudaTypedefs.h>
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
  // gathered mode: per (index head, sequence, block) bitmask of the query
  // tokens whose canonical list holds the block, [nih][n_seq][nblk_cap][wps]
  // (bit i of word w: token 32w + i of the sequence); NULL in union mode
  uint32_t* flags;
  int32_t wps;             // words per (sequence, block)
  int32_t wpt;             // words per query tile (TT / 32)
  // Work chunk of the launch: sequences [s0, s0 + sn), query tile pairs
  // [pj0, pj0 + npj) of each (pair j: tiles 2j, 2j+1, tokens [2j TT,
  // 2(j+1) TT)), kv heads [hk0, hk0 + grid.y).  Union mode: everything.
  int32_t s0, sn, pj0, npj;
  int32_t hk0;
  // gathered mode: the partials of this chunk, query heads [hq0, hq0 + hqn);
  // entry (((s - s0) * prows + i - 2 pj0 TT) * hqn + hq - hq0) * (K + 1) + j
  // for token i: list slot j < K (the routed block's keys, no bias) or the
  // window part (j = K); the normalised output (bf16/fp16 bits, [.][128]) and
  // its log2-sum-exp, combined by the merge kernel
  int32_t hq0, hqn;
  int32_t prows;           // partial rows per sequence (= 2 npj TT)
  const uint16_t* part_o;
  const float* part_lse;
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
// Launches the routed (gathered) kernel over the plan's chunk (hcn kv heads
// from p.hk0): K/V tensor maps with boxes of min(block_size, 64) rows.
int launch_prefill_routed(const DashPrefillArgs& c, const PrefillPlan& p, const CUtensorMap& mk,
                          const CUtensorMap& mv, int hcn, cudaStream_t st);
// Launches the merge of the chunk's partials into the output (and the peer
// copies, lse).
int launch_prefill_merge(const DashPrefillArgs& c, const PrefillPlan& p, cudaStream_t st);

// Routed slots per row (K) the plan and the gathered kernels take.
constexpr int kPlanMaxSlots = 256;

}  // namespace dash
