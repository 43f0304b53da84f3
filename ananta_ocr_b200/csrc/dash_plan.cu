// dash_plan.cu -- per-step serving plans computed on the device: which pages
// of each request's block table need their k-bar summary refreshed (and how
// many live tokens each holds), and the request that owns every query row.
//
// One CTA per request; its threads write the request's plan entries and its
// rows of the row -> request map.  Everything stays on the device: the sizes
// (entries per request, total rows) come from the caller, so no host sync.
//
// Semantics: WHL route_triton.py:576-601 (kbar_all_plan), :605-620
// (prefill_row2req), :682-703 (kbar_tail_plan).
#include "dash_internal.h"

namespace dash {

constexpr int kPlanThreads = 128;

__global__ void __launch_bounds__(kPlanThreads) serving_plan_kernel(const DashServingPlanArgs a) {
  const int r = blockIdx.x;
  const int bs = a.block_size;
  const int sl = a.seq_lens[r];
  if (a.pages) {
    const int32_t* bt_row = a.block_table + (int64_t)r * a.bt_stride;
    // last block holding a token of the request (block 0 for an empty one)
    const int last = sl > 0 ? (sl - 1) / bs : 0;
    const int first = a.mode == 0 ? a.context_lens[r] / bs : 0;
    for (int j = threadIdx.x; j < a.width; j += kPlanThreads) {
      // mode 0: the blocks a prefill chunk wrote, from the one holding the
      // first new token on; mode 1: the tail blocks, newest first
      const int b = a.mode == 0 ? first + j : max(last - j, 0);
      const int col = min(b, a.bt_width - 1);
      const int live = min(max(sl - b * bs, 0), bs);
      const int64_t e = (int64_t)r * a.width + j;
      a.pages[e] = (int64_t)bt_row[col];
      a.ntok[e] = live;
    }
  }
  if (a.row2req) {
    const int r0 = a.cu_seqlens_q[r], r1 = a.cu_seqlens_q[r + 1];
    for (int i = r0 + threadIdx.x; i < r1; i += kPlanThreads) a.row2req[i] = r;
  }
}

int launch_serving_plan(const DashServingPlanArgs& a, cudaStream_t st) {
  if (a.n_req == 0) return DASH_OK;
  serving_plan_kernel<<<a.n_req, kPlanThreads, 0, st>>>(a);
  count_launch();
  return check_launch("serving_plan_kernel");
}

}  // namespace dash
