// dash_internal.h -- host-side glue shared by the translation units of
// libdash_b200.so (error reporting, launch accounting, kernel launchers).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include "../../include/dash_b200.h"

namespace dash {

int set_error(int code, const char* fmt, ...);   // stores the message, returns code
int check_launch(const char* kernel);            // cudaGetLastError -> status
void count_launch();

int launch_kbar(const DashKbarArgs& a, cudaStream_t st);
int launch_route(const DashRouteArgs& a, int64_t n_rows, cudaStream_t st);
// the routing with a paged k-bar refresh folded into the decode launch where it can be
int launch_route_refresh(const DashRouteArgs& a, int64_t n_rows, const DashKbarArgs& ka, cudaStream_t st);
int launch_block_max(const DashBlockMaxArgs& a, cudaStream_t st);
int launch_decode(const DashDecodeArgs& a, int64_t n_rows, int splits, cudaStream_t st);
int launch_prefill(const DashPrefillArgs& a, int64_t n_rows, cudaStream_t st);
size_t prefill_workspace(const DashPrefillArgs& a, int64_t n_rows);
// the routed part gathered by key block is implemented for these arguments
bool prefill_gathered_supported(const DashPrefillArgs& a);
size_t decode_workspace(const DashDecodeArgs& a, int64_t n_rows, int splits);
int decode_auto_splits(const DashDecodeArgs& a, int64_t n_rows);
// paged bf16/fp16 caches with 128-dim heads: K/V streamed by TMA (dash_decode_tma.cu)
bool decode_tma_supported(const DashDecodeArgs& a);
int decode_tma_slots();
int launch_decode_tma(const DashDecodeArgs& a, int64_t n_rows, int splits, float* part, int* counters,
                      cudaStream_t st);
int validate_decode(const DashDecodeArgs* a, int* splits);   // DASH_OK or a status with message
int launch_page_ids(const DashPageIdsArgs& a, cudaStream_t st);
int launch_page_state(const DashPageStateArgs& a, cudaStream_t st);
int launch_page_allow(const DashPageAllowArgs& a, cudaStream_t st);
int launch_page_decode(const DashPageDecodeArgs& a, cudaStream_t st);
int launch_block_any(const DashBlockAnyArgs& a, cudaStream_t st);
int launch_page_blocks(const DashPageBlocksArgs& a, cudaStream_t st);
int launch_index_proj(const DashIndexProjArgs& a, cudaStream_t st);
int launch_rope_kv(const DashRopeKVArgs& a, cudaStream_t st);
int launch_attn_bwd(const DashAttnBwdArgs& a, cudaStream_t st);
size_t attn_bwd_flag_words(const DashAttnBwdArgs& a);
size_t attn_bwd_tc_acc_bytes(const DashAttnBwdArgs& a);
int launch_attn_bwd_tc(const DashAttnBwdArgs& a, int nblk, int words, cudaStream_t st);
int launch_entmax15(const DashEntmaxArgs& a, bool backward, cudaStream_t st);
int launch_serving_plan(const DashServingPlanArgs& a, cudaStream_t st);
int launch_page_coords(const DashPageCoordArgs& a, cudaStream_t st);
int launch_cos_sin_2d(const DashCosSin2DArgs& a, cudaStream_t st);

}  // namespace dash
