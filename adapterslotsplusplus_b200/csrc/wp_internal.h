// wp_internal.h -- structures shared by the host side of libwp_b200.so and
// its kernels. Not part of the public C ABI (include/wp_api.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wp {

// Largest token count of one compute segment. Runs of equal adapter ids are
// split into pieces of at most this many tokens, exactly as the reference's
// build_seg_bounds_kernel does (WP_MAX_SEGMENT_TOKENS,
// csrc/bridge/warp_pipe_metadata.h:22, split at csrc/kernels/warp_pipe_r32.cu:498-511).
constexpr int kSegTokens = 32;

// One entry of a device segment table (32 bytes).
//   live table (build_seg_bounds): adapter_id/token_start/token_count only; the
//     apply kernels resolve weights as base + adapter_id * stride.
//   registry table (build_segments): a/b/alpha carry the resolved weight
//     pointers (original tensors or a staging slot) and the adapter's scale.
struct DevSeg {
  int32_t adapter_id;
  int32_t token_start;
  int32_t token_count;
  float alpha;
  const void* a;
  const void* b;
};
static_assert(sizeof(DevSeg) == 32, "DevSeg is 32 bytes");

struct ShrinkArgs {
  const void* x;  // [T, d] rows of x_ld elements
  int64_t x_ld;
  float* h;  // [T, R] fp32 output (ld = R)
  float* partial;  // [nsplit][cap_t][R] split-K partials
  uint32_t* counters;  // per-segment arrival counters (zero between calls)
  const DevSeg* segs;
  const int* num_segs;
  const void* wa_base;  // live mode: A_i = wa_base + i * wa_stride
  int64_t wa_stride;
  float scale;
  int registry;  // 1: weights and alpha from the table entries
  int d;
  int nsplit;
  int split_len;  // elements of d per split (multiple of 8)
  int cap_t;  // row capacity of one partial plane
  int* err;
};

struct ExpandArgs {
  const float* h;  // [T, R] fp32
  void* y;  // [T, y_ld]; columns y_off .. y_off+o are updated
  int64_t y_ld;
  int y_off;
  const DevSeg* segs;
  const int* num_segs;
  const void* wb_base;  // live mode: B_i = wb_base + i * wb_stride
  int64_t wb_stride;
  int registry;
  int o;
  int n_ochunks;
  int y_bulk;  // 1: y rows can be bulk-copied (16-byte aligned rows and offset)
  int* err;
};

struct LaunchCfg {
  int grid;
  cudaStream_t stream;
  bool pdl;
};

// dtype: 0 = f16, 1 = bf16 (WP_DTYPE_*). Return a cudaError_t.
cudaError_t launch_shrink(int dtype, int rank, const ShrinkArgs& a, const LaunchCfg& lc);
cudaError_t launch_expand(int dtype, int rank, const ExpandArgs& a, const LaunchCfg& lc);
// Column chunk width of one expand work item.
int expand_chunk_cols(int rank);
// K elements per pipeline stage of the shrink kernel.
int shrink_chunk_k(int rank);

// idx_dtype: WP_DTYPE_I32 or WP_DTYPE_I64.
cudaError_t launch_seg_bounds(const void* idx, int idx_dtype, int T, DevSeg* segs, int* num_segs,
                              int* run_starts, cudaStream_t stream);

}  // namespace wp
