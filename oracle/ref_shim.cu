// ref_shim.cu -- TEST INFRASTRUCTURE ONLY (oracle). A C ABI over the
// reference's own, unmodified CUDA kernels (csrc/kernels/warp_pipe_r32.cu,
// warp_pipe_r{8,16,64}.cu of vac014/AdapterSlotsPlusPlus), compiled from the
// reference checkout by oracle/build_ref.sh into oracle/_ref/libwpref.so.
//
// It exists so that GPU tests can compare libwp_b200.so with the reference
// itself on the same inputs:
//   ref_seg_bounds    -> launch_build_seg_bounds_r32 (warp_pipe_r32.cu:612-619),
//                        then reads the segment table back (the reference's
//                        binding has no readback);
//   ref_add_lora_r32  -> launch_bgmv_shrink_dsak_r32 + launch_bgmv_expand_dsak_r32
//                        (warp_pipe_r32.cu:621-637) on the table built above,
//                        as WarpPipeExtension::add_lora_packed does
//                        (warp_pipe_bindings.cpp:195-234);
//   ref_registry_apply-> launch_bgmv_shrink_r{8,16,32,64} / expand
//                        (the registry path, warp_pipe_dispatcher.cpp:33-53)
//                        on a table filled like build_segment_table
//                        (segment_builder.cpp:5-50).
// The reference's limits apply: fp16, T <= 256, segments <= 32 tokens,
// d_model and out_features multiples of 256, live path rank 32.
// Nothing in the product links or loads this library.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "warp_pipe_r16.h"
#include "warp_pipe_r32.h"
#include "warp_pipe_r64.h"
#include "warp_pipe_r8.h"

namespace {
WarpPipeMetadata* g_meta = nullptr;  // device copy of the reference's metadata
half* g_h = nullptr;  // [256, 32] fp16 H buffer of the live path

int ensure() {
  if (!g_meta && cudaMalloc(&g_meta, sizeof(WarpPipeMetadata)) != cudaSuccess) return -2;
  if (!g_h && cudaMalloc(&g_h, sizeof(half) * WP_MAX_SEGMENTS * 64) != cudaSuccess) return -2;
  return 0;
}
}  // namespace

extern "C" {

int ref_max_tokens(void) { return WP_MAX_SEGMENTS; }

// d_idx: device int64[T]. out: host int32[3 * WP_MAX_SEGMENTS] triples.
int ref_seg_bounds(const int64_t* d_idx, int T, int32_t* out, int32_t* num) {
  if (T > WP_MAX_SEGMENTS) return 1;  // the reference returns False here
  if (ensure()) return -2;
  cudaMemset(g_meta, 0, sizeof(WarpPipeMetadata));
  launch_build_seg_bounds_r32(d_idx, T, g_meta, 0);
  if (cudaDeviceSynchronize() != cudaSuccess) return -2;
  static WarpPipeMetadata host;
  if (cudaMemcpy(&host, g_meta, sizeof(host), cudaMemcpyDeviceToHost) != cudaSuccess) return -2;
  *num = static_cast<int32_t>(host.num_segments);
  for (uint32_t i = 0; i < host.num_segments && i < WP_MAX_SEGMENTS; ++i) {
    out[3 * i + 0] = host.segments[i].adapter_id;
    out[3 * i + 1] = host.segments[i].token_start;
    out[3 * i + 2] = host.segments[i].token_count;
  }
  return 0;
}

// Live path on the table of the last ref_seg_bounds call (rank 32, fp16).
int ref_add_lora_r32(half* y, const half* x, const half* wa, int64_t wa_stride0, const half* wb, int64_t wb_stride0,
                     float scale, int d_model, int out_features, void* stream) {
  if (ensure()) return -2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  launch_bgmv_shrink_dsak_r32(x, g_h, g_meta, wa, wa_stride0, scale, d_model, s);
  launch_bgmv_expand_dsak_r32(g_h, y, g_meta, wb, wb_stride0, out_features, s);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Registry path: K segments given as host arrays of device pointers.
int ref_registry_apply(int rank, const half* X, half* H, half* Y, const uint64_t* a_ptrs, const uint64_t* b_ptrs,
                       const int32_t* starts, const int32_t* counts, const float* alphas, int K, int d_model,
                       int out_features, void* stream) {
  if (K > WP_MAX_SEGMENTS) return 1;
  if (ensure()) return -2;
  static WarpPipeMetadata host;
  memset(&host, 0, sizeof(host));
  for (int i = 0; i < K; ++i) {
    SegmentDescriptor& sd = host.segments[i];
    sd.adapter_id = i;
    sd.token_start = starts[i];
    sd.token_count = counts[i];
    sd.rank = rank;
    sd.d_model = d_model;
    sd.out_features = out_features;
    sd.alpha_scale = alphas[i];
    sd.A_ptr = static_cast<uintptr_t>(a_ptrs[i]);
    sd.B_ptr = static_cast<uintptr_t>(b_ptrs[i]);
  }
  host.num_segments = static_cast<uint32_t>(K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(g_meta, &host, sizeof(host), cudaMemcpyHostToDevice, s) != cudaSuccess) return -2;
  switch (rank) {
    case 8: launch_bgmv_shrink_r8(X, H, g_meta, d_model, s); launch_bgmv_expand_r8(H, Y, g_meta, out_features, s); break;
    case 16: launch_bgmv_shrink_r16(X, H, g_meta, d_model, s); launch_bgmv_expand_r16(H, Y, g_meta, out_features, s); break;
    case 32: launch_bgmv_shrink_r32(X, H, g_meta, d_model, s); launch_bgmv_expand_r32(H, Y, g_meta, out_features, s); break;
    case 64: launch_bgmv_shrink_r64(X, H, g_meta, d_model, s); launch_bgmv_expand_r64(H, Y, g_meta, out_features, s); break;
    default: return -1;
  }
  if (cudaStreamSynchronize(s) != cudaSuccess) return -2;
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // extern "C"
