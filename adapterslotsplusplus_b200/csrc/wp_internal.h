// wp_internal.h -- structures shared by the host side of libwp_b200.so and
// its kernels. Not part of the public C ABI (include/wp_api.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wp {

// Largest token count of one compute segment. Runs of equal adapter ids are
// split into pieces of at most this many tokens, exactly as the reference's
// build_seg_bounds_kernel does (WP_MAX_SEGMENT_TOKENS,
// csrc/bridge/warp_pipe_metadata.h:22, split at csrc/kernels/warp_pipe_r32.cu:498-511).
constexpr int kSegTokens = 32;
// Prefill tiles (tokens per tcgen05 tile, M of the MMAs) and the shortest run
// the segmenter's prefill mode sends to the prefill kernels.
constexpr int kPrefillTile = 128;
constexpr int kPrefillMinRun = 128;

// One entry of a device segment table (32 bytes).
//   live table (build_seg_bounds): adapter_id/token_start/token_count only; the
//     apply kernel resolves weights as base + adapter_id * stride.
//   registry table (build_segments): `a` is the device address of a TMA
//     descriptor of the adapter's A [r, d]; `b` is, for r >= 16, the address
//     of a TMA descriptor of its B [o, r] and, for r = 8, B's address
//     (original tensor or staging slot); alpha is the adapter's scale.
struct DevSeg {
  int32_t adapter_id;
  int32_t token_start;
  int32_t token_count;
  float alpha;
  const void* a;
  const void* b;
};
static_assert(sizeof(DevSeg) == 32, "DevSeg is 32 bytes");

// Columns of one TMA box (128 bytes of 16-bit elements).
constexpr int kBoxCols = 64;
// K elements per shrink stage and output columns per expand stage (4 boxes).
constexpr int kStageK = 256;
constexpr int kStageCols = 256;

// Per-cluster work assignment of the clustered apply kernel, computed once
// per step by the segmenter for one cluster count G: segments ordered by
// decreasing token count; mode 1 (fewer segments than clusters) gives the
// largest segments (at most kPlanMaxHelpers) a helper cluster that takes half
// of their output columns, the helper pairs on the lowest clusters; mode 2
// (up to kPlanMaxSegs segments) deals them in snake order; mode 0: no plan
// (the kernel deals round robin). Slot r * G + c holds round r of
// cluster c.
constexpr int kPlanRounds = 4;
constexpr int kPlanMaxClusters = 160;
constexpr int kPlanMaxSegs = 128;
// Helper pairs per plan. The helper pairs hold the largest segments and go
// first (the hardware dispatches low clusters first); measured on the
// config-1 step at 8 / 32 / 64 / 128 resident adapters, 8 pairs first beat
// every pair the free clusters allow placed after the whole segments
// (1.43 / 1.83 / 2.13 / 2.63 ms against 1.46 / 1.86 / 2.17 / 2.81 ms):
// more pairs first push the 16-stage whole segments to the clusters that
// start last, fewer leave the largest segments whole.
constexpr int kPlanMaxHelpers = 8;
struct ClusterPlan {
  int4 hdr;  // x: mode, y: segments, z: G, w: helper count (mode 1)
  int count[kPlanMaxClusters];  // segments of cluster c
  int half[kPlanMaxClusters];  // mode 1: -1 whole segment, 0 / 1 first / second half of the output columns
  DevSeg seg[kPlanRounds * kPlanMaxClusters];
};

// Slices of one multi-slice call (q, k, v of a fused qkv projection).
constexpr int kMaxSlices = 3;
constexpr int kMaxTp = 8;  // tensor-parallel ranks of the peer-memory exchange
constexpr int kMaxRank = 64;  // largest LoRA rank

// Which halves of the apply one launch runs.
enum : int { kModeShrink = 1, kModeExpand = 2, kModeFused = 3 };

// Arguments of one apply launch. Tensor maps (TMA descriptors, 64-byte
// aligned) come first; index i of tmap_x / tmap_y is the map whose box is
// (8 << i) rows high (8, 16, 32), so a segment loads only the rows it needs.
struct ApplyArgs {
  // x / y / A maps are "sliced" when d (x, A) or o (y) is a multiple of 64:
  // the row is viewed as [d / 64 slices][64 columns] and one box brings the 4
  // slices of a stage ([4][rows][64] in shared memory, 128B swizzle) in a
  // single instruction; otherwise they are plain maps loaded 64 columns at a
  // time into the same layout.
  CUtensorMap tmap_x[3];  // x [T, d], 8 << i rows per box
  CUtensorMap tmap_y[3];  // y columns [y_off, y_off + o) x T rows, 8 << i rows per box
  CUtensorMap tmap_a;  // live mode: A stack [L, r, d]
  CUtensorMap tmap_b;  // live mode, r >= 16: B stack [L, o, r], box r x 256 x 1, swizzle = 2r bytes
  CUtensorMap tmap_x128;  // prefill kernels: x [T, d] in 128-row boxes (sliced, {64, 128, 4})
  CUtensorMap tmap_y128;  // prefill kernels: y columns [y_off, y_off + o), boxes of 128 rows x 64 columns
  CUtensorMap tmap_b64;  // prefill kernels: B stack [L, o, r], box r x 64 x 1
  // multi-slice calls (nslices > 1, clustered kernel, live mode): slices 1
  // and 2 share x and the table; their A / B stacks and y column ranges
  CUtensorMap tmap_a_x[kMaxSlices - 1];
  CUtensorMap tmap_b_x[kMaxSlices - 1];
  CUtensorMap tmap_y_x[kMaxSlices - 1][3];
  const DevSeg* segs;
  const int* num_segs;
  float* h;  // shrink-only: H [T, r] fp32 written; expand-only: read
  void* y;  // [T, y_ld]; columns y_off .. y_off+o are updated
  int64_t y_ld;
  int y_off;
  const void* wb_base;  // live mode: B_i = wb_base + i * wb_stride ([o, r] row-major)
  int64_t wb_stride;
  float scale;  // live mode alpha
  int mode;  // kModeShrink | kModeExpand
  int registry;  // 1: A through DevSeg.a, B from DevSeg.b, alpha from DevSeg.alpha
  int d;
  int o;
  int split_len;  // d elements per cluster rank (multiple of kStageK)
  int oslice;  // o columns per cluster rank (multiple of kStageCols)
  int y_tma;  // 1: tmap_y is valid; else y is read and written directly
  int d_sliced;  // tmap_x and the A maps are sliced (d % 64 == 0)
  int o_sliced;  // tmap_y is sliced (o % 64 == 0)
  int prefetch_weights;  // 1: table and weight loads may start before the dependency wait
  int prefetch_inputs;  // 1 (fused live calls): x loads and the shrink may also run before it
  int pf_late_wait;  // prefill shrink: the previous kernel is this call's decode kernel (disjoint rows): wait for it only before exiting
  int* err;
  unsigned long long* trace;  // optional per-CTA phase timestamps (kTraceSlots per CTA), else null
  // split (balanced decode) kernel only
  float* part;  // shrink partials [T, pmax, r] fp32
  float* hsplit;  // H [T, r] fp32 (alpha applied)
  int* sync;  // per-segment counters: H readers done [cap]; zero between launches
  int* rflag;  // per shrink item: 1 once the run starting at that item published its partial; zero between launches
  int pmax;  // partial slots per token (>= d / 256 rounded up)
  int nslices;  // 1, or up to kMaxSlices slices sharing x (virtual segment v = slice * segments + segment)
  int y_off_x[kMaxSlices - 1];  // y column offset of slices 1, 2
  const void* wb_base_x[kMaxSlices - 1];  // rank-8 bulk B of slices 1, 2
  int64_t wb_stride_x[kMaxSlices - 1];
  const ClusterPlan* plan;  // clustered kernel: the segmenter's assignment for this table, or null
  int sync_cap;  // segments the counters cover
  // Row-parallel tensor parallelism over peer memory (clustered decode
  // kernel, tp_world > 1): after its cluster exchange, a segment's partial H
  // (this rank's slice of d) goes into every peer's mailbox, and the full H is
  // the sum of all ranks' partials in rank order. Mailbox of rank q (mapped
  // in this process at tp_mail[q]): TpMail::data / flag below.
  float* tp_mail[kMaxTp];
  int* tp_seq;  // [2] on this rank: launch epoch of the exchange, CTAs finished in this launch
  int tp_world;
  int tp_rank;
  int tp_tmax;  // token rows per (parity, source rank) in a mailbox
  int tp_smax;  // segment flags per (parity, source rank)
  unsigned long long tp_wait_ns;  // bound of each wait on a peer (wp_config.peer_wait_ms)
};

// Mailbox layout: partial rows [2 parities][world][tmax][kMaxRank] fp32, then
// flags [2][world][smax] int (the epoch that wrote the segment's rows), then
// done[world] int: the latest epoch whose launch has finished on rank `src`
// (after which that rank reads nothing more of that epoch's parity).
struct TpMail {
  static __host__ __device__ size_t data_floats(int world, int tmax) {
    return static_cast<size_t>(2) * world * tmax * kMaxRank;
  }
  static __host__ __device__ size_t bytes(int world, int tmax, int smax) {
    return data_floats(world, tmax) * 4 + static_cast<size_t>(2) * world * smax * 4 + static_cast<size_t>(world) * 4;
  }
  static __host__ __device__ int* done(float* mail, int world, int tmax, int smax, int src) {
    return reinterpret_cast<int*>(mail + data_floats(world, tmax)) + static_cast<size_t>(2) * world * smax + src;
  }
  static __host__ __device__ float* row(float* mail, int world, int tmax, int par, int src, int t) {
    return mail + ((static_cast<size_t>(par) * world + src) * tmax + t) * kMaxRank;
  }
  static __host__ __device__ int* flag(float* mail, int world, int tmax, int smax, int par, int src, int seg) {
    return reinterpret_cast<int*>(mail + data_floats(world, tmax)) + (static_cast<size_t>(par) * world + src) * smax + seg;
  }
};

// Per-CTA trace record (globaltimer ns) of the clustered apply kernel:
// start, after the dependency wait (compute warps), first stage ready, end,
// stages consumed, ns consumers spent waiting for stages, 0, 0; twelve marks
// (8: shrink of the first segment done, 9: its partials received from the
// cluster, 10: its H complete, 11: its partials pushed, 12: set-up done, 13:
// unused, 14: producer past the dependency wait, 15: table read, 16:
// producer before the dependency wait, 17: producer start, 18: first unit
// issued, 19: unused); then, for the first kTraceUnits stages that thread 0
// consumes, 8 timestamps each: before the stage wait, after it, four phase
// marks (expand: y in the accumulators, MMAs done, results in shared memory,
// stage released), 0, and the producer's issue of that stage-unit.
constexpr int kTraceUnits = 16;
constexpr int kTraceMarks = 8;
constexpr int kTraceSegMarks = 12;
constexpr int kTraceSlots = 8 + kTraceSegMarks + kTraceMarks * kTraceUnits;

struct LaunchCfg {
  int grid;
  int cluster;
  cudaStream_t stream;
  bool pdl;
};

// dtype: 0 = f16, 1 = bf16 (WP_DTYPE_*). Launches the clustered apply kernel
// on `lc.grid` CTAs in clusters of `lc.cluster`. Returns a cudaError_t.
cudaError_t launch_apply(int dtype, int rank, const ApplyArgs& a, const LaunchCfg& lc);
// Balanced decode kernel (no clusters): grid = one CTA per SM.
cudaError_t launch_apply_split(int dtype, int rank, const ApplyArgs& a, const LaunchCfg& lc);
int apply_split_max_grid(int dtype, int rank);

// Largest co-resident persistent grid for the apply kernel of (dtype, rank)
// with clusters of `cluster` CTAs (0 if that cluster size cannot be scheduled).
int apply_max_grid(int dtype, int rank, int cluster);
// co-resident CTAs of the clusters-of-4 live fused instantiation (ranks 8-32; else 0)
int apply_max_grid4(int dtype, int rank);

// idx_dtype: WP_DTYPE_I32 or WP_DTYPE_I64.
// Prefill mode of the segmenter (wp_segment.cu): tiles of long runs and the
// pieces of the short ones, besides the full table. tiles == nullptr: off.
struct PrefillTables {
  DevSeg* tiles = nullptr;
  int* tiles_num = nullptr;
  DevSeg* short_segs = nullptr;
  int* short_num = nullptr;
  int min_run = 0;
};

// slot_map / map_size (optional): translate adapter ids to adapter-pool
// slots as the table is written (see wp_segment.cu).
cudaError_t launch_seg_bounds(const void* idx, int idx_dtype, int T, DevSeg* segs, int* num_segs, ClusterPlan* plan,
                              int plan_g, int* run_starts, cudaStream_t stream, const int* slot_map = nullptr,
                              int map_size = 0, int* err = nullptr, PrefillTables pf = PrefillTables{});

// Prefill kernels (wp_prefill.cu): tcgen05 GEMMs over the tiles of long runs.
// a.segs / a.num_segs: the tile table; a.part / a.pmax: partials [T, pmax >=
// ceil(d / 1024), r]; a.tmap_x128: x with 128-row boxes; a.tmap_a / a.tmap_b
// as for the apply kernel. Ranks 16, 32, 64; d % 64 == 0, o % 64 == 0 and a
// 16-byte-addressable y.
cudaError_t launch_prefill(int dtype, int rank, const ApplyArgs& a, const LaunchCfg& lc);

}  // namespace wp
