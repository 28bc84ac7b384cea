// wp_api.cu -- host side of libwp_b200.so: the C ABI declared in
// include/wp_api.h. Owns the device segment tables, split-K workspaces, the
// adapter store (device tensors or the library's own pinned-host copies), the
// staging-slot pool with its private prefetch stream, the TMA descriptors of
// every launch, and the optional NCCL communicator for tensor-parallel shrink
// partials.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/wp_api.h"
#include "wp_internal.h"

using wp::DevSeg;

namespace {

thread_local std::string g_err;  // message for calls without a handle

struct Adapter {
  int32_t id = 0;
  const void* A = nullptr;  // device pointer (device adapters)
  const void* B = nullptr;
  void* hostA = nullptr;  // page-locked copies (host-store adapters)
  void* hostB = nullptr;
  bool host = false;
  int32_t r = 0, d = 0, o = 0;
  float alpha = 0.f;
  int32_t dtype = 0;
  size_t a_bytes = 0, b_bytes = 0;
};

struct Slot {
  int32_t adapter = -1;
  void* a = nullptr;  // inside the slot pool
  void* b = nullptr;
  cudaEvent_t ready = nullptr;
  bool issued = false;
  bool pinned = false;  // acquired by prefetch_adapter (released explicitly)
  uint64_t last_use = 0;  // build_segments generation (LRU for on-demand slots)
};

}  // namespace

struct wp_handle {
  wp_config cfg{};
  int device = 0;
  int num_sms = 148;
  std::string err;

  // live table (build_seg_bounds)
  DevSeg* d_live = nullptr;
  int* d_live_num = nullptr;
  // prefill mode of the latest build: 128-token tiles of the long runs and
  // the pieces of the short runs (the full table stays in d_live)
  DevSeg* d_tiles = nullptr;
  int* d_tiles_num = nullptr;
  DevSeg* d_short = nullptr;
  int* d_short_num = nullptr;
  bool live_prefill = false;
  int* d_run_starts = nullptr;
  // registry table (build_segments): unsplit host copy + split device copy
  DevSeg* d_reg = nullptr;
  int* d_reg_num = nullptr;
  // pinned upload buffers, double-buffered so that a build_segments call
  // waits only for the upload two calls back (cap + 1 entries, count in the tail)
  DevSeg* h_reg_stage[2] = {nullptr, nullptr};
  CUtensorMap* d_reg_maps = nullptr;  // TMA descriptors of the registry table's A matrices
  CUtensorMap* h_reg_maps[2] = {nullptr, nullptr};  // pinned upload buffers of the descriptors
  cudaEvent_t reg_uploaded[2] = {nullptr, nullptr};
  int reg_buf = 0;  // upload buffer of the next build_segments call
  std::vector<wp_segment> reg_table;
  std::vector<DevSeg> reg_pieces;
  int reg_rank = 0;
  int reg_dtype = -1;

  int* d_err = nullptr;  // device error word (wp::kErr* bits)
  // balanced decode (split) kernel: shrink partials, H, per-segment counters
  float* d_part = nullptr;
  size_t part_bytes = 0;
  float* d_hsplit = nullptr;
  size_t hsplit_bytes = 0;
  int* d_rflag = nullptr;  // per shrink item publication flags (zero between launches)
  size_t rflag_bytes = 0;
  int* d_sync = nullptr;  // 3 x cap ints, zero between launches
  std::vector<void*> retired;  // outgrown split buffers, freed by wp_destroy (graphs may hold them)
  // segment count of the latest build_seg_bounds, copied to pinned memory
  // without a sync; a hint for the automatic kernel choice
  int* h_nseg = nullptr;
  cudaEvent_t nseg_ready = nullptr;
  bool nseg_pending = false;
  int nseg_hint = -1;
  int last_kernel = -1;  // wp_last_apply_kernel
  // the segmenter's per-cluster assignment of the live table for plan_g clusters
  // [0]: clusters of the common launch; [1]: clusters of 4 (few-segment calls)
  wp::ClusterPlan* d_plan = nullptr;
  int plan_g = 0;
  int plan_g4 = 0;  // clusters of the clusters-of-4 launch (0: none)
  int sync_cap = 0;
  int split_grid[8] = {};

  // store + slots
  std::unordered_map<int32_t, Adapter> store;
  std::vector<Slot> slots;
  void* slot_pool = nullptr;
  cudaStream_t prefetch_stream = nullptr;
  cudaEvent_t caller_ready = nullptr;  // caller-stream point the prefetch waits on
  cudaEvent_t registry_done = nullptr;  // after the latest registry kernels
  bool registry_used = false;
  uint64_t generation = 0;

  // apply kernel plan per (dtype, rank): cluster size and persistent grid
  // launch plans per (variant, dtype, rank)
  int plan_cluster[16] = {};
  int plan_grid[16] = {};
  // optional per-CTA phase traces of the latest launch (0: fused/shrink, 1: expand-only)
  unsigned long long* d_trace[2] = {nullptr, nullptr};
  bool trace_on = false;

  // launch bookkeeping
  int64_t launches = 0;
  bool last_was_segmenter = false;
  bool input_written = false;  // wp_note_input_write: the next apply call's x was just written

  // tensor parallel
  ncclComm_t comm = nullptr;
  int tp_rank = 0, tp_world = 1;
  // row-parallel exchange over peer memory: this rank's mailbox, every
  // rank's mailbox as mapped here (own at tp_rank), the exchange epoch
  void* tp_mail_own = nullptr;
  float* tp_mail[wp::kMaxTp] = {};
  int mail_world = 0, mail_rank = 0, mail_tmax = 0;
  int* d_tp_seq = nullptr;
  bool tp_exchange = false;  // set for the duration of one row-parallel launch

  // scheduler bridge: page-locked, mapped into the device address space
  wp_bridge* bridge = nullptr;
  wp_bridge* d_bridge = nullptr;  // device alias of `bridge`
  float* d_bridge_out = nullptr;  // readback kernel output [WP_BRIDGE_MAX + 3]
};

namespace {

int fail(wp_handle* h, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (h)
    h->err = buf;
  else
    g_err = buf;
  return code;
}

#define WP_CUDA(h, call)                                                                              \
  do {                                                                                                \
    cudaError_t e_ = (call);                                                                          \
    if (e_ != cudaSuccess) return fail((h), WP_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

bool rank_ok(int r) { return r == 8 || r == 16 || r == 32 || r == 64; }
bool dtype16(int t) { return t == WP_DTYPE_F16 || t == WP_DTYPE_BF16; }
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Guard that makes the handle's device current for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Tiled map over 16-bit elements with the 128-byte swizzle. dims[0] is the
// innermost (contiguous) dimension; strides are in bytes for dims 1..rank-1.
bool encode_map(CUtensorMap* m, int dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides, const uint32_t* box,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t gd[4], gs[3];
  cuuint32_t bx[4], es[4] = {1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides[i];
  const CUtensorMapDataType dt =
      dtype == WP_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(m, dt, rank, const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// A stack [L, r, d] (row stride d, adapter stride `stride0` elements): box 64 x r x 1.
// d (A, x) or o (y) allows the sliced view [cols / 64][64] of a row.
bool sliced(int cols) { return cols % wp::kBoxCols == 0; }

// A stack [L, r, d]: sliced view [L][d / 64][r][64] with box {64, r, 4, 1}
// (4 slices of one stage, one instruction), else box {64, r, 1}.
bool encode_a_map(CUtensorMap* m, int dtype, const void* base, int d, int r, int64_t L, int64_t stride0) {
  if (sliced(d)) {
    const uint64_t dims[4] = {static_cast<uint64_t>(wp::kBoxCols), static_cast<uint64_t>(r),
                              static_cast<uint64_t>(d / wp::kBoxCols), static_cast<uint64_t>(L)};
    const uint64_t strides[3] = {static_cast<uint64_t>(d) * 2, static_cast<uint64_t>(wp::kBoxCols) * 2,
                                 static_cast<uint64_t>(stride0) * 2};
    const uint32_t box[4] = {static_cast<uint32_t>(wp::kBoxCols), static_cast<uint32_t>(r), 4, 1};
    return encode_map(m, dtype, 4, base, dims, strides, box);
  }
  const uint64_t dims[3] = {static_cast<uint64_t>(d), static_cast<uint64_t>(r), static_cast<uint64_t>(L)};
  const uint64_t strides[2] = {static_cast<uint64_t>(d) * 2, static_cast<uint64_t>(stride0) * 2};
  const uint32_t box[3] = {static_cast<uint32_t>(wp::kBoxCols), static_cast<uint32_t>(r), 1};
  return encode_map(m, dtype, 3, base, dims, strides, box);
}

// B stack [L, o, r] (row stride r, adapter stride `stride0` elements): box
// r x 128 x 1 with the swizzle whose span is one 2r-byte row (r >= 16).
bool encode_b_map(CUtensorMap* m, int dtype, const void* base, int o, int r, int64_t L, int64_t stride0,
                  uint32_t box_rows = 256) {
  const uint64_t dims[3] = {static_cast<uint64_t>(r), static_cast<uint64_t>(o), static_cast<uint64_t>(L)};
  const uint64_t strides[2] = {static_cast<uint64_t>(r) * 2, static_cast<uint64_t>(stride0) * 2};
  const uint32_t box[3] = {static_cast<uint32_t>(r), box_rows, 1};
  const CUtensorMapSwizzle sw =
      r == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : (r == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  return encode_map(m, dtype, 3, base, dims, strides, box, sw);
}

// Activation rows [T, cols] with row stride ld elements: box 64 x box_rows.
// Rows of x or y ([T, cols], leading dimension ld): sliced view
// [cols / 64][T][64] with box {64, box_rows, 4}, else box {64, box_rows}.
bool encode_rows_map(CUtensorMap* m, int dtype, const void* base, int cols, int T, int64_t ld, int box_rows,
                     int slices = 4) {
  if (sliced(cols)) {
    const uint64_t dims[3] = {static_cast<uint64_t>(wp::kBoxCols), static_cast<uint64_t>(T),
                              static_cast<uint64_t>(cols / wp::kBoxCols)};
    const uint64_t strides[2] = {static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(wp::kBoxCols) * 2};
    const uint32_t box[3] = {static_cast<uint32_t>(wp::kBoxCols), static_cast<uint32_t>(box_rows),
                             static_cast<uint32_t>(slices)};
    return encode_map(m, dtype, 3, base, dims, strides, box);
  }
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(T)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 2};
  const uint32_t box[2] = {static_cast<uint32_t>(wp::kBoxCols), static_cast<uint32_t>(box_rows)};
  return encode_map(m, dtype, 2, base, dims, strides, box);
}

// Upper bound on the CTAs of one apply launch (sizes the trace buffers).
int grid_size(const wp_handle* h) { return h->num_sms * 4; }

size_t slot_b_offset(size_t a_bytes) { return (a_bytes + 255) / 256 * 256; }

void wait_caller(wp_handle* h, cudaStream_t caller) {
  if (caller == nullptr) return;
  cudaEventRecord(h->caller_ready, caller);
  cudaStreamWaitEvent(h->prefetch_stream, h->caller_ready, 0);
}

// Copies an adapter into slot `si` on the prefetch stream and records its
// ready event. A slot reused after registry kernels read it waits for them.
int issue_slot_copy(wp_handle* h, int si, const Adapter& ad) {
  Slot& s = h->slots[si];
  const size_t boff = slot_b_offset(ad.a_bytes);
  s.a = static_cast<char*>(h->slot_pool) + static_cast<size_t>(si) * h->cfg.slot_bytes;
  s.b = static_cast<char*>(s.a) + boff;
  if (h->registry_used) cudaStreamWaitEvent(h->prefetch_stream, h->registry_done, 0);
  const cudaMemcpyKind kind = ad.host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  WP_CUDA(h, cudaMemcpyAsync(s.a, ad.host ? ad.hostA : ad.A, ad.a_bytes, kind, h->prefetch_stream));
  WP_CUDA(h, cudaMemcpyAsync(s.b, ad.host ? ad.hostB : ad.B, ad.b_bytes, kind, h->prefetch_stream));
  WP_CUDA(h, cudaEventRecord(s.ready, h->prefetch_stream));
  s.issued = true;
  return WP_OK;
}

int find_slot(const wp_handle* h, int32_t id) {
  for (size_t i = 0; i < h->slots.size(); ++i)
    if (h->slots[i].adapter == id) return static_cast<int>(i);
  return -1;
}

void release_slot(wp_handle* h, int si) {
  if (si < 0 || si >= static_cast<int>(h->slots.size())) return;
  h->slots[si].adapter = -1;
  h->slots[si].issued = false;
  h->slots[si].pinned = false;
}

bool fits_slot(const wp_handle* h, const Adapter& ad) {
  return slot_b_offset(ad.a_bytes) + ad.b_bytes <= static_cast<size_t>(h->cfg.slot_bytes);
}

void free_adapter(Adapter& ad) {
  if (ad.hostA) cudaFreeHost(ad.hostA);
  if (ad.hostB) cudaFreeHost(ad.hostB);
  ad.hostA = ad.hostB = nullptr;
}

}  // namespace

extern "C" {

const char* wp_last_error(const wp_handle* h) { return h ? h->err.c_str() : g_err.c_str(); }

int wp_set_global_error(int code, const char* msg) {
  g_err = msg ? msg : "";
  return code;
}

int wp_rank_supported(int32_t rank) { return rank_ok(rank) ? 1 : 0; }

int64_t wp_kernel_launch_count(const wp_handle* h) { return h ? h->launches : 0; }

int32_t wp_last_apply_kernel(const wp_handle* h) { return h ? h->last_kernel : -1; }

int wp_create(const wp_config* cfg_in, wp_handle** out) {
  if (!out) return fail(nullptr, WP_ERR_INVALID, "wp_create: out is NULL");
  *out = nullptr;
  wp_config cfg{};
  if (cfg_in) cfg = *cfg_in;
  if (cfg.max_tokens <= 0) cfg.max_tokens = 16384;
  if (cfg.num_staging_slots < 0) cfg.num_staging_slots = 0;
  if (cfg.slot_bytes <= 0) cfg.slot_bytes = static_cast<int64_t>(2) * 64 * 16384 * 2;
  cfg.slot_bytes = (cfg.slot_bytes + 255) / 256 * 256;
  if (cfg.ctas_per_sm < 0) cfg.ctas_per_sm = 0;
  if (cfg.kernel < 0 || cfg.kernel > 2) return fail(nullptr, WP_ERR_INVALID, "wp_create: kernel must be 0..2");

  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return fail(nullptr, WP_ERR_CUDA, "wp_create: no CUDA device is visible");
  if (cfg.device < 0 || cfg.device >= ndev) return fail(nullptr, WP_ERR_INVALID, "wp_create: bad device %d", cfg.device);

  wp_handle* h = new wp_handle();
  h->cfg = cfg;
  h->device = cfg.device;
  DeviceGuard dg(h->device);
  cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, h->device);

  const int cap = cfg.max_tokens;
  auto bail = [&](const char* what, cudaError_t e) {
    g_err = std::string("wp_create: ") + what + ": " + cudaGetErrorString(e);
    wp_destroy(h);
    return WP_ERR_CUDA;
  };
  cudaError_t e;
  if ((e = cudaMalloc(&h->d_live, sizeof(DevSeg) * cap)) != cudaSuccess) return bail("live table", e);
  if ((e = cudaMalloc(&h->d_tiles, sizeof(DevSeg) * (cap / wp::kPrefillTile + 1))) != cudaSuccess)
    return bail("prefill tile table", e);
  if ((e = cudaMalloc(&h->d_short, sizeof(DevSeg) * cap)) != cudaSuccess) return bail("short-run table", e);
  if ((e = cudaMalloc(&h->d_tiles_num, sizeof(int) * 4)) != cudaSuccess) return bail("tile count", e);
  if ((e = cudaMalloc(&h->d_short_num, sizeof(int) * 4)) != cudaSuccess) return bail("short-run count", e);
  cudaMemset(h->d_tiles_num, 0, sizeof(int) * 4);
  cudaMemset(h->d_short_num, 0, sizeof(int) * 4);
  if ((e = cudaMalloc(&h->d_live_num, sizeof(int) * 4)) != cudaSuccess) return bail("live count", e);
  if ((e = cudaMalloc(&h->d_run_starts, sizeof(int) * cap)) != cudaSuccess) return bail("run starts", e);
  if ((e = cudaMalloc(&h->d_reg, sizeof(DevSeg) * (cap + 1))) != cudaSuccess) return bail("registry table", e);
  if ((e = cudaMalloc(&h->d_reg_num, sizeof(int) * 4)) != cudaSuccess) return bail("registry count", e);
  for (int b = 0; b < 2; ++b)
    if ((e = cudaHostAlloc(&h->h_reg_stage[b], sizeof(DevSeg) * (cap + 1), cudaHostAllocDefault)) != cudaSuccess)
      return bail("registry upload buffer", e);
  if ((e = cudaMalloc(&h->d_reg_maps, sizeof(CUtensorMap) * cap)) != cudaSuccess) return bail("registry maps", e);
  for (int b = 0; b < 2; ++b)
    if ((e = cudaHostAlloc(&h->h_reg_maps[b], sizeof(CUtensorMap) * cap, cudaHostAllocDefault)) != cudaSuccess)
      return bail("registry map upload buffer", e);
  if ((e = cudaMalloc(&h->d_err, sizeof(int) * 4)) != cudaSuccess) return bail("error word", e);
  if ((e = cudaMalloc(&h->d_sync, sizeof(int) * 3 * cap)) != cudaSuccess) return bail("segment counters", e);
  if ((e = cudaHostAlloc(&h->h_nseg, sizeof(int) * 4, cudaHostAllocDefault)) != cudaSuccess)
    return bail("segment count buffer", e);
  if ((e = cudaMalloc(&h->d_plan, 2 * sizeof(wp::ClusterPlan))) != cudaSuccess) return bail("cluster plan", e);
  cudaMemset(h->d_plan, 0, 2 * sizeof(wp::ClusterPlan));
  cudaEventCreateWithFlags(&h->nseg_ready, cudaEventDisableTiming);
  cudaMemset(h->d_sync, 0, sizeof(int) * 3 * cap);
  h->sync_cap = cap;
  cudaMemset(h->d_live_num, 0, sizeof(int) * 4);
  cudaMemset(h->d_reg_num, 0, sizeof(int) * 4);
  cudaMemset(h->d_err, 0, sizeof(int) * 4);
  if ((e = cudaStreamCreateWithFlags(&h->prefetch_stream, cudaStreamNonBlocking)) != cudaSuccess)
    return bail("prefetch stream", e);
  for (int b = 0; b < 2; ++b) cudaEventCreateWithFlags(&h->reg_uploaded[b], cudaEventDisableTiming);
  cudaEventCreateWithFlags(&h->caller_ready, cudaEventDisableTiming);
  cudaEventCreateWithFlags(&h->registry_done, cudaEventDisableTiming);
  if (cfg.num_staging_slots > 0) {
    if ((e = cudaMalloc(&h->slot_pool, static_cast<size_t>(cfg.slot_bytes) * cfg.num_staging_slots)) != cudaSuccess)
      return bail("slot pool", e);
    h->slots.resize(cfg.num_staging_slots);
    for (auto& s : h->slots) cudaEventCreateWithFlags(&s.ready, cudaEventDisableTiming);
  }
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return bail("init sync", e);
  *out = h;
  return WP_OK;
}

int wp_destroy(wp_handle* h) {
  if (!h) return WP_OK;
  DeviceGuard dg(h->device);
  if (h->comm) ncclCommDestroy(h->comm);
  wp_tp_mailbox_close(h);
  if (h->prefetch_stream) cudaStreamSynchronize(h->prefetch_stream);
  cudaDeviceSynchronize();
  for (auto& kv : h->store) free_adapter(kv.second);
  for (auto& s : h->slots)
    if (s.ready) cudaEventDestroy(s.ready);
  if (h->slot_pool) cudaFree(h->slot_pool);
  cudaFree(h->d_live);
  cudaFree(h->d_tiles);
  cudaFree(h->d_short);
  cudaFree(h->d_tiles_num);
  cudaFree(h->d_short_num);
  cudaFree(h->d_live_num);
  cudaFree(h->d_run_starts);
  cudaFree(h->d_reg);
  cudaFree(h->d_reg_num);
  for (int b = 0; b < 2; ++b)
    if (h->h_reg_stage[b]) cudaFreeHost(h->h_reg_stage[b]);
  cudaFree(h->d_reg_maps);
  for (int b = 0; b < 2; ++b)
    if (h->h_reg_maps[b]) cudaFreeHost(h->h_reg_maps[b]);
  cudaFree(h->d_trace[0]);
  cudaFree(h->d_trace[1]);
  cudaFree(h->d_err);
  cudaFree(h->d_part);
  cudaFree(h->d_hsplit);
  cudaFree(h->d_rflag);
  for (void* p : h->retired) cudaFree(p);
  cudaFree(h->d_sync);
  cudaFree(h->d_plan);
  if (h->bridge) cudaFreeHost(h->bridge);
  cudaFree(h->d_bridge_out);
  if (h->h_nseg) cudaFreeHost(h->h_nseg);
  if (h->nseg_ready) cudaEventDestroy(h->nseg_ready);
  for (int b = 0; b < 2; ++b)
    if (h->reg_uploaded[b]) cudaEventDestroy(h->reg_uploaded[b]);
  if (h->caller_ready) cudaEventDestroy(h->caller_ready);
  if (h->registry_done) cudaEventDestroy(h->registry_done);
  if (h->prefetch_stream) cudaStreamDestroy(h->prefetch_stream);
  delete h;
  return WP_OK;
}

// ---- adapter store ---------------------------------------------------------

static int register_common(wp_handle* h, int32_t id, int32_t r, int32_t d, int32_t o, int32_t dtype) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "register_adapter: NULL handle");
  if (!rank_ok(r)) return fail(h, WP_ERR_INVALID, "register_adapter: unsupported rank %d (only 8/16/32/64)", r);
  if (!dtype16(dtype)) return fail(h, WP_ERR_INVALID, "register_adapter: A/B must be fp16 or bf16");
  if (d <= 0 || o <= 0 || d % 8 || o % 8)
    return fail(h, WP_ERR_INVALID, "register_adapter: d_model (%d) and out_features (%d) must be positive multiples of 8", d, o);
  (void)id;
  return WP_OK;
}

int wp_register_adapter(wp_handle* h, int32_t adapter_id, const void* A, const void* B, int32_t rank,
                        int32_t d_model, int32_t out_features, float alpha_scale, int32_t dtype) {
  int rc = register_common(h, adapter_id, rank, d_model, out_features, dtype);
  if (rc) return rc;
  if (!al16(A) || !al16(B))
    return fail(h, WP_ERR_INVALID, "AdapterStore::register_adapter: A/B pointer not 16-byte aligned");
  auto it = h->store.find(adapter_id);
  if (it != h->store.end()) free_adapter(it->second);
  Adapter ad;
  ad.id = adapter_id;
  ad.A = A;
  ad.B = B;
  ad.r = rank;
  ad.d = d_model;
  ad.o = out_features;
  ad.alpha = alpha_scale;
  ad.dtype = dtype;
  ad.a_bytes = static_cast<size_t>(rank) * d_model * 2;
  ad.b_bytes = static_cast<size_t>(out_features) * rank * 2;
  h->store[adapter_id] = ad;
  // A slot holding the previous weights of this id is stale now.
  int si = find_slot(h, adapter_id);
  if (si >= 0) release_slot(h, si);
  return WP_OK;
}

int wp_register_adapter_host(wp_handle* h, int32_t adapter_id, const void* A_host, const void* B_host,
                             int32_t rank, int32_t d_model, int32_t out_features, float alpha_scale,
                             int32_t dtype) {
  int rc = register_common(h, adapter_id, rank, d_model, out_features, dtype);
  if (rc) return rc;
  if (!A_host || !B_host) return fail(h, WP_ERR_INVALID, "register_adapter_host: NULL host pointer");
  DeviceGuard dg(h->device);
  Adapter ad;
  ad.id = adapter_id;
  ad.host = true;
  ad.r = rank;
  ad.d = d_model;
  ad.o = out_features;
  ad.alpha = alpha_scale;
  ad.dtype = dtype;
  ad.a_bytes = static_cast<size_t>(rank) * d_model * 2;
  ad.b_bytes = static_cast<size_t>(out_features) * rank * 2;
  if (!fits_slot(h, ad))
    return fail(h, WP_ERR_CAPACITY, "register_adapter_host: adapter (%zu B) exceeds slot_bytes (%lld)",
                slot_b_offset(ad.a_bytes) + ad.b_bytes, static_cast<long long>(h->cfg.slot_bytes));
  WP_CUDA(h, cudaHostAlloc(&ad.hostA, ad.a_bytes, cudaHostAllocDefault));
  if (cudaHostAlloc(&ad.hostB, ad.b_bytes, cudaHostAllocDefault) != cudaSuccess) {
    cudaFreeHost(ad.hostA);
    return fail(h, WP_ERR_CUDA, "register_adapter_host: cudaHostAlloc failed");
  }
  std::memcpy(ad.hostA, A_host, ad.a_bytes);
  std::memcpy(ad.hostB, B_host, ad.b_bytes);
  int si = find_slot(h, adapter_id);
  if (si >= 0) {
    // the old weights may still be in flight into the slot
    cudaEventSynchronize(h->slots[si].ready);
    release_slot(h, si);
  }
  auto it = h->store.find(adapter_id);
  if (it != h->store.end()) {
    cudaStreamSynchronize(h->prefetch_stream);  // old pinned copies may be read by a copy in flight
    free_adapter(it->second);
  }
  h->store[adapter_id] = ad;
  return WP_OK;
}

int wp_evict_adapter(wp_handle* h, int32_t adapter_id) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "evict_adapter: NULL handle");
  auto it = h->store.find(adapter_id);
  if (it == h->store.end()) return WP_OK;
  DeviceGuard dg(h->device);
  int si = find_slot(h, adapter_id);
  if (si >= 0) release_slot(h, si);
  if (it->second.host) cudaStreamSynchronize(h->prefetch_stream);
  free_adapter(it->second);
  h->store.erase(it);
  return WP_OK;
}

// ---- staging slots -----------------------------------------------------------

int32_t wp_prefetch_adapter(wp_handle* h, int32_t adapter_id) { return wp_prefetch_adapter_on(h, adapter_id, nullptr); }

int32_t wp_prefetch_adapter_on(wp_handle* h, int32_t adapter_id, void* caller_stream) {
  if (!h) return -1;
  auto it = h->store.find(adapter_id);
  if (it == h->store.end()) return -1;
  const Adapter& ad = it->second;
  int si = find_slot(h, adapter_id);
  if (si >= 0) {
    h->slots[si].pinned = true;
    return si;
  }
  if (!fits_slot(h, ad)) return -1;
  for (size_t i = 0; i < h->slots.size(); ++i) {
    if (h->slots[i].adapter == -1) {
      si = static_cast<int>(i);
      break;
    }
  }
  if (si < 0) return -1;  // pool exhausted: the reference returns -1 too
  DeviceGuard dg(h->device);
  Slot& s = h->slots[si];
  s.adapter = adapter_id;
  s.pinned = true;
  s.issued = false;
  wait_caller(h, static_cast<cudaStream_t>(caller_stream));
  if (issue_slot_copy(h, si, ad) != WP_OK) {
    release_slot(h, si);
    return -1;
  }
  return si;
}

int32_t wp_is_prefetch_ready(wp_handle* h, int32_t adapter_id) {
  if (!h) return 0;
  int si = find_slot(h, adapter_id);
  if (si < 0 || !h->slots[si].issued) return 0;
  DeviceGuard dg(h->device);
  return cudaEventQuery(h->slots[si].ready) == cudaSuccess ? 1 : 0;
}

int wp_release_prefetch(wp_handle* h, int32_t adapter_id) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "release_prefetch: NULL handle");
  release_slot(h, find_slot(h, adapter_id));
  return WP_OK;
}

int wp_slot_stats(wp_handle* h, int32_t* num_slots, int32_t* in_use) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "slot_stats: NULL handle");
  int used = 0;
  for (auto& s : h->slots) used += s.adapter >= 0;
  if (num_slots) *num_slots = static_cast<int32_t>(h->slots.size());
  if (in_use) *in_use = used;
  return WP_OK;
}

int wp_device_error(wp_handle* h, int32_t clear, int32_t* flag) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "device_error: NULL handle");
  DeviceGuard dg(h->device);
  WP_CUDA(h, cudaDeviceSynchronize());
  int v = 0;
  WP_CUDA(h, cudaMemcpy(&v, h->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (flag) *flag = v;
  if (clear) {
    WP_CUDA(h, cudaMemset(h->d_err, 0, sizeof(int)));
  }
  return WP_OK;
}

// ---- segment tables ----------------------------------------------------------

int wp_build_segments(wp_handle* h, const int32_t* ids, const int32_t* offs, int32_t K, void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "build_segments: NULL handle");
  if (K < 0 || (K > 0 && (!ids || !offs)))
    return fail(h, WP_ERR_INVALID, "build_segment_table: seg_offsets must have K+1 entries");
  if (K > h->cfg.max_tokens) return fail(h, WP_ERR_INVALID, "build_segment_table: K exceeds the table capacity (%d)", h->cfg.max_tokens);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  DeviceGuard dg(h->device);
  ++h->generation;

  std::vector<wp_segment> table(K);
  std::vector<DevSeg> pieces;
  pieces.reserve(K);
  std::vector<int> wait_slots;
  std::vector<CUtensorMap> maps;  // one TMA descriptor per distinct A matrix
  std::unordered_map<const void*, int> map_of;
  int rank = 0, dtype = -1;
  for (int i = 0; i < K; ++i) {
    auto it = h->store.find(ids[i]);
    if (it == h->store.end()) return fail(h, WP_ERR_UNKNOWN_ADAPTER, "AdapterStore::lookup: unknown adapter_id %d", ids[i]);
    const Adapter& ad = it->second;
    const int start = offs[i], count = offs[i + 1] - offs[i];
    if (count < 0 || start < 0) return fail(h, WP_ERR_INVALID, "build_segment_table: seg_offsets must be non-decreasing");
    if (offs[i + 1] > h->cfg.max_tokens) return fail(h, WP_ERR_INVALID, "build_segment_table: offsets exceed max_tokens (%d)", h->cfg.max_tokens);
    if (rank == 0) rank = ad.r;
    if (dtype < 0) dtype = ad.dtype;
    table[i] = wp_segment{ids[i], start, count};

    // weight pointers: a ready slot wins (reference: segment_builder.cpp:36-42);
    // host-store adapters always come from a slot, staged on demand.
    const void* pa = ad.A;
    const void* pb = ad.B;
    int si = find_slot(h, ids[i]);
    if (ad.host) {
      if (si < 0) {
        // free slot, else the least recently used on-demand slot not needed by this table
        for (size_t k = 0; k < h->slots.size(); ++k)
          if (h->slots[k].adapter == -1) {
            si = static_cast<int>(k);
            break;
          }
        if (si < 0) {
          uint64_t best = ~0ull;
          for (size_t k = 0; k < h->slots.size(); ++k) {
            const Slot& s = h->slots[k];
            if (!s.pinned && s.last_use < h->generation && s.last_use < best) {
              best = s.last_use;
              si = static_cast<int>(k);
            }
          }
        }
        if (si < 0) return fail(h, WP_ERR_CAPACITY, "build_segments: no staging slot free for host adapter %d", ids[i]);
        Slot& s = h->slots[si];
        s.adapter = ids[i];
        s.pinned = false;
        s.issued = false;
        if (issue_slot_copy(h, si, ad) != WP_OK) return WP_ERR_CUDA;
      }
      if (std::find(wait_slots.begin(), wait_slots.end(), si) == wait_slots.end()) wait_slots.push_back(si);
      pa = h->slots[si].a;
      pb = h->slots[si].b;
    } else if (si >= 0 && h->slots[si].issued && cudaEventQuery(h->slots[si].ready) == cudaSuccess) {
      pa = h->slots[si].a;
      pb = h->slots[si].b;
    }
    if (si >= 0) h->slots[si].last_use = h->generation;
    auto mit = map_of.find(pa);
    if (mit == map_of.end()) {
      // maps[2k] describes A of the k-th distinct adapter, maps[2k + 1] its B (ranks >= 16)
      CUtensorMap m[2];
      std::memset(m, 0, sizeof(m));
      if (!encode_a_map(&m[0], ad.dtype, pa, ad.d, ad.r, 1, static_cast<int64_t>(ad.r) * ad.d) ||
          (ad.r >= 16 && !encode_b_map(&m[1], ad.dtype, pb, ad.o, ad.r, 1, static_cast<int64_t>(ad.o) * ad.r)))
        return fail(h, WP_ERR_CUDA, "build_segments: cuTensorMapEncodeTiled failed for adapter %d", ids[i]);
      if (2 * maps.size() + 2 > static_cast<size_t>(h->cfg.max_tokens))
        return fail(h, WP_ERR_CAPACITY, "build_segments: too many distinct adapters in one table");
      mit = map_of.emplace(pa, static_cast<int>(maps.size())).first;  // index of A's map
      maps.push_back(m[0]);
      maps.push_back(m[1]);
    }
    for (int p = 0; p < count; p += wp::kSegTokens) {
      DevSeg s;
      s.adapter_id = ids[i];
      s.token_start = start + p;
      s.token_count = std::min(wp::kSegTokens, count - p);
      s.alpha = ad.alpha;
      s.a = h->d_reg_maps + mit->second;  // the kernel reads A through this descriptor
      s.b = ad.r >= 16 ? static_cast<const void*>(h->d_reg_maps + mit->second + 1) : pb;
      pieces.push_back(s);
    }
  }
  if (static_cast<int>(pieces.size()) > h->cfg.max_tokens)
    return fail(h, WP_ERR_CAPACITY, "build_segments: %zu pieces exceed the table capacity", pieces.size());
  for (int si : wait_slots) WP_CUDA(h, cudaStreamWaitEvent(stream, h->slots[si].ready, 0));

  // upload through one of the two pinned buffers; the host waits only until
  // the upload that used it two calls back has left it
  const int ub = h->reg_buf;
  h->reg_buf ^= 1;
  WP_CUDA(h, cudaEventSynchronize(h->reg_uploaded[ub]));
  DevSeg* stage = h->h_reg_stage[ub];
  const int np = static_cast<int>(pieces.size());
  if (np) std::memcpy(stage, pieces.data(), sizeof(DevSeg) * np);
  int* cnt = reinterpret_cast<int*>(stage + h->cfg.max_tokens);
  *cnt = np;
  if (np) WP_CUDA(h, cudaMemcpyAsync(h->d_reg, stage, sizeof(DevSeg) * np, cudaMemcpyHostToDevice, stream));
  if (!maps.empty()) {
    std::memcpy(h->h_reg_maps[ub], maps.data(), sizeof(CUtensorMap) * maps.size());
    WP_CUDA(h, cudaMemcpyAsync(h->d_reg_maps, h->h_reg_maps[ub], sizeof(CUtensorMap) * maps.size(),
                               cudaMemcpyHostToDevice, stream));
  }
  WP_CUDA(h, cudaMemcpyAsync(h->d_reg_num, cnt, sizeof(int), cudaMemcpyHostToDevice, stream));
  WP_CUDA(h, cudaEventRecord(h->reg_uploaded[ub], stream));
  h->reg_table.swap(table);
  h->reg_pieces.swap(pieces);
  h->reg_rank = rank;
  h->reg_dtype = dtype;
  h->last_was_segmenter = false;
  return WP_OK;
}

}  // extern "C"
namespace {
void apply_plan(wp_handle* h, int dtype, int r, int* cluster, int* grid);
int plan_clusters4(wp_handle* h);
}  // namespace
extern "C" {

int wp_build_seg_bounds(wp_handle* h, const void* idx, int32_t idx_dtype, int32_t T, void* stream_v) {
  return wp_build_seg_bounds_ex(h, idx, idx_dtype, T, WP_SEG_AUTO, stream_v);
}

int wp_build_seg_bounds_ex(wp_handle* h, const void* idx, int32_t idx_dtype, int32_t T, int32_t flags,
                           void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "build_seg_bounds: NULL handle");
  if (flags < WP_SEG_DECODE || flags > WP_SEG_AUTO) return fail(h, WP_ERR_INVALID, "build_seg_bounds: bad flags %d", flags);
  if (idx_dtype != WP_DTYPE_I32 && idx_dtype != WP_DTYPE_I64)
    return fail(h, WP_ERR_INVALID, "build_seg_bounds: token_lora_indices must be int32 or int64");
  if (T < 0) return fail(h, WP_ERR_INVALID, "build_seg_bounds: negative token count");
  if (T > h->cfg.max_tokens) return WP_NOT_HANDLED;
  if (T > 0 && !idx) return fail(h, WP_ERR_INVALID, "build_seg_bounds: NULL indices");
  DeviceGuard dg(h->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (h->plan_g == 0) {
    // the clustered decode plan of the common case (bf16, rank 32): every
    // rank plans the same cluster count on B200, and a launch whose count
    // differs ignores the assignment
    int c = 1, g = 1;
    apply_plan(h, WP_DTYPE_BF16, 32, &c, &g);
    h->plan_g = g / std::max(c, 1);
    h->plan_g4 = plan_clusters4(h);
  }
  const bool prefill =
      flags == WP_SEG_PREFILL || (flags == WP_SEG_AUTO && h->cfg.prefill_tokens > 0 && T >= h->cfg.prefill_tokens);
  wp::PrefillTables pf;
  if (prefill) {
    pf.tiles = h->d_tiles;
    pf.tiles_num = h->d_tiles_num;
    pf.short_segs = h->d_short;
    pf.short_num = h->d_short_num;
    pf.min_run = wp::kPrefillMinRun;
  }
  cudaError_t e = wp::launch_seg_bounds(idx, idx_dtype, T, h->d_live, h->d_live_num, h->d_plan,
                                        h->plan_g | (h->plan_g4 << 16), h->d_run_starts, stream, nullptr, 0, nullptr,
                                        pf);
  if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "build_seg_bounds launch: %s", cudaGetErrorString(e));
  h->live_prefill = prefill;
  ++h->launches;
  h->last_was_segmenter = true;
  // the segment count travels to the host asynchronously (outside graph
  // capture); later calls read it once it has landed
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone && h->h_nseg &&
      cudaMemcpyAsync(h->h_nseg, h->d_live_num, sizeof(int), cudaMemcpyDeviceToHost, stream) == cudaSuccess &&
      cudaEventRecord(h->nseg_ready, stream) == cudaSuccess) {
    h->nseg_pending = true;
    h->last_was_segmenter = false;  // the copy sits between the segmenter and the next kernel
  }
  return WP_OK;
}

int wp_read_seg_table(wp_handle* h, int32_t which, wp_segment* out, int32_t cap, int32_t* num) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "read_seg_table: NULL handle");
  DeviceGuard dg(h->device);
  if (which == WP_TABLE_TILES || which == WP_TABLE_SHORT) {
    const DevSeg* segs = which == WP_TABLE_TILES ? h->d_tiles : h->d_short;
    const int* cnt = which == WP_TABLE_TILES ? h->d_tiles_num : h->d_short_num;
    WP_CUDA(h, cudaDeviceSynchronize());
    int n = 0;
    WP_CUDA(h, cudaMemcpy(&n, cnt, sizeof(int), cudaMemcpyDeviceToHost));
    if (!h->live_prefill) n = 0;
    if (num) *num = n;
    const int m = std::min(n, cap);
    std::vector<DevSeg> tmp(std::max(m, 0));
    if (m > 0) WP_CUDA(h, cudaMemcpy(tmp.data(), segs, sizeof(DevSeg) * m, cudaMemcpyDeviceToHost));
    for (int i = 0; i < m; ++i) out[i] = wp_segment{tmp[i].adapter_id, tmp[i].token_start, tmp[i].token_count};
    return WP_OK;
  }
  if (which == WP_TABLE_REGISTRY) {
    const int n = static_cast<int>(h->reg_table.size());
    if (num) *num = n;
    for (int i = 0; i < std::min(n, cap); ++i) out[i] = h->reg_table[i];
    return WP_OK;
  }
  WP_CUDA(h, cudaDeviceSynchronize());
  int n = 0;
  WP_CUDA(h, cudaMemcpy(&n, h->d_live_num, sizeof(int), cudaMemcpyDeviceToHost));
  if (num) *num = n;
  const int m = std::min(n, cap);
  if (m > 0) {
    std::vector<DevSeg> tmp(m);
    WP_CUDA(h, cudaMemcpy(tmp.data(), h->d_live, sizeof(DevSeg) * m, cudaMemcpyDeviceToHost));
    for (int i = 0; i < m; ++i) out[i] = wp_segment{tmp[i].adapter_id, tmp[i].token_start, tmp[i].token_count};
  }
  return WP_OK;
}

// ---- apply -------------------------------------------------------------------

}  // extern "C"

namespace {

// Cluster size and persistent grid of the apply kernel for (dtype, rank):
// the largest cluster whose co-resident grid keeps at least 95% of the CTAs
// that the best cluster size achieves (cached per handle).
void apply_plan(wp_handle* h, int dtype, int r, int* cluster, int* grid) {
  const int key = (dtype == WP_DTYPE_BF16 ? 4 : 0) + (r == 8 ? 0 : r == 16 ? 1 : r == 32 ? 2 : 3);
  if (h->plan_grid[key] == 0) {
    const int sizes[4] = {8, 4, 2, 1};
    int g[4], best = 0;
    for (int i = 0; i < 4; ++i) {
      g[i] = wp::apply_max_grid(dtype, r, sizes[i]);
      if (h->cfg.ctas_per_sm > 0) g[i] = std::min(g[i], h->num_sms * h->cfg.ctas_per_sm / sizes[i] * sizes[i]);
      best = std::max(best, g[i]);
    }
    int pick = 3;
    for (int i = 0; i < 4; ++i)
      if (g[i] > 0 && g[i] * 100 >= best * 95) {
        pick = i;
        break;
      }
    // tuning override: WP_CLUSTER=1|2|4|8 forces the cluster size (when schedulable)
    if (const char* env = std::getenv("WP_CLUSTER")) {
      const int want = std::atoi(env);
      for (int i = 0; i < 4; ++i)
        if (sizes[i] == want && g[i] > 0) pick = i;
    }
    h->plan_cluster[key] = sizes[pick];
    h->plan_grid[key] = std::max(g[pick], sizes[pick]);
  }
  *cluster = h->plan_cluster[key];
  *grid = h->plan_grid[key];
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

// Clusters of the clusters-of-4 launch (bf16, rank 32: the same count for
// every rank and dtype on B200), within the plan's capacity; 0 when off
// (WP_CLUSTER4=0, a tuning knob) or not schedulable.
int plan_clusters4(wp_handle* h) {
  static const bool off = [] {
    const char* e = std::getenv("WP_CLUSTER4");
    return e && std::strcmp(e, "0") == 0;
  }();
  if (off) return 0;
  int g = wp::apply_max_grid4(WP_DTYPE_BF16, 32);
  if (h->cfg.ctas_per_sm > 0) g = std::min(g, h->num_sms * h->cfg.ctas_per_sm / 4 * 4);
  g = std::min(g / 4, wp::kPlanMaxClusters);
  return g >= 2 ? g : 0;
}

// Kernel choice (wp_config.kernel; 0 = automatic, or WP_KERNEL when set, a
// tuning knob): 1 = clustered, 2 = balanced ("split") for fused live-mode
// calls. Returns 0 for split, 1 for clustered, -1 for automatic.
int kernel_choice(const wp_handle* h) {
  static const int env = [] {
    const char* e = std::getenv("WP_KERNEL");
    if (e && std::strcmp(e, "split") == 0) return 0;
    if (e && (std::strcmp(e, "dec") == 0 || std::strcmp(e, "cluster") == 0)) return 1;
    return -1;
  }();
  switch (h->cfg.kernel) {
    case 1: return 1;
    case 2: return 0;
    default: return env;
  }
}

// Automatic choice for a fused live-mode call, from a cost model of the two
// decode kernels fitted to B200 measurements (rank 32, bf16, 256 tokens,
// 1-512 resident adapters, q / gate / down shapes; us per launch inside a
// CUDA graph):
//   clustered: ~2.0 + 0.33 x (pipeline stages of the busiest CTA), where a
//     segment's CTA pair streams half of d each and a helper pair halves the
//     output columns when clusters are left over;
//   balanced ("split"): ~9.2 + 0.9 x (stages per CTA with every segment's
//     stages spread over the whole grid) -- its flag exchange through L2
//     costs a fixed ~7 us more.
// On the measured shapes the clustered kernel is always the faster one; the
// balanced kernel wins only for a few segments of a very large d or o.
// The segment count is the latest segmenter's (read without a sync); before
// one has landed, the bound min(T, A + ceil(T / 32)) for A adapters among T
// tokens stands in.
// The latest segmenter's segment count, once its copy to pinned memory has
// landed (checked without a sync, outside stream capture); -1 before.
int nseg_latest(wp_handle* h, cudaStream_t stream) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (h->nseg_pending && cudaStreamIsCapturing(stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone &&
      cudaEventQuery(h->nseg_ready) == cudaSuccess) {
    h->nseg_hint = *h->h_nseg;
    h->nseg_pending = false;
  }
  cudaGetLastError();  // a not-ready query is not an error
  return h->nseg_hint;
}

bool auto_split(wp_handle* h, cudaStream_t stream, int T, int64_t num_adapters, int clusters, int cluster, int d,
                int o) {
  int64_t nseg = nseg_latest(h, stream);
  if (nseg < 0) nseg = std::min<int64_t>(T, std::max<int64_t>(num_adapters, 1) + (T + wp::kSegTokens - 1) / wp::kSegTokens);
  if (nseg <= 0 || clusters <= 0) return false;
  const int64_t cl = std::max(cluster, 1);
  auto stages = [](int64_t cols) { return (cols + wp::kStageK - 1) / wp::kStageK; };
  const int64_t nA = stages((d + cl - 1) / cl);
  const int64_t nB = stages((o + cl - 1) / cl);
  const int64_t half = (((o + 1) / 2) + wp::kStageCols - 1) / wp::kStageCols * wp::kStageCols;
  const int64_t nB_half = stages((half + cl - 1) / cl);
  int64_t busiest;
  if (nseg <= clusters) {
    const int64_t helpers = std::min<int64_t>(nseg, clusters - nseg);
    busiest = nA + (helpers == nseg ? nB_half : nB);
  } else {
    busiest = (nseg + clusters - 1) / clusters * (nA + nB);
  }
  const double cost_cluster = 2.0 + 0.33 * static_cast<double>(busiest);
  const double per_cta = static_cast<double>(nseg * (stages(d) + stages(o))) / static_cast<double>(h->num_sms);
  const double cost_split = 9.2 + 0.9 * per_cta;
  return cost_split < cost_cluster;
}

// Makes the split kernel's buffers hold T tokens of nchunk partials of rank r.
// Outside stream capture they grow as needed (at least doubling); under
// capture (no allocation allowed) a call that does not fit returns false and
// runs the clustered kernel instead. A buffer that is outgrown is never freed
// before wp_destroy: a CUDA graph captured earlier keeps its address in its
// kernel arguments and may still be replayed.
bool grow_buffer(wp_handle* h, void** buf, size_t* have, size_t need, bool zero, cudaStream_t stream) {
  if (need <= *have) return true;
  const size_t want = std::max(need, *have * 2);
  void* p = nullptr;
  if (cudaMalloc(&p, want) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (zero && cudaMemsetAsync(p, 0, want, stream) != cudaSuccess) {
    cudaFree(p);
    return false;
  }
  if (*buf) h->retired.push_back(*buf);
  *buf = p;
  *have = want;
  return true;
}

bool split_buffers(wp_handle* h, int T, int nchunk, int r, cudaStream_t stream) {
  const size_t part = static_cast<size_t>(T) * nchunk * r * 4;
  const size_t hs = static_cast<size_t>(T) * r * 4;
  const size_t rf = static_cast<size_t>(T) * nchunk * 4;
  if (part <= h->part_bytes && hs <= h->hsplit_bytes && rf <= h->rflag_bytes) return true;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
  return grow_buffer(h, reinterpret_cast<void**>(&h->d_part), &h->part_bytes, part, false, stream) &&
         grow_buffer(h, reinterpret_cast<void**>(&h->d_hsplit), &h->hsplit_bytes, hs, false, stream) &&
         grow_buffer(h, reinterpret_cast<void**>(&h->d_rflag), &h->rflag_bytes, rf, true, stream);
}

// One apply launch. mode: wp::kModeShrink / kModeExpand / kModeFused.
int do_apply(wp_handle* h, int mode, int registry, const DevSeg* segs, const int* nseg, int T, int r, int dtype,
             const void* x, int64_t x_ld, int d, const void* wa, int64_t wa_stride, int64_t num_adapters, float scale,
             void* y, int64_t y_ld, int y_off, int o, const void* wb, int64_t wb_stride, float* H,
             cudaStream_t stream) {
  if (T == 0) return WP_OK;  // no rows: nothing to launch
  wp::ApplyArgs a{};
  a.segs = segs;
  a.num_segs = nseg;
  a.plan = (!registry && segs == h->d_live) ? h->d_plan : nullptr;
  a.h = H;
  a.mode = mode;
  a.registry = registry;
  a.scale = scale;
  a.err = h->d_err;
  a.trace = h->trace_on ? h->d_trace[mode == wp::kModeExpand ? 1 : 0] : nullptr;
  if (mode & wp::kModeShrink) {
    a.d = d;
    a.d_sliced = sliced(d) ? 1 : 0;
    for (int i = 0; i < 3; ++i)
      if (!encode_rows_map(&a.tmap_x[i], dtype, x, d, T, x_ld, 8 << i))
        return fail(h, WP_ERR_CUDA, "apply: cuTensorMapEncodeTiled(x) failed");
    if (!registry && !encode_a_map(&a.tmap_a, dtype, wa, d, r, std::max<int64_t>(1, num_adapters), wa_stride))
      return fail(h, WP_ERR_CUDA, "apply: cuTensorMapEncodeTiled(wa_t_all) failed");
  }
  if (mode & wp::kModeExpand) {
    a.y = y;
    a.y_ld = y_ld;
    a.y_off = y_off;
    a.o = o;
    a.wb_base = wb;
    a.wb_stride = wb_stride;
    a.y_tma = al16(y) && (y_ld % 8 == 0) && (y_off % 8 == 0);
    a.o_sliced = sliced(o) ? 1 : 0;
    if (!registry && r >= 16 && !encode_b_map(&a.tmap_b, dtype, wb, o, r, std::max<int64_t>(1, num_adapters), wb_stride))
      return fail(h, WP_ERR_CUDA, "apply: cuTensorMapEncodeTiled(wb_t_all) failed");
    for (int i = 0; a.y_tma && i < 3; ++i)
      if (!encode_rows_map(&a.tmap_y[i], dtype, static_cast<const char*>(y) + static_cast<int64_t>(y_off) * 2, o, T,
                           y_ld, 8 << i))
        return fail(h, WP_ERR_CUDA, "apply: cuTensorMapEncodeTiled(y) failed");
  }
  if (h->tp_exchange) {
    a.tp_world = h->mail_world;
    a.tp_rank = h->mail_rank;
    a.tp_tmax = h->mail_tmax;
    a.tp_smax = h->mail_tmax;
    a.tp_seq = h->d_tp_seq;
    a.tp_wait_ns = static_cast<unsigned long long>(h->cfg.peer_wait_ms > 0 ? h->cfg.peer_wait_ms : 5000) * 1000000ull;
    for (int p = 0; p < wp::kMaxTp; ++p) a.tp_mail[p] = h->tp_mail[p];
  }
  const bool pdl = h->cfg.use_pdl != 0;
  // Without PDL the kernel starts after its predecessor completed, so the
  // table and weights can always be read first. With PDL that needs the
  // caller's promise (prefetch_weights) that the preceding kernel writes no
  // adapter weights, and a preceding kernel that is not the segmenter.
  a.prefetch_weights = !pdl || (h->cfg.prefetch_weights != 0 && !h->last_was_segmenter);
  // x as well (fused live calls): the caller's further promise
  // (prefetch_inputs) that the preceding kernel writes no x, unless it said
  // otherwise for this call (wp_note_input_write)
  a.prefetch_inputs = pdl && a.prefetch_weights && h->cfg.prefetch_inputs != 0 && !h->input_written &&
                      mode == wp::kModeFused && !registry && !h->tp_exchange && a.y_tma;
  h->input_written = false;
  const int nchunk = (d + wp::kStageK - 1) / wp::kStageK;
  const int64_t nchunk_max = std::max<int64_t>(nchunk, (o + wp::kStageCols - 1) / wp::kStageCols);
  // the split kernel's item arithmetic is 32-bit (items x grid < 2^31) and its
  // run masks cover 2048 chunks
  const bool split_fits = static_cast<int64_t>(T) * nchunk_max * h->num_sms < (int64_t{1} << 31) && nchunk_max <= 2048;
  bool want_split = kernel_choice(h) == 0 && !h->tp_exchange;
  if (kernel_choice(h) < 0 && mode == wp::kModeFused && !registry && !h->tp_exchange) {
    int c0 = 1, g0 = 1;
    apply_plan(h, dtype, r, &c0, &g0);
    want_split = auto_split(h, stream, T, num_adapters, g0 / std::max(c0, 1), c0, d, o);
  }
  if (mode == wp::kModeFused && !registry && want_split && T <= h->sync_cap && split_fits) {
    const int key = (dtype == WP_DTYPE_BF16 ? 4 : 0) + (r == 8 ? 0 : r == 16 ? 1 : r == 32 ? 2 : 3);
    if (h->split_grid[key] == 0) h->split_grid[key] = wp::apply_split_max_grid(dtype, r);
    if (h->split_grid[key] > 0 && split_buffers(h, T, nchunk, r, stream)) {
      a.part = h->d_part;
      a.hsplit = h->d_hsplit;
      a.sync = h->d_sync;
      a.rflag = h->d_rflag;
      a.pmax = nchunk;
      a.sync_cap = h->sync_cap;
      a.scale = scale;
      wp::LaunchCfg lc{h->split_grid[key], 1, stream, pdl};
      cudaError_t e = wp::launch_apply_split(dtype, r, a, lc);
      if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "apply launch (split): %s", cudaGetErrorString(e));
      h->last_kernel = 0;
      ++h->launches;
      h->last_was_segmenter = false;
      return WP_OK;
    }
  }
  int cluster = 1, grid = 1;
  apply_plan(h, dtype, r, &cluster, &grid);
  // Few segments (no more than the clusters of 4): clusters of 4 spread each
  // segment's shrink and expand over four CTAs instead of two, which halves
  // the busiest CTA's stages; with more segments a cluster would hold two.
  // The segment count is the latest segmenter's (see auto_split).
  if (cluster == 2 && h->plan_g4 > 0 && mode == wp::kModeFused && !registry && !h->tp_exchange && !h->trace_on &&
      r <= 32 && a.y_tma && sliced(d) && sliced(o) && a.plan != nullptr) {
    const int64_t nseg = nseg_latest(h, stream);
    const int min_cols = 4 * wp::kStageCols;  // a cluster's output columns split four ways
    if (nseg > 0 && nseg < h->plan_g4 && o >= 2 * min_cols && d >= min_cols) {
      cluster = 4;
      grid = 4 * h->plan_g4;
      a.plan = h->d_plan + 1;
    }
  }
  a.split_len = round_up((std::max(d, 1) + cluster - 1) / cluster, wp::kStageK);
  a.oslice = round_up((std::max(o, 1) + cluster - 1) / cluster, wp::kStageCols);
  wp::LaunchCfg lc{grid, cluster, stream, pdl};
  cudaError_t e = wp::launch_apply(dtype, r, a, lc);
  if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "apply launch: %s", cudaGetErrorString(e));
  h->last_kernel = cluster == 4 ? 3 : 1;
  ++h->launches;
  h->last_was_segmenter = false;
  return WP_OK;
}

// Whether a fused live call goes to the prefill kernels (its long runs) and
// the decode kernel on the short-run table: the latest build was in prefill
// mode; rank 16, 32 or 64; d and o multiples of 64 (the sliced tensor maps);
// y 16-byte addressable; T within the tables; the partial scratch fits.
// Otherwise the full table goes to the decode kernel.
bool prefill_eligible(wp_handle* h, int T, int r, int d, int o, const void* y, int64_t y_ld, int y_off,
                      cudaStream_t stream) {
  if (!h->live_prefill || T == 0 || h->tp_exchange) return false;
  if (!(r == 16 || r == 32 || r == 64) || d % 64 != 0 || o % 64 != 0) return false;
  if (!(al16(y) && y_ld % 8 == 0 && y_off % 8 == 0) || T > h->sync_cap) return false;
  const int nchunk = (d + wp::kStageK - 1) / wp::kStageK;  // >= the prefill shrink's 1024-column chunks
  return split_buffers(h, T, nchunk, r, stream);
}

// The prefill kernels over the tile table. late_wait: the previous kernel on
// the stream is this call's decode kernel on the short runs (the prefill
// shrink then runs beside it, see wp_prefill.cu).
int launch_prefill_call(wp_handle* h, int T, int r, int dtype, const void* x, int64_t x_ld, int d, const void* wa,
                        int64_t wa_stride, int64_t num_adapters, float scale, void* y, int64_t y_ld, int y_off, int o,
                        const void* wb, int64_t wb_stride, bool late_wait, cudaStream_t stream) {
  const int nchunk = (d + wp::kStageK - 1) / wp::kStageK;
  wp::ApplyArgs a{};
  a.segs = h->d_tiles;
  a.num_segs = h->d_tiles_num;
  a.sync_cap = h->sync_cap / wp::kPrefillTile + 1;
  a.part = h->d_part;
  a.pmax = nchunk;
  a.err = h->d_err;
  a.d = d;
  a.o = o;
  a.y = y;
  a.y_ld = y_ld;
  a.y_off = y_off;
  a.scale = scale;
  a.pf_late_wait = late_wait && h->cfg.use_pdl != 0 ? 1 : 0;
  a.trace = h->trace_on ? h->d_trace[1] : nullptr;  // the expand kernel's timeline
  if (!encode_rows_map(&a.tmap_x128, dtype, x, d, T, x_ld, wp::kPrefillTile) ||
      !encode_rows_map(&a.tmap_y128, dtype, static_cast<const char*>(y) + static_cast<int64_t>(y_off) * 2, o, T,
                       y_ld, wp::kPrefillTile, 1) ||
      !encode_a_map(&a.tmap_a, dtype, wa, d, r, std::max<int64_t>(1, num_adapters), wa_stride) ||
      !encode_b_map(&a.tmap_b64, dtype, wb, o, r, std::max<int64_t>(1, num_adapters), wb_stride, 64))
    return fail(h, WP_ERR_CUDA, "prefill: cuTensorMapEncodeTiled failed");
  wp::LaunchCfg lc{h->num_sms, 1, stream, h->cfg.use_pdl != 0};
  cudaError_t e = wp::launch_prefill(dtype, r, a, lc);
  if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "prefill launch: %s", cudaGetErrorString(e));
  h->launches += 2;
  h->last_was_segmenter = false;
  return WP_OK;
}

}  // namespace

extern "C" {

int wp_shrink(wp_handle* h, const void* X, void* H, int32_t d_model, int32_t rank, int32_t T, int32_t dtype,
              void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "shrink: NULL handle");
  if (!rank_ok(rank)) return fail(h, WP_ERR_INVALID, "dispatch_bgmv_shrink: unsupported rank (only 8/16/32/64)");
  if (!dtype16(dtype)) return fail(h, WP_ERR_INVALID, "shrink: X must be fp16 or bf16");
  if (d_model <= 0 || d_model % 8) return fail(h, WP_ERR_INVALID, "shrink: d_model must be a positive multiple of 8");
  if (T < 0 || T > h->cfg.max_tokens) return fail(h, WP_ERR_INVALID, "shrink: total_tokens %d outside [0, %d]", T, h->cfg.max_tokens);
  if (!al16(X) || !al16(H)) return fail(h, WP_ERR_INVALID, "shrink: X/H must be 16-byte aligned");
  for (const DevSeg& s : h->reg_pieces) {
    const Adapter* ad = nullptr;
    auto it = h->store.find(s.adapter_id);
    if (it != h->store.end()) ad = &it->second;
    if (!ad) return fail(h, WP_ERR_UNKNOWN_ADAPTER, "shrink: adapter %d was evicted after build_segments", s.adapter_id);
    if (ad->r != rank || ad->d != d_model || ad->dtype != dtype)
      return fail(h, WP_ERR_INVALID, "shrink: adapter %d is rank %d, d_model %d; the call asks for rank %d, d_model %d",
                  s.adapter_id, ad->r, ad->d, rank, d_model);
    if (s.token_start + s.token_count > T)
      return fail(h, WP_ERR_INVALID, "shrink: segment [%d, %d) exceeds total_tokens %d", s.token_start,
                  s.token_start + s.token_count, T);
  }
  DeviceGuard dg(h->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  int rc = do_apply(h, wp::kModeShrink, 1, h->d_reg, h->d_reg_num, T, rank, dtype, X, d_model, d_model, nullptr, 0,
                    0, 0.f, nullptr, 0, 0, 0, nullptr, 0, static_cast<float*>(H), stream);
  if (rc) return rc;
  cudaEventRecord(h->registry_done, stream);
  h->registry_used = true;
  return WP_OK;
}

int wp_expand(wp_handle* h, const void* H, void* Y, int32_t out_features, int32_t rank, int32_t T, int32_t dtype,
              void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "expand: NULL handle");
  if (!rank_ok(rank)) return fail(h, WP_ERR_INVALID, "dispatch_bgmv_expand: unsupported rank (only 8/16/32/64)");
  if (!dtype16(dtype)) return fail(h, WP_ERR_INVALID, "expand: Y must be fp16 or bf16");
  if (out_features <= 0 || out_features % 8)
    return fail(h, WP_ERR_INVALID, "expand: out_features must be a positive multiple of 8");
  if (T < 0 || T > h->cfg.max_tokens) return fail(h, WP_ERR_INVALID, "expand: total_tokens outside [0, %d]", h->cfg.max_tokens);
  if (!al16(H)) return fail(h, WP_ERR_INVALID, "expand: H must be 16-byte aligned");
  for (const DevSeg& s : h->reg_pieces) {
    auto it = h->store.find(s.adapter_id);
    if (it == h->store.end()) return fail(h, WP_ERR_UNKNOWN_ADAPTER, "expand: adapter %d was evicted after build_segments", s.adapter_id);
    if (it->second.r != rank || it->second.o != out_features || it->second.dtype != dtype)
      return fail(h, WP_ERR_INVALID, "expand: adapter %d is rank %d, out_features %d; the call asks for rank %d, out_features %d",
                  s.adapter_id, it->second.r, it->second.o, rank, out_features);
    if (s.token_start + s.token_count > T)
      return fail(h, WP_ERR_INVALID, "expand: segment exceeds total_tokens %d", T);
  }
  DeviceGuard dg(h->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  int rc = do_apply(h, wp::kModeExpand, 1, h->d_reg, h->d_reg_num, T, rank, dtype, nullptr, 0, 0, nullptr, 0, 0, 0.f,
                    Y, out_features, 0, out_features, nullptr, 0, const_cast<float*>(static_cast<const float*>(H)),
                    stream);
  if (rc) return rc;
  cudaEventRecord(h->registry_done, stream);
  h->registry_used = true;
  return WP_OK;
}

static int check_live(wp_handle* h, int32_t T, int32_t rank, int32_t dtype) {
  if (!rank_ok(rank)) return fail(h, WP_ERR_INVALID, "add_lora: unsupported rank %d (only 8/16/32/64)", rank);
  if (!dtype16(dtype)) return fail(h, WP_ERR_INVALID, "add_lora_packed: x/y must be fp16 or bf16");
  if (T < 0 || T > h->cfg.max_tokens) return fail(h, WP_ERR_INVALID, "add_lora: %d tokens outside [0, %d]", T, h->cfg.max_tokens);
  return WP_OK;
}

static int check_shrink_args(wp_handle* h, const void* x, int64_t x_ld, int32_t d_model, const void* wa_base,
                             int64_t wa_stride0, int32_t num_adapters) {
  if (d_model <= 0 || d_model % 8) return fail(h, WP_ERR_INVALID, "add_lora: d_model must be a positive multiple of 8");
  if (num_adapters < 1) return fail(h, WP_ERR_INVALID, "add_lora: num_adapters must be >= 1");
  if (!al16(x) || !al16(wa_base) || x_ld % 8 || x_ld < d_model || wa_stride0 % 8)
    return fail(h, WP_ERR_INVALID, "add_lora: x and wa_t_all need 16-byte aligned rows");
  return WP_OK;
}

static int check_expand_args(wp_handle* h, const void* y, int64_t y_ld, int32_t y_offset, int32_t out_features,
                             const void* wb_base, int64_t wb_stride0) {
  if (out_features <= 0 || out_features % 8)
    return fail(h, WP_ERR_INVALID, "add_lora: out_features must be a positive multiple of 8");
  if (y_offset < 0 || y_ld < y_offset + out_features)
    return fail(h, WP_ERR_INVALID, "add_lora: y slice [%d, %d) exceeds the row length %lld", y_offset,
                y_offset + out_features, static_cast<long long>(y_ld));
  if (!al16(wb_base) || wb_stride0 % 8 || (reinterpret_cast<uintptr_t>(y) & 1))
    return fail(h, WP_ERR_INVALID, "add_lora: wb_t_all needs 16-byte alignment and y 2-byte alignment");
  return WP_OK;
}

int wp_add_lora_shrink(wp_handle* h, void* H, const void* x, const void* wa_base, int64_t wa_stride0,
                       int32_t num_adapters, float scale, int32_t T, int32_t d_model, int32_t rank, int64_t x_ld,
                       int32_t dtype, void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "add_lora_shrink: NULL handle");
  int rc = check_live(h, T, rank, dtype);
  if (!rc) rc = check_shrink_args(h, x, x_ld, d_model, wa_base, wa_stride0, num_adapters);
  if (rc) return rc;
  if (!al16(H)) return fail(h, WP_ERR_INVALID, "add_lora_shrink: H must be 16-byte aligned");
  DeviceGuard dg(h->device);
  return do_apply(h, wp::kModeShrink, 0, h->d_live, h->d_live_num, T, rank, dtype, x, x_ld, d_model, wa_base,
                  wa_stride0, num_adapters, scale, nullptr, 0, 0, 0, nullptr, 0, static_cast<float*>(H),
                  static_cast<cudaStream_t>(stream_v));
}

int wp_add_lora_expand(wp_handle* h, void* y, const void* H, const void* wb_base, int64_t wb_stride0,
                       int32_t num_adapters, int32_t T, int32_t out_features, int32_t rank, int64_t y_ld,
                       int32_t y_offset, int32_t dtype, void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "add_lora_expand: NULL handle");
  int rc = check_live(h, T, rank, dtype);
  if (!rc) rc = check_expand_args(h, y, y_ld, y_offset, out_features, wb_base, wb_stride0);
  if (rc) return rc;
  if (num_adapters < 1) return fail(h, WP_ERR_INVALID, "add_lora_expand: num_adapters must be >= 1");
  if (!al16(H)) return fail(h, WP_ERR_INVALID, "add_lora_expand: H must be 16-byte aligned");
  DeviceGuard dg(h->device);
  // the B tensor map spans the whole stack (num_adapters), so every live
  // adapter id addresses its own B
  return do_apply(h, wp::kModeExpand, 0, h->d_live, h->d_live_num, T, rank, dtype, nullptr, 0, 0, nullptr, 0,
                  num_adapters, 0.f, y, y_ld, y_offset, out_features, wb_base, wb_stride0,
                  const_cast<float*>(static_cast<const float*>(H)), static_cast<cudaStream_t>(stream_v));
}

int wp_add_lora(wp_handle* h, void* y, const void* x, const void* wa_base, int64_t wa_stride0, const void* wb_base,
                int64_t wb_stride0, int32_t num_adapters, float scale, int32_t T, int32_t d_model,
                int32_t out_features, int32_t rank, int64_t x_ld, int64_t y_ld, int32_t y_offset, int32_t dtype,
                void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "add_lora: NULL handle");
  int rc = check_live(h, T, rank, dtype);
  if (!rc) rc = check_shrink_args(h, x, x_ld, d_model, wa_base, wa_stride0, num_adapters);
  if (!rc) rc = check_expand_args(h, y, y_ld, y_offset, out_features, wb_base, wb_stride0);
  if (rc) return rc;
  DeviceGuard dg(h->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (prefill_eligible(h, T, rank, d_model, out_features, y, y_ld, y_offset, stream)) {
    // the short runs on the decode kernel, then the long runs on the prefill
    // kernels, whose shrink runs beside it (disjoint rows)
    int rc = do_apply(h, wp::kModeFused, 0, h->d_short, h->d_short_num, T, rank, dtype, x, x_ld, d_model, wa_base,
                      wa_stride0, num_adapters, scale, y, y_ld, y_offset, out_features, wb_base, wb_stride0, nullptr,
                      stream);
    if (rc) return rc;
    return launch_prefill_call(h, T, rank, dtype, x, x_ld, d_model, wa_base, wa_stride0, num_adapters, scale, y, y_ld,
                               y_offset, out_features, wb_base, wb_stride0, true, stream);
  }
  return do_apply(h, wp::kModeFused, 0, h->d_live, h->d_live_num, T, rank, dtype, x, x_ld, d_model, wa_base,
                  wa_stride0, num_adapters, scale, y, y_ld, y_offset, out_features, wb_base, wb_stride0, nullptr,
                  stream);
}

// Several output slices that share x (vLLM's add_lora_packed_nslice: q/k/v,
// gate/up) in ONE clustered launch: slice s adds x . A_s^T . B_s^T into
// y[:, y_offsets[s] : y_offsets[s] + out_features]. Every slice has the same
// rank, d_model and out_features; the kernel treats (slice, segment) pairs as
// its work items, so the slices overlap instead of running back to back.
int wp_add_lora_slices(wp_handle* h, void* y, const void* x, int32_t nslices, const void* const* wa_bases,
                       const int64_t* wa_strides, const void* const* wb_bases, const int64_t* wb_strides,
                       const int32_t* y_offsets, int32_t num_adapters, float scale, int32_t T, int32_t d_model,
                       int32_t out_features, int32_t rank, int64_t x_ld, int64_t y_ld, int32_t dtype,
                       void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "add_lora_slices: NULL handle");
  if (nslices < 1 || nslices > wp::kMaxSlices)
    return fail(h, WP_ERR_INVALID, "add_lora_slices: %d slices outside [1, %d]", nslices, wp::kMaxSlices);
  if (!wa_bases || !wa_strides || !wb_bases || !wb_strides || !y_offsets)
    return fail(h, WP_ERR_INVALID, "add_lora_slices: NULL slice arrays");
  int rc = check_live(h, T, rank, dtype);
  for (int s = 0; !rc && s < nslices; ++s) {
    rc = check_shrink_args(h, x, x_ld, d_model, wa_bases[s], wa_strides[s], num_adapters);
    if (!rc) rc = check_expand_args(h, y, y_ld, y_offsets[s], out_features, wb_bases[s], wb_strides[s]);
  }
  if (rc) return rc;
  DeviceGuard dg(h->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (nslices == 1 || h->live_prefill)  // plain calls (prefill tables: per slice)
    for (int s = 0; s < nslices; ++s) {
      rc = wp_add_lora(h, y, x, wa_bases[s], wa_strides[s], wb_bases[s], wb_strides[s], num_adapters, scale, T,
                       d_model, out_features, rank, x_ld, y_ld, y_offsets[s], dtype, stream);
      if (rc) return rc;
    }
  if (nslices == 1 || h->live_prefill) return WP_OK;
  if (T == 0) return WP_OK;
  wp::ApplyArgs a{};
  a.segs = h->d_live;
  a.num_segs = h->d_live_num;
  a.plan = nullptr;  // the precomputed plan covers one slice only
  a.mode = wp::kModeFused;
  a.scale = scale;
  a.err = h->d_err;
  a.trace = h->trace_on ? h->d_trace[0] : nullptr;
  a.d = d_model;
  a.d_sliced = sliced(d_model) ? 1 : 0;
  a.nslices = nslices;
  const int64_t L = std::max<int32_t>(1, num_adapters);
  for (int i = 0; i < 3; ++i)
    if (!encode_rows_map(&a.tmap_x[i], dtype, x, d_model, T, x_ld, 8 << i))
      return fail(h, WP_ERR_CUDA, "add_lora_slices: cuTensorMapEncodeTiled(x) failed");
  a.y = y;
  a.y_ld = y_ld;
  a.o = out_features;
  a.o_sliced = sliced(out_features) ? 1 : 0;
  a.y_tma = al16(y) && (y_ld % 8 == 0);
  for (int s = 0; s < nslices; ++s) a.y_tma = a.y_tma && y_offsets[s] % 8 == 0;
  for (int s = 0; s < nslices; ++s) {
    CUtensorMap* am = s ? &a.tmap_a_x[s - 1] : &a.tmap_a;
    CUtensorMap* bm = s ? &a.tmap_b_x[s - 1] : &a.tmap_b;
    CUtensorMap* ym = s ? a.tmap_y_x[s - 1] : a.tmap_y;
    if (!encode_a_map(am, dtype, wa_bases[s], d_model, rank, L, wa_strides[s]))
      return fail(h, WP_ERR_CUDA, "add_lora_slices: cuTensorMapEncodeTiled(wa_t_all) failed");
    if (rank >= 16 && !encode_b_map(bm, dtype, wb_bases[s], out_features, rank, L, wb_strides[s]))
      return fail(h, WP_ERR_CUDA, "add_lora_slices: cuTensorMapEncodeTiled(wb_t_all) failed");
    for (int i = 0; a.y_tma && i < 3; ++i)
      if (!encode_rows_map(&ym[i], dtype, static_cast<const char*>(y) + static_cast<int64_t>(y_offsets[s]) * 2,
                           out_features, T, y_ld, 8 << i))
        return fail(h, WP_ERR_CUDA, "add_lora_slices: cuTensorMapEncodeTiled(y) failed");
    if (s == 0) {
      a.y_off = y_offsets[0];
      a.wb_base = wb_bases[0];
      a.wb_stride = wb_strides[0];
    } else {
      a.y_off_x[s - 1] = y_offsets[s];
      a.wb_base_x[s - 1] = wb_bases[s];
      a.wb_stride_x[s - 1] = wb_strides[s];
    }
  }
  const bool pdl = h->cfg.use_pdl != 0;
  a.prefetch_weights = !pdl || (h->cfg.prefetch_weights != 0 && !h->last_was_segmenter);
  a.prefetch_inputs = pdl && a.prefetch_weights && h->cfg.prefetch_inputs != 0 && !h->input_written && a.y_tma;
  h->input_written = false;
  int cluster = 1, grid = 1;
  apply_plan(h, dtype, rank, &cluster, &grid);
  a.split_len = round_up((std::max<int>(d_model, 1) + cluster - 1) / cluster, wp::kStageK);
  a.oslice = round_up((std::max<int>(out_features, 1) + cluster - 1) / cluster, wp::kStageCols);
  wp::LaunchCfg lc{grid, cluster, stream, pdl};
  cudaError_t e = wp::launch_apply(dtype, rank, a, lc);
  if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "add_lora_slices launch: %s", cudaGetErrorString(e));
  h->last_kernel = 1;
  ++h->launches;
  h->last_was_segmenter = false;
  return WP_OK;
}

int wp_note_input_write(wp_handle* h) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "note_input_write: NULL handle");
  h->input_written = true;
  return WP_OK;
}

// ---- tracing -------------------------------------------------------------------

int wp_trace_enable(wp_handle* h, int32_t enable) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "trace_enable: NULL handle");
  DeviceGuard dg(h->device);
  if (enable && !h->d_trace[0]) {
    const size_t n = static_cast<size_t>(grid_size(h)) * wp::kTraceSlots;
    for (int k = 0; k < 2; ++k) {
      WP_CUDA(h, cudaMalloc(&h->d_trace[k], n * sizeof(unsigned long long)));
      WP_CUDA(h, cudaMemset(h->d_trace[k], 0, n * sizeof(unsigned long long)));
    }
  }
  h->trace_on = enable != 0;
  return WP_OK;
}

int wp_trace_read(wp_handle* h, int32_t kernel, uint64_t* out, int32_t cap, int32_t* n) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "trace_read: NULL handle");
  if (kernel < 0 || kernel > 1 || !h->d_trace[kernel]) return fail(h, WP_ERR_INVALID, "trace_read: tracing is off");
  DeviceGuard dg(h->device);
  const int total = grid_size(h) * wp::kTraceSlots;
  if (n) *n = total;
  WP_CUDA(h, cudaDeviceSynchronize());
  if (out && cap > 0)
    WP_CUDA(h, cudaMemcpy(out, h->d_trace[kernel], sizeof(uint64_t) * std::min(cap, total), cudaMemcpyDeviceToHost));
  return WP_OK;
}

int wp_apply_plan(wp_handle* h, int32_t dtype, int32_t rank, int32_t* cluster, int32_t* grid) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "apply_plan: NULL handle");
  if (!rank_ok(rank) || !dtype16(dtype)) return fail(h, WP_ERR_INVALID, "apply_plan: bad rank or dtype");
  DeviceGuard dg(h->device);
  int c = 0, g = 0;
  apply_plan(h, dtype, rank, &c, &g);
  if (cluster) *cluster = c;
  if (grid) *grid = g;
  return WP_OK;
}

}  // extern "C"

// ---- tensor parallel ---------------------------------------------------------

// ---- row-parallel exchange over peer memory -----------------------------------

extern "C" int32_t wp_tp_mailbox_handle_bytes(void) { return static_cast<int32_t>(sizeof(cudaIpcMemHandle_t)); }

extern "C" int wp_tp_mailbox_create(wp_handle* h, int32_t rank, int32_t world, int32_t max_tokens, void* handle_out) {
  if (!h || !handle_out) return fail(h, WP_ERR_INVALID, "tp_mailbox_create: NULL argument");
  if (world < 2 || world > wp::kMaxTp || rank < 0 || rank >= world)
    return fail(h, WP_ERR_INVALID, "tp_mailbox_create: rank %d / world %d outside [2, %d] ranks", rank, world, wp::kMaxTp);
  if (max_tokens < 1 || max_tokens > h->cfg.max_tokens)
    return fail(h, WP_ERR_INVALID, "tp_mailbox_create: max_tokens %d outside [1, %d]", max_tokens, h->cfg.max_tokens);
  DeviceGuard dg(h->device);
  wp_tp_mailbox_close(h);
  const size_t bytes = wp::TpMail::bytes(world, max_tokens, max_tokens);
  WP_CUDA(h, cudaMalloc(&h->tp_mail_own, bytes));
  WP_CUDA(h, cudaMemset(h->tp_mail_own, 0, bytes));
  WP_CUDA(h, cudaMalloc(&h->d_tp_seq, 2 * sizeof(int)));
  WP_CUDA(h, cudaMemset(h->d_tp_seq, 0, 2 * sizeof(int)));
  cudaIpcMemHandle_t mh;
  WP_CUDA(h, cudaIpcGetMemHandle(&mh, h->tp_mail_own));
  std::memcpy(handle_out, &mh, sizeof(mh));
  h->mail_world = world;
  h->mail_rank = rank;
  h->mail_tmax = max_tokens;
  return WP_OK;
}

extern "C" int wp_tp_mailbox_open(wp_handle* h, const void* handles) {
  if (!h || !handles) return fail(h, WP_ERR_INVALID, "tp_mailbox_open: NULL argument");
  if (!h->tp_mail_own) return fail(h, WP_ERR_INVALID, "tp_mailbox_open: wp_tp_mailbox_create was not called");
  DeviceGuard dg(h->device);
  const char* hs = static_cast<const char*>(handles);
  for (int p = 0; p < h->mail_world; ++p) {
    if (p == h->mail_rank) {
      h->tp_mail[p] = static_cast<float*>(h->tp_mail_own);
      continue;
    }
    cudaIpcMemHandle_t mh;
    std::memcpy(&mh, hs + p * sizeof(mh), sizeof(mh));
    void* ptr = nullptr;
    WP_CUDA(h, cudaIpcOpenMemHandle(&ptr, mh, cudaIpcMemLazyEnablePeerAccess));
    h->tp_mail[p] = static_cast<float*>(ptr);
  }
  return WP_OK;
}

extern "C" int wp_tp_mailbox_close(wp_handle* h) {
  if (!h) return WP_OK;
  DeviceGuard dg(h->device);
  if (h->tp_mail_own || h->d_tp_seq) cudaDeviceSynchronize();
  for (int p = 0; p < wp::kMaxTp; ++p) {
    if (h->tp_mail[p] && p != h->mail_rank) cudaIpcCloseMemHandle(h->tp_mail[p]);
    h->tp_mail[p] = nullptr;
  }
  if (h->tp_mail_own) cudaFree(h->tp_mail_own);
  if (h->d_tp_seq) cudaFree(h->d_tp_seq);
  h->tp_mail_own = nullptr;
  h->d_tp_seq = nullptr;
  h->mail_world = 0;
  return WP_OK;
}

extern "C" int wp_add_lora_row_parallel(wp_handle* h, void* y, const void* x, const void* wa_base, int64_t wa_stride0,
                                        const void* wb_base, int64_t wb_stride0, int32_t num_adapters, float scale,
                                        int32_t T, int32_t d_shard, int32_t out_features, int32_t rank, int64_t x_ld,
                                        int64_t y_ld, int32_t y_offset, int32_t dtype, void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "add_lora_row_parallel: NULL handle");
  if (!h->tp_mail[h->mail_rank] || h->mail_world < 2)
    return fail(h, WP_ERR_INVALID, "add_lora_row_parallel: the peer mailboxes are not open");
  int rc = check_live(h, T, rank, dtype);
  if (!rc) rc = check_shrink_args(h, x, x_ld, d_shard, wa_base, wa_stride0, num_adapters);
  if (!rc) rc = check_expand_args(h, y, y_ld, y_offset, out_features, wb_base, wb_stride0);
  if (rc) return rc;
  if (T > h->mail_tmax) return fail(h, WP_ERR_INVALID, "add_lora_row_parallel: %d tokens exceed the mailbox (%d)", T, h->mail_tmax);
  if (!al16(y) || y_ld % 8 || y_offset % 8)
    return fail(h, WP_ERR_INVALID, "add_lora_row_parallel: y needs 16-byte aligned rows and column offset");
  DeviceGuard dg(h->device);
  h->tp_exchange = true;
  rc = do_apply(h, wp::kModeFused, 0, h->d_live, h->d_live_num, T, rank, dtype, x, x_ld, d_shard, wa_base, wa_stride0,
                num_adapters, scale, y, y_ld, y_offset, out_features, wb_base, wb_stride0, nullptr,
                static_cast<cudaStream_t>(stream_v));
  h->tp_exchange = false;
  return rc;
}

extern "C" int32_t wp_tp_unique_id_bytes(void) { return static_cast<int32_t>(sizeof(ncclUniqueId)); }

extern "C" int wp_tp_get_unique_id(void* id) {
  if (!id) return fail(nullptr, WP_ERR_INVALID, "tp_get_unique_id: NULL");
  ncclResult_t r = ncclGetUniqueId(static_cast<ncclUniqueId*>(id));
  if (r != ncclSuccess) return fail(nullptr, WP_ERR_NCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  return WP_OK;
}

extern "C" int wp_tp_init(wp_handle* h, const void* id, int32_t rank, int32_t world) {
  if (!h || !id) return fail(h, WP_ERR_INVALID, "tp_init: NULL argument");
  if (world < 1 || rank < 0 || rank >= world) return fail(h, WP_ERR_INVALID, "tp_init: bad rank %d / world %d", rank, world);
  DeviceGuard dg(h->device);
  if (h->comm) {
    ncclCommDestroy(h->comm);
    h->comm = nullptr;
  }
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = ncclCommInitRank(&h->comm, world, uid, rank);
  if (r != ncclSuccess) {
    h->comm = nullptr;
    return fail(h, WP_ERR_NCCL, "ncclCommInitRank: %s", ncclGetErrorString(r));
  }
  h->tp_rank = rank;
  h->tp_world = world;
  return WP_OK;
}

extern "C" int wp_tp_allreduce_f32(wp_handle* h, void* buf, int64_t n, void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "tp_allreduce: NULL handle");
  if (!h->comm) return fail(h, WP_ERR_INVALID, "tp_allreduce: wp_tp_init was not called");
  DeviceGuard dg(h->device);
  ncclResult_t r = ncclAllReduce(buf, buf, static_cast<size_t>(n), ncclFloat32, ncclSum, h->comm,
                                 static_cast<cudaStream_t>(stream_v));
  if (r != ncclSuccess) return fail(h, WP_ERR_NCCL, "ncclAllReduce: %s", ncclGetErrorString(r));
  h->last_was_segmenter = false;
  return WP_OK;
}

extern "C" int wp_tp_destroy(wp_handle* h) {
  if (!h) return WP_OK;
  if (h->comm) {
    DeviceGuard dg(h->device);
    ncclCommDestroy(h->comm);
    h->comm = nullptr;
  }
  return WP_OK;
}

// ---- adapter pool (live path over a pinned-host store) -------------------------
//
// The reference stages host-store adapters only for its registry path
// (StagingBufferPool, csrc/memory/staging_buffer.h:29-105; prefetch_adapter,
// csrc/pybind/warp_pipe_bindings.cpp:46-64), and its live DSAK path reads
// only device stacks (warp_pipe_r32.cu:263-269). The pool gives the live
// path the same store: a tenant's adapter for every LoRA projection of a
// model (one pinned host blob per adapter) is paged into one of num_slots
// GPU slots, and the slots of projection p form the stacked tensors the
// live apply takes (A_p at slot * slot_bytes + a_off[p], B_p likewise). The
// segmenter translates adapter ids to slots through a device map, so the
// apply kernels run unchanged.

struct wp_pool {
  wp_handle* h = nullptr;
  int32_t num_slots = 0, num_proj = 0, rank = 0, dtype = 0, max_adapters = 0;
  std::vector<int32_t> d, o;
  std::vector<int64_t> a_off, b_off;  // byte offsets of projection p inside a slot
  int64_t slot_bytes = 0;
  char* dev = nullptr;  // [num_slots][slot_bytes]
  std::unordered_map<int32_t, const void*> host;  // adapter id -> caller's pinned blob (slot layout)
  struct PSlot {
    int32_t adapter = -1;
    cudaEvent_t ready = nullptr;
    bool issued = false;
    bool pinned = false;  // held by wp_pool_prefetch until wp_pool_release
    uint64_t last_use = 0;  // step (prepare generation) that last read the slot; 0 = never
  };
  std::vector<PSlot> slots;
  std::vector<int32_t> map_host;  // adapter id -> slot (-1: not resident)
  int32_t* d_map = nullptr;
  int32_t* h_map[2] = {nullptr, nullptr};  // pinned upload buffers
  cudaEvent_t map_up[2] = {nullptr, nullptr};
  int map_buf = 0;
  cudaStream_t side = nullptr;  // copies
  // step_done[g % kRing] is recorded on the step stream when prepare(g + 1)
  // starts, i.e. after every kernel of step g was queued
  static constexpr int kRing = 8;
  cudaEvent_t step_done[kRing] = {};
  uint64_t gen = 0;  // steps prepared so far
  cudaStream_t last_stream = nullptr;
  int64_t copies = 0, bytes = 0;
};

namespace {

int pool_fail(wp_pool* p, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  if (p && p->h)
    p->h->err = buf;
  else
    g_err = buf;
  return code;
}

int pool_find(const wp_pool* p, int32_t id) {
  if (id < 0 || id >= p->max_adapters) return -1;
  return p->map_host[id];
}

// A slot for a new adapter: a free one, else the least recently used that is
// neither pinned nor read by the step being prepared or run (`busy_gen`).
int pool_victim(wp_pool* p, uint64_t busy_gen) {
  int best = -1;
  uint64_t best_use = ~0ull;
  for (int i = 0; i < p->num_slots; ++i) {
    const wp_pool::PSlot& s = p->slots[i];
    if (s.adapter < 0) return i;
    if (s.pinned || s.last_use >= busy_gen) continue;
    if (s.last_use < best_use) {
      best_use = s.last_use;
      best = i;
    }
  }
  return best;
}

// Copies adapter `id` into slot `si` on the side stream. A slot that a
// previous step read is overwritten only after that step's kernels (the side
// stream waits on the event recorded after them).
int pool_issue(wp_pool* p, int si, int32_t id) {
  wp_pool::PSlot& s = p->slots[si];
  if (s.adapter >= 0 && s.adapter < p->max_adapters) p->map_host[s.adapter] = -1;
  if (s.last_use > 0) {
    // step_done[j % kRing] holds the event of step j or of a later step
    // j + m * kRing (recorded further down the stream): waiting on it covers
    // every kernel of step j
    if (s.last_use >= p->gen) return pool_fail(p, WP_ERR_INVALID, "pool: slot %d is read by the current step", si);
    WP_CUDA(p->h, cudaStreamWaitEvent(p->side, p->step_done[s.last_use % wp_pool::kRing], 0));
  }
  WP_CUDA(p->h, cudaMemcpyAsync(p->dev + static_cast<int64_t>(si) * p->slot_bytes, p->host[id], p->slot_bytes,
                                cudaMemcpyHostToDevice, p->side));
  WP_CUDA(p->h, cudaEventRecord(s.ready, p->side));
  s.adapter = id;
  s.issued = true;
  s.pinned = false;
  p->map_host[id] = si;
  ++p->copies;
  p->bytes += p->slot_bytes;
  return WP_OK;
}

}  // namespace

extern "C" {

int wp_pool_create(wp_handle* h, int32_t num_slots, int32_t num_proj, int32_t rank, const int32_t* d,
                   const int32_t* o, int32_t dtype, int32_t max_adapters, wp_pool** out) {
  if (!h || !out) return fail(nullptr, WP_ERR_INVALID, "pool_create: NULL handle or output");
  if (num_slots < 1 || num_proj < 1 || !d || !o || max_adapters < 1 || !rank_ok(rank) || !dtype16(dtype))
    return fail(h, WP_ERR_INVALID, "pool_create: bad sizes, rank or dtype");
  DeviceGuard dg(h->device);
  auto p = std::make_unique<wp_pool>();
  p->h = h;
  p->num_slots = num_slots;
  p->num_proj = num_proj;
  p->rank = rank;
  p->dtype = dtype;
  p->max_adapters = max_adapters;
  int64_t off = 0;
  for (int i = 0; i < num_proj; ++i) {
    if (d[i] < 1 || o[i] < 1) return fail(h, WP_ERR_INVALID, "pool_create: projection %d has no size", i);
    p->d.push_back(d[i]);
    p->o.push_back(o[i]);
    p->a_off.push_back(off);
    off += (static_cast<int64_t>(rank) * d[i] * 2 + 255) / 256 * 256;
    p->b_off.push_back(off);
    off += (static_cast<int64_t>(o[i]) * rank * 2 + 255) / 256 * 256;
  }
  p->slot_bytes = off;
  cudaError_t e;
  if ((e = cudaMalloc(&p->dev, static_cast<size_t>(p->slot_bytes) * num_slots)) != cudaSuccess)
    return fail(h, WP_ERR_CUDA, "pool_create: %zu bytes of slots: %s", static_cast<size_t>(p->slot_bytes) * num_slots,
                cudaGetErrorString(e));
  cudaMemset(p->dev, 0, static_cast<size_t>(p->slot_bytes) * num_slots);
  if ((e = cudaMalloc(&p->d_map, sizeof(int32_t) * max_adapters)) != cudaSuccess)
    return fail(h, WP_ERR_CUDA, "pool_create: slot map: %s", cudaGetErrorString(e));
  cudaMemset(p->d_map, 0xff, sizeof(int32_t) * max_adapters);
  for (int b = 0; b < 2; ++b) {
    if ((e = cudaHostAlloc(&p->h_map[b], sizeof(int32_t) * max_adapters, cudaHostAllocDefault)) != cudaSuccess)
      return fail(h, WP_ERR_CUDA, "pool_create: map upload buffer: %s", cudaGetErrorString(e));
    cudaEventCreateWithFlags(&p->map_up[b], cudaEventDisableTiming);
  }
  for (auto& ev : p->step_done) cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  if ((e = cudaStreamCreateWithFlags(&p->side, cudaStreamNonBlocking)) != cudaSuccess)
    return fail(h, WP_ERR_CUDA, "pool_create: copy stream: %s", cudaGetErrorString(e));
  p->slots.resize(num_slots);
  for (auto& s : p->slots) cudaEventCreateWithFlags(&s.ready, cudaEventDisableTiming);
  p->map_host.assign(max_adapters, -1);
  *out = p.release();
  return WP_OK;
}

int wp_pool_destroy(wp_pool* p) {
  if (!p) return WP_OK;
  DeviceGuard dg(p->h->device);
  if (p->side) cudaStreamSynchronize(p->side);
  cudaDeviceSynchronize();
  for (auto& s : p->slots)
    if (s.ready) cudaEventDestroy(s.ready);
  for (auto& ev : p->step_done)
    if (ev) cudaEventDestroy(ev);
  for (int b = 0; b < 2; ++b) {
    if (p->h_map[b]) cudaFreeHost(p->h_map[b]);
    if (p->map_up[b]) cudaEventDestroy(p->map_up[b]);
  }
  cudaFree(p->d_map);
  cudaFree(p->dev);
  if (p->side) cudaStreamDestroy(p->side);
  delete p;
  return WP_OK;
}

int wp_pool_layout(wp_pool* p, int32_t proj, int64_t* a_off, int64_t* b_off, int64_t* slot_bytes) {
  if (!p || proj < 0 || proj >= p->num_proj) return fail(p ? p->h : nullptr, WP_ERR_INVALID, "pool_layout: bad projection");
  if (a_off) *a_off = p->a_off[proj];
  if (b_off) *b_off = p->b_off[proj];
  if (slot_bytes) *slot_bytes = p->slot_bytes;
  return WP_OK;
}

int wp_pool_stack(wp_pool* p, int32_t proj, void** wa, void** wb, int64_t* stride0) {
  if (!p || proj < 0 || proj >= p->num_proj) return fail(p ? p->h : nullptr, WP_ERR_INVALID, "pool_stack: bad projection");
  if (wa) *wa = p->dev + p->a_off[proj];
  if (wb) *wb = p->dev + p->b_off[proj];
  if (stride0) *stride0 = p->slot_bytes / 2;  // elements of the 16-bit type
  return WP_OK;
}

int wp_pool_register_host(wp_pool* p, int32_t adapter_id, const void* blob) {
  if (!p) return fail(nullptr, WP_ERR_INVALID, "pool_register_host: NULL pool");
  if (adapter_id < 0 || adapter_id >= p->max_adapters)
    return pool_fail(p, WP_ERR_INVALID, "pool_register_host: adapter id %d outside [0, %d)", adapter_id, p->max_adapters);
  if (!blob) return pool_fail(p, WP_ERR_INVALID, "pool_register_host: NULL blob");
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, blob) != cudaSuccess || at.type != cudaMemoryTypeHost) {
    cudaGetLastError();
    return pool_fail(p, WP_ERR_INVALID, "pool_register_host: the blob must be page-locked host memory");
  }
  // re-registering a resident adapter drops its slot copy
  const int si = pool_find(p, adapter_id);
  if (si >= 0 && !(p->slots[si].last_use >= p->gen && p->gen > 0)) {
    p->slots[si].adapter = -1;
    p->slots[si].issued = false;
    p->slots[si].pinned = false;
    p->map_host[adapter_id] = -1;
  }
  p->host[adapter_id] = blob;
  return WP_OK;
}

int wp_pool_evict(wp_pool* p, int32_t adapter_id) {
  if (!p) return fail(nullptr, WP_ERR_INVALID, "pool_evict: NULL pool");
  const int si = pool_find(p, adapter_id);
  if (si >= 0) {
    if (p->slots[si].last_use >= p->gen && p->gen > 0)
      return pool_fail(p, WP_ERR_INVALID, "pool_evict: adapter %d is read by the current step", adapter_id);
    p->slots[si].adapter = -1;
    p->slots[si].issued = false;
    p->slots[si].pinned = false;
    p->map_host[adapter_id] = -1;
  }
  p->host.erase(adapter_id);
  return WP_OK;
}

int32_t wp_pool_prefetch(wp_pool* p, int32_t adapter_id) {
  if (!p || p->host.find(adapter_id) == p->host.end()) return -1;
  DeviceGuard dg(p->h->device);
  int si = pool_find(p, adapter_id);
  if (si < 0) {
    si = pool_victim(p, p->gen);  // not a slot the current step reads
    if (si < 0) return -1;
    if (pool_issue(p, si, adapter_id) != WP_OK) return -1;
  }
  p->slots[si].pinned = true;
  return si;
}

int32_t wp_pool_is_ready(wp_pool* p, int32_t adapter_id) {
  if (!p) return 0;
  const int si = pool_find(p, adapter_id);
  if (si < 0 || !p->slots[si].issued) return 0;
  const cudaError_t e = cudaEventQuery(p->slots[si].ready);
  if (e == cudaErrorNotReady) cudaGetLastError();
  return e == cudaSuccess ? 1 : 0;
}

int wp_pool_release(wp_pool* p, int32_t adapter_id) {
  if (!p) return WP_OK;
  const int si = pool_find(p, adapter_id);
  if (si >= 0) p->slots[si].pinned = false;
  return WP_OK;
}

int wp_pool_prepare(wp_pool* p, const int32_t* ids, int32_t n, void* stream_v) {
  if (!p) return fail(nullptr, WP_ERR_INVALID, "pool_prepare: NULL pool");
  if (n < 0 || (n > 0 && !ids)) return pool_fail(p, WP_ERR_INVALID, "pool_prepare: bad id list");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  DeviceGuard dg(p->h->device);
  // the previous step's kernels are all queued before this point
  if (p->gen > 0) WP_CUDA(p->h, cudaEventRecord(p->step_done[p->gen % wp_pool::kRing], stream));
  ++p->gen;
  p->last_stream = stream;
  int misses = 0;
  std::vector<int> used;
  used.reserve(n);
  for (int i = 0; i < n; ++i) {
    const int32_t id = ids[i];
    if (id < 0) continue;  // tokens without an adapter
    if (p->host.find(id) == p->host.end())
      return pool_fail(p, WP_ERR_UNKNOWN_ADAPTER, "pool_prepare: adapter %d is not registered", id);
    int si = pool_find(p, id);
    if (si < 0) {
      si = pool_victim(p, p->gen);
      if (si < 0) return pool_fail(p, WP_ERR_CAPACITY, "pool_prepare: more adapters than free slots in one step");
      const int rc = pool_issue(p, si, id);
      if (rc != WP_OK) return rc;
      ++misses;
    }
    if (p->slots[si].last_use != p->gen) {
      p->slots[si].last_use = p->gen;
      used.push_back(si);
    }
  }
  // the step's kernels wait for every copy they read (no host sync)
  for (int si : used) WP_CUDA(p->h, cudaStreamWaitEvent(stream, p->slots[si].ready, 0));
  // slot map upload through a pinned double buffer
  const int ub = p->map_buf;
  p->map_buf ^= 1;
  WP_CUDA(p->h, cudaEventSynchronize(p->map_up[ub]));
  std::memcpy(p->h_map[ub], p->map_host.data(), sizeof(int32_t) * p->max_adapters);
  WP_CUDA(p->h, cudaMemcpyAsync(p->d_map, p->h_map[ub], sizeof(int32_t) * p->max_adapters, cudaMemcpyHostToDevice,
                                stream));
  WP_CUDA(p->h, cudaEventRecord(p->map_up[ub], stream));
  return misses;
}

int wp_pool_stats(wp_pool* p, int64_t* copies, int64_t* bytes, int32_t* resident) {
  if (!p) return fail(nullptr, WP_ERR_INVALID, "pool_stats: NULL pool");
  if (copies) *copies = p->copies;
  if (bytes) *bytes = p->bytes;
  if (resident) {
    int r = 0;
    for (const auto& s : p->slots) r += s.adapter >= 0 ? 1 : 0;
    *resident = r;
  }
  return WP_OK;
}

int wp_build_seg_bounds_pool(wp_handle* h, wp_pool* p, const void* idx, int32_t idx_dtype, int32_t T,
                             void* stream_v) {
  if (!h || !p || p->h != h) return fail(h, WP_ERR_INVALID, "build_seg_bounds_pool: NULL or foreign pool");
  if (idx_dtype != WP_DTYPE_I32 && idx_dtype != WP_DTYPE_I64)
    return fail(h, WP_ERR_INVALID, "build_seg_bounds_pool: token_lora_indices must be int32 or int64");
  if (T < 0) return fail(h, WP_ERR_INVALID, "build_seg_bounds_pool: negative token count");
  if (T > h->cfg.max_tokens) return WP_NOT_HANDLED;
  if (T > 0 && !idx) return fail(h, WP_ERR_INVALID, "build_seg_bounds_pool: NULL indices");
  DeviceGuard dg(h->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  if (h->plan_g == 0) {
    int c = 1, g = 1;
    apply_plan(h, WP_DTYPE_BF16, 32, &c, &g);
    h->plan_g = g / std::max(c, 1);
    h->plan_g4 = plan_clusters4(h);
  }
  cudaError_t e = wp::launch_seg_bounds(idx, idx_dtype, T, h->d_live, h->d_live_num, h->d_plan,
                                        h->plan_g | (h->plan_g4 << 16), h->d_run_starts, stream, p->d_map,
                                        p->max_adapters, h->d_err);
  if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "build_seg_bounds_pool launch: %s", cudaGetErrorString(e));
  h->live_prefill = false;
  ++h->launches;
  h->last_was_segmenter = true;
  return WP_OK;
}

}  // extern "C"

// ---- scheduler bridge ------------------------------------------------------------

namespace wp {
// One thread per adapter slot: the bridge is read through the device mapping
// of the host's page-locked copy, as the reference's bridge_ptr is.
__global__ void bridge_readback_kernel(const wp_bridge* b, float* out) {
  const uint32_t n = b->num_active_adapters < WP_BRIDGE_MAX ? b->num_active_adapters : WP_BRIDGE_MAX;
  const uint32_t i = threadIdx.x;
  if (i < n) out[i] = b->whittle_scores[i];
  if (i == 0) {
    out[n] = static_cast<float>(n);
    out[n + 1] = static_cast<float>(b->num_segments);
    out[n + 2] = static_cast<float>(b->step_id);
  }
}
}  // namespace wp

namespace {
int bridge_init(wp_handle* h) {
  if (h->bridge) return WP_OK;
  void* p = nullptr;
  WP_CUDA(h, cudaHostAlloc(&p, sizeof(wp_bridge), cudaHostAllocMapped));
  std::memset(p, 0, sizeof(wp_bridge));
  h->bridge = static_cast<wp_bridge*>(p);
  void* dp = nullptr;
  WP_CUDA(h, cudaHostGetDevicePointer(&dp, p, 0));
  h->d_bridge = static_cast<wp_bridge*>(dp);
  WP_CUDA(h, cudaMalloc(&h->d_bridge_out, sizeof(float) * (WP_BRIDGE_MAX + 3)));
  return WP_OK;
}
}  // namespace

extern "C" {

int wp_write_bridge(wp_handle* h, const wp_bridge* b) {
  if (!h || !b) return fail(h, WP_ERR_INVALID, "write_bridge: NULL handle or bridge");
  if (b->num_active_adapters > WP_BRIDGE_MAX)
    return fail(h, WP_ERR_INVALID, "write_bridge: num_active_adapters %u exceeds WP_MAX_ADAPTERS (%d)",
                b->num_active_adapters, WP_BRIDGE_MAX);
  DeviceGuard dg(h->device);
  const int rc = bridge_init(h);
  if (rc) return rc;
  std::memcpy(h->bridge, b, sizeof(wp_bridge));
  return WP_OK;
}

int wp_read_bridge(wp_handle* h, wp_bridge* out) {
  if (!h || !out) return fail(h, WP_ERR_INVALID, "read_bridge: NULL handle or output");
  if (!h->bridge) {
    std::memset(out, 0, sizeof(wp_bridge));
    return WP_OK;
  }
  std::memcpy(out, h->bridge, sizeof(wp_bridge));
  return WP_OK;
}

int wp_read_bridge_kernel(wp_handle* h, float* out, int32_t cap, int32_t* count) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "read_bridge_kernel: NULL handle");
  DeviceGuard dg(h->device);
  const int rc = bridge_init(h);
  if (rc) return rc;
  wp::bridge_readback_kernel<<<1, WP_BRIDGE_MAX>>>(h->d_bridge, h->d_bridge_out);
  WP_CUDA(h, cudaGetLastError());
  ++h->launches;
  WP_CUDA(h, cudaDeviceSynchronize());
  const uint32_t n = std::min<uint32_t>(h->bridge->num_active_adapters, WP_BRIDGE_MAX);
  if (count) *count = static_cast<int32_t>(n + 3);
  if (out && cap > 0)
    WP_CUDA(h, cudaMemcpy(out, h->d_bridge_out, sizeof(float) * std::min<int64_t>(cap, n + 3), cudaMemcpyDeviceToHost));
  return WP_OK;
}

}  // extern "C"
