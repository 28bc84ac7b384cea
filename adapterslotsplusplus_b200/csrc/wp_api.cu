// wp_api.cu -- host side of libwp_b200.so: the C ABI declared in
// include/wp_api.h. Owns the device segment tables, split-K workspaces, the
// adapter store (device tensors or the library's own pinned-host copies), the
// staging-slot pool with its private prefetch stream, and the optional NCCL
// communicator for tensor-parallel shrink partials.

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
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
  int* d_run_starts = nullptr;
  // registry table (build_segments): unsplit host copy + split device copy
  DevSeg* d_reg = nullptr;
  int* d_reg_num = nullptr;
  DevSeg* h_reg_stage = nullptr;  // pinned upload buffer (cap + 1 entries, count in the tail)
  cudaEvent_t reg_uploaded = nullptr;
  std::vector<wp_segment> reg_table;
  std::vector<DevSeg> reg_pieces;
  int reg_rank = 0;
  int reg_dtype = -1;

  // workspaces
  float* d_partial = nullptr;
  int64_t partial_floats = 0;
  uint32_t* d_counters = nullptr;
  float* d_live_h = nullptr;  // [max_tokens, 64] fp32 H of wp_add_lora
  int* d_err = nullptr;

  // store + slots
  std::unordered_map<int32_t, Adapter> store;
  std::vector<Slot> slots;
  void* slot_pool = nullptr;
  cudaStream_t prefetch_stream = nullptr;
  cudaEvent_t caller_ready = nullptr;  // caller-stream point the prefetch waits on
  cudaEvent_t registry_done = nullptr;  // after the latest registry kernels
  bool registry_used = false;
  uint64_t generation = 0;

  // launch bookkeeping
  int64_t launches = 0;
  bool last_was_segmenter = false;

  // tensor parallel
  ncclComm_t comm = nullptr;
  int tp_rank = 0, tp_world = 1;
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

// Split-K plan for shrink: splits of d, each a multiple of the stage width.
void shrink_plan(const wp_handle* h, int d, int T, int rank, int* nsplit, int* split_len) {
  const int kc = wp::shrink_chunk_k(rank);
  int len = std::max(512, ((d + 15) / 16 + kc - 1) / kc * kc);
  int ns = (d + len - 1) / len;
  const int64_t plane = static_cast<int64_t>(h->cfg.max_tokens) * rank;
  const int64_t max_planes = plane > 0 ? h->partial_floats / plane : 1;
  while (ns > 1 && ns > max_planes) {
    len += kc;
    ns = (d + len - 1) / len;
  }
  (void)T;
  *nsplit = ns;
  *split_len = len;
}

int grid_size(const wp_handle* h) { return h->num_sms * std::max(1, h->cfg.ctas_per_sm); }

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

int wp_rank_supported(int32_t rank) { return rank_ok(rank) ? 1 : 0; }

int64_t wp_kernel_launch_count(const wp_handle* h) { return h ? h->launches : 0; }

int wp_create(const wp_config* cfg_in, wp_handle** out) {
  if (!out) return fail(nullptr, WP_ERR_INVALID, "wp_create: out is NULL");
  *out = nullptr;
  wp_config cfg{};
  if (cfg_in) cfg = *cfg_in;
  if (cfg.max_tokens <= 0) cfg.max_tokens = 16384;
  if (cfg.num_staging_slots < 0) cfg.num_staging_slots = 0;
  if (cfg.slot_bytes <= 0) cfg.slot_bytes = static_cast<int64_t>(2) * 64 * 16384 * 2;
  cfg.slot_bytes = (cfg.slot_bytes + 255) / 256 * 256;
  if (cfg.ctas_per_sm <= 0) cfg.ctas_per_sm = 1;

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
  if ((e = cudaMalloc(&h->d_live_num, sizeof(int) * 4)) != cudaSuccess) return bail("live count", e);
  if ((e = cudaMalloc(&h->d_run_starts, sizeof(int) * cap)) != cudaSuccess) return bail("run starts", e);
  if ((e = cudaMalloc(&h->d_reg, sizeof(DevSeg) * (cap + 1))) != cudaSuccess) return bail("registry table", e);
  if ((e = cudaMalloc(&h->d_reg_num, sizeof(int) * 4)) != cudaSuccess) return bail("registry count", e);
  if ((e = cudaHostAlloc(&h->h_reg_stage, sizeof(DevSeg) * (cap + 1), cudaHostAllocDefault)) != cudaSuccess)
    return bail("registry upload buffer", e);
  // Split-K partials: up to 16 planes of [max_tokens, 64] fp32.
  h->partial_floats = static_cast<int64_t>(16) * cap * 64;
  if ((e = cudaMalloc(&h->d_partial, sizeof(float) * h->partial_floats)) != cudaSuccess) return bail("partials", e);
  if ((e = cudaMalloc(&h->d_counters, sizeof(uint32_t) * cap)) != cudaSuccess) return bail("counters", e);
  if ((e = cudaMalloc(&h->d_err, sizeof(int) * 4)) != cudaSuccess) return bail("error word", e);
  if ((e = cudaMalloc(&h->d_live_h, sizeof(float) * static_cast<size_t>(cap) * 64)) != cudaSuccess)
    return bail("H scratch", e);
  cudaMemset(h->d_live_num, 0, sizeof(int) * 4);
  cudaMemset(h->d_reg_num, 0, sizeof(int) * 4);
  cudaMemset(h->d_counters, 0, sizeof(uint32_t) * cap);
  cudaMemset(h->d_err, 0, sizeof(int) * 4);
  if ((e = cudaStreamCreateWithFlags(&h->prefetch_stream, cudaStreamNonBlocking)) != cudaSuccess)
    return bail("prefetch stream", e);
  cudaEventCreateWithFlags(&h->reg_uploaded, cudaEventDisableTiming);
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
  if (h->prefetch_stream) cudaStreamSynchronize(h->prefetch_stream);
  cudaDeviceSynchronize();
  for (auto& kv : h->store) free_adapter(kv.second);
  for (auto& s : h->slots)
    if (s.ready) cudaEventDestroy(s.ready);
  if (h->slot_pool) cudaFree(h->slot_pool);
  cudaFree(h->d_live);
  cudaFree(h->d_live_num);
  cudaFree(h->d_run_starts);
  cudaFree(h->d_reg);
  cudaFree(h->d_reg_num);
  if (h->h_reg_stage) cudaFreeHost(h->h_reg_stage);
  cudaFree(h->d_partial);
  cudaFree(h->d_counters);
  cudaFree(h->d_err);
  cudaFree(h->d_live_h);
  if (h->reg_uploaded) cudaEventDestroy(h->reg_uploaded);
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
    // a kernel that gave up may have left split-K counters raised
    WP_CUDA(h, cudaMemset(h->d_counters, 0, sizeof(uint32_t) * h->cfg.max_tokens));
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
    for (int p = 0; p < count; p += wp::kSegTokens) {
      DevSeg s;
      s.adapter_id = ids[i];
      s.token_start = start + p;
      s.token_count = std::min(wp::kSegTokens, count - p);
      s.alpha = ad.alpha;
      s.a = pa;
      s.b = pb;
      pieces.push_back(s);
    }
  }
  if (static_cast<int>(pieces.size()) > h->cfg.max_tokens)
    return fail(h, WP_ERR_CAPACITY, "build_segments: %zu pieces exceed the table capacity", pieces.size());
  for (int si : wait_slots) WP_CUDA(h, cudaStreamWaitEvent(stream, h->slots[si].ready, 0));

  // upload through the pinned buffer (the previous upload must have left it)
  WP_CUDA(h, cudaEventSynchronize(h->reg_uploaded));
  const int np = static_cast<int>(pieces.size());
  if (np) std::memcpy(h->h_reg_stage, pieces.data(), sizeof(DevSeg) * np);
  int* cnt = reinterpret_cast<int*>(h->h_reg_stage + h->cfg.max_tokens);
  *cnt = np;
  if (np) WP_CUDA(h, cudaMemcpyAsync(h->d_reg, h->h_reg_stage, sizeof(DevSeg) * np, cudaMemcpyHostToDevice, stream));
  WP_CUDA(h, cudaMemcpyAsync(h->d_reg_num, cnt, sizeof(int), cudaMemcpyHostToDevice, stream));
  WP_CUDA(h, cudaEventRecord(h->reg_uploaded, stream));
  h->reg_table.swap(table);
  h->reg_pieces.swap(pieces);
  h->reg_rank = rank;
  h->reg_dtype = dtype;
  h->last_was_segmenter = false;
  return WP_OK;
}

int wp_build_seg_bounds(wp_handle* h, const void* idx, int32_t idx_dtype, int32_t T, void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "build_seg_bounds: NULL handle");
  if (idx_dtype != WP_DTYPE_I32 && idx_dtype != WP_DTYPE_I64)
    return fail(h, WP_ERR_INVALID, "build_seg_bounds: token_lora_indices must be int32 or int64");
  if (T < 0) return fail(h, WP_ERR_INVALID, "build_seg_bounds: negative token count");
  if (T > h->cfg.max_tokens) return WP_NOT_HANDLED;
  if (T > 0 && !idx) return fail(h, WP_ERR_INVALID, "build_seg_bounds: NULL indices");
  DeviceGuard dg(h->device);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  cudaError_t e = wp::launch_seg_bounds(idx, idx_dtype, T, h->d_live, h->d_live_num, h->d_run_starts, stream);
  if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "build_seg_bounds launch: %s", cudaGetErrorString(e));
  ++h->launches;
  h->last_was_segmenter = true;
  return WP_OK;
}

int wp_read_seg_table(wp_handle* h, int32_t which, wp_segment* out, int32_t cap, int32_t* num) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "read_seg_table: NULL handle");
  DeviceGuard dg(h->device);
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

static int do_shrink(wp_handle* h, const void* x, int64_t x_ld, float* H, const DevSeg* segs, const int* nseg,
                     const void* wa, int64_t wa_stride, float scale, int registry, int T, int d, int r, int dtype,
                     cudaStream_t stream) {
  wp::ShrinkArgs a{};
  a.x = x;
  a.x_ld = x_ld;
  a.h = H;
  a.partial = h->d_partial;
  a.counters = h->d_counters;
  a.segs = segs;
  a.num_segs = nseg;
  a.wa_base = wa;
  a.wa_stride = wa_stride;
  a.scale = scale;
  a.registry = registry;
  a.d = d;
  shrink_plan(h, d, T, r, &a.nsplit, &a.split_len);
  a.cap_t = h->cfg.max_tokens;
  a.err = h->d_err;
  wp::LaunchCfg lc{grid_size(h), stream, h->cfg.use_pdl != 0 && !h->last_was_segmenter};
  cudaError_t e = wp::launch_shrink(dtype, r, a, lc);
  if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "shrink launch: %s", cudaGetErrorString(e));
  ++h->launches;
  h->last_was_segmenter = false;
  return WP_OK;
}

static int do_expand(wp_handle* h, void* y, int64_t y_ld, int y_off, const float* H, const DevSeg* segs,
                     const int* nseg, const void* wb, int64_t wb_stride, int registry, int o, int r, int dtype,
                     cudaStream_t stream) {
  wp::ExpandArgs a{};
  a.h = H;
  a.y = y;
  a.y_ld = y_ld;
  a.y_off = y_off;
  a.segs = segs;
  a.num_segs = nseg;
  a.wb_base = wb;
  a.wb_stride = wb_stride;
  a.registry = registry;
  a.o = o;
  const int W = wp::expand_chunk_cols(r);
  a.n_ochunks = (o + W - 1) / W;
  a.y_bulk = al16(y) && (y_ld % 8 == 0) && (y_off % 8 == 0);
  a.err = h->d_err;
  wp::LaunchCfg lc{grid_size(h), stream, h->cfg.use_pdl != 0 && !h->last_was_segmenter};
  cudaError_t e = wp::launch_expand(dtype, r, a, lc);
  if (e != cudaSuccess) return fail(h, WP_ERR_CUDA, "expand launch: %s", cudaGetErrorString(e));
  ++h->launches;
  h->last_was_segmenter = false;
  return WP_OK;
}

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
  int rc = do_shrink(h, X, d_model, static_cast<float*>(H), h->d_reg, h->d_reg_num, nullptr, 0, 0.f, 1, T,
                     d_model, rank, dtype, stream);
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
  int rc = do_expand(h, Y, out_features, 0, static_cast<const float*>(H), h->d_reg, h->d_reg_num, nullptr, 0, 1,
                     out_features, rank, dtype, stream);
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

int wp_add_lora_shrink(wp_handle* h, void* H, const void* x, const void* wa_base, int64_t wa_stride0, float scale,
                       int32_t T, int32_t d_model, int32_t rank, int64_t x_ld, int32_t dtype, void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "add_lora_shrink: NULL handle");
  int rc = check_live(h, T, rank, dtype);
  if (rc) return rc;
  if (d_model <= 0 || d_model % 8) return fail(h, WP_ERR_INVALID, "add_lora: d_model must be a positive multiple of 8");
  if (!al16(x) || !al16(wa_base) || !al16(H) || x_ld % 8 || wa_stride0 % 8)
    return fail(h, WP_ERR_INVALID, "add_lora: x, wa_t_all and H need 16-byte aligned rows");
  DeviceGuard dg(h->device);
  return do_shrink(h, x, x_ld, static_cast<float*>(H), h->d_live, h->d_live_num, wa_base, wa_stride0, scale, 0, T,
                   d_model, rank, dtype, static_cast<cudaStream_t>(stream_v));
}

int wp_add_lora_expand(wp_handle* h, void* y, const void* H, const void* wb_base, int64_t wb_stride0, int32_t T,
                       int32_t out_features, int32_t rank, int64_t y_ld, int32_t y_offset, int32_t dtype,
                       void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "add_lora_expand: NULL handle");
  int rc = check_live(h, T, rank, dtype);
  if (rc) return rc;
  if (out_features <= 0 || out_features % 8)
    return fail(h, WP_ERR_INVALID, "add_lora: out_features must be a positive multiple of 8");
  if (y_offset < 0 || y_ld < y_offset + out_features)
    return fail(h, WP_ERR_INVALID, "add_lora: y slice [%d, %d) exceeds the row length %lld", y_offset,
                y_offset + out_features, static_cast<long long>(y_ld));
  if (!al16(wb_base) || !al16(H) || wb_stride0 % 8 || (reinterpret_cast<uintptr_t>(y) & 1))
    return fail(h, WP_ERR_INVALID, "add_lora: wb_t_all and H need 16-byte alignment");
  DeviceGuard dg(h->device);
  return do_expand(h, y, y_ld, y_offset, static_cast<const float*>(H), h->d_live, h->d_live_num, wb_base,
                   wb_stride0, 0, out_features, rank, dtype, static_cast<cudaStream_t>(stream_v));
}

}  // extern "C"

extern "C" int wp_add_lora(wp_handle* h, void* y, const void* x, const void* wa_base, int64_t wa_stride0,
                           const void* wb_base, int64_t wb_stride0, float scale, int32_t T, int32_t d_model,
                           int32_t out_features, int32_t rank, int64_t x_ld, int64_t y_ld, int32_t y_offset,
                           int32_t dtype, void* stream_v) {
  if (!h) return fail(nullptr, WP_ERR_INVALID, "add_lora: NULL handle");
  DeviceGuard dg(h->device);
  float* H = h->d_live_h;
  int rc = wp_add_lora_shrink(h, H, x, wa_base, wa_stride0, scale, T, d_model, rank, x_ld, dtype, stream_v);
  if (rc) return rc;
  return wp_add_lora_expand(h, y, H, wb_base, wb_stride0, T, out_features, rank, y_ld, y_offset, dtype, stream_v);
}

// ---- tensor parallel ---------------------------------------------------------

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
