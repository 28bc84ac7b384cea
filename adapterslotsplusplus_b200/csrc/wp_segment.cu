// wp_segment.cu -- device segmenter: token -> adapter id vector to the
// segment table, once per step, without a host sync.
//
// Output contract (bit-exact with build_seg_bounds_kernel,
// csrc/kernels/warp_pipe_r32.cu:461-512 of the reference): walk the ids in
// token order; a run starts at i == 0 or where idx[i] != idx[i-1]; runs with
// id < 0 are dropped; every other run [s, e) becomes ceil((e-s)/32) entries
// (id, s + 32*j, min(32, e - s - 32*j)); entries are ordered by token
// position; num_segments is their count.
//
// Design: one CTA of 1024 threads walks the tokens in 1024-wide tiles with
// two block-wide prefix sums. Pass 1 compacts run-start positions into
// `run_starts` (a device workspace), pass 2 turns run k into its piece count
// (its length is run_starts[k+1] - run_starts[k]) and scatters the pieces at
// the exclusive prefix of the counts. Work is O(T) with no serial scan of a
// run, so a 4096-token prefill run costs no more than 4096 one-token runs.
// The reference's cap of 256 tokens (one thread per token) is lifted: T is
// bounded only by the caller's table capacity.

#include <cuda_runtime.h>
#include <stdint.h>

#include "wp_internal.h"

namespace wp {

constexpr int kSegThreads = 1024;

// Block-wide exclusive scan of one int per thread; *total receives the sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_buf, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += n;
  }
  if (lane == 31) warp_buf[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_buf[lane];  // 32 warps in a 1024-thread block
    int wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += n;
    }
    warp_buf[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) warp_buf[32] = wi;
  }
  __syncthreads();
  const int excl = warp_buf[warp] + incl - v;
  *total = warp_buf[32];
  __syncthreads();  // warp_buf is reused by the next call
  return excl;
}

// Pass 3: the clustered apply kernel's per-cluster assignment for G
// clusters (ClusterPlan). Segments are ranked by decreasing token count
// (ties by position); fewer segments than clusters: position p of the
// first `helpers` (at most kPlanMaxHelpers) goes to clusters 2p and 2p + 1
// (output-column halves), the rest to one cluster each after them; more: round r gives cluster c the segment
// at position r*G + c (r*G + G-1-c on odd rounds).
__device__ void write_cluster_plan(const DevSeg* segs, int nseg, ClusterPlan* plan, int G) {
  __shared__ int order[kPlanMaxSegs];
  const int tid = threadIdx.x;
  int mode = 0;
  if (G > 1 && G <= kPlanMaxClusters && nseg > 0 && nseg <= kPlanMaxSegs && nseg != G &&
      (nseg + G - 1) / G <= kPlanRounds)
    mode = nseg < G ? 1 : 2;
  const int helpers = mode == 1 ? min(min(nseg, G - nseg), kPlanMaxHelpers) : 0;
  if (mode) {
    if (tid < nseg) {
      const int ct = segs[tid].token_count;
      int p = 0;
      for (int j = 0; j < nseg; ++j) {
        const int cj = segs[j].token_count;
        p += (cj > ct || (cj == ct && j < tid)) ? 1 : 0;
      }
      order[p] = tid;
    }
    __syncthreads();
    for (int c = tid; c < G; c += kSegThreads) {
      plan->half[c] = -1;
      int n = 0;
      if (mode == 1) {
        // the helper pairs of the largest segments take the lowest
        // clusters, which the hardware dispatches first; the whole segments
        // follow in decreasing size
        const int V = nseg + helpers;
        if (c < V) {
          const bool pair = c < 2 * helpers;
          const int pos = pair ? c >> 1 : c - helpers;
          plan->half[c] = pair ? (c & 1) : -1;
          plan->seg[c] = segs[order[pos]];
          n = 1;
        }
      } else {
        // snake dealing whose last (partial) round runs forward, so the
        // clusters holding one segment more are the lowest ones
        const int rounds = (nseg + G - 1) / G;
        for (int r = 0; r < kPlanRounds; ++r) {
          const int p = r * G + (((rounds - 1 - r) & 1) ? G - 1 - c : c);
          if (p < nseg) {
            plan->seg[r * G + c] = segs[order[p]];
            n = r + 1;
          }
        }
      }
      plan->count[c] = n;
    }
  }
  __syncthreads();
  if (tid == 0) plan->hdr = make_int4(mode, nseg, G, helpers);
}

// slot_map (optional): the adapter pool's device map from adapter id to the
// slot holding it (-1: not resident); table entries then carry the slot,
// and a run whose adapter is not resident is dropped with kErrBadSegment
// raised in *err. Runs are found on the original ids either way.
// pf (optional, prefill mode): besides the full table, runs of at least
// pf->min_run tokens become tiles of kPrefillTile tokens in pf->tiles, and
// the pieces of the other runs a second table pf->short_segs (in token
// order) -- the prefill kernels take the first, the decode kernel the second.
template <typename I>
__global__ void __launch_bounds__(kSegThreads, 1)
    seg_bounds_kernel(const I* __restrict__ idx, int T, DevSeg* __restrict__ segs, int* __restrict__ num_segs,
                      int* __restrict__ run_starts, ClusterPlan* __restrict__ plan, int plan_g,
                      const int* __restrict__ slot_map, int map_size, int* err, PrefillTables pf) {
  __shared__ int warp_buf[33];
  const int tid = threadIdx.x;

  // Pass 1: positions where a run starts, compacted in token order.
  int nruns = 0;
  for (int base = 0; base < T; base += kSegThreads) {
    const int i = base + tid;
    int flag = 0;
    if (i < T) flag = (i == 0) || (idx[i] != idx[i - 1]);
    int total;
    const int pos = block_exclusive_scan(flag, warp_buf, &total);
    if (flag) run_starts[nruns + pos] = i;
    nruns += total;
  }
  __syncthreads();  // run_starts written by other threads of this block

  // Pass 2: each run -> ceil(len / 32) pieces, skipping id < 0.
  int nseg = 0, nshort = 0, ntiles = 0;
  for (int base = 0; base < nruns; base += kSegThreads) {
    const int k = base + tid;
    int pieces = 0, start = 0, len = 0;
    int32_t id = -1;
    if (k < nruns) {
      start = run_starts[k];
      const int end = (k + 1 < nruns) ? run_starts[k + 1] : T;
      len = end - start;
      const I raw = idx[start];
      if (raw >= 0) {
        id = static_cast<int32_t>(raw);
        if (slot_map) {
          id = raw < static_cast<I>(map_size) ? __ldcg(slot_map + raw) : -1;
          if (id < 0 && err) atomicOr(err, 2);  // kErrBadSegment: adapter not resident
        }
        if (id >= 0) pieces = (len + kSegTokens - 1) / kSegTokens;
      }
    }
    int total;
    const int slot = nseg + block_exclusive_scan(pieces, warp_buf, &total);
    for (int j = 0; j < pieces; ++j) {
      DevSeg s;
      s.adapter_id = id;
      s.token_start = start + j * kSegTokens;
      s.token_count = min(kSegTokens, len - j * kSegTokens);
      s.alpha = 0.f;
      s.a = nullptr;
      s.b = nullptr;
      segs[slot + j] = s;
    }
    nseg += total;
    if (pf.tiles) {
      const bool longrun = pieces > 0 && len >= pf.min_run;
      const int tl = longrun ? (len + kPrefillTile - 1) / kPrefillTile : 0;
      const int sp = longrun ? 0 : pieces;
      int tt, ts;
      const int tslot = ntiles + block_exclusive_scan(tl, warp_buf, &tt);
      const int sslot = nshort + block_exclusive_scan(sp, warp_buf, &ts);
      for (int j = 0; j < tl; ++j) {
        DevSeg s;
        s.adapter_id = id;
        s.token_start = start + j * kPrefillTile;
        s.token_count = min(kPrefillTile, len - j * kPrefillTile);
        s.alpha = 0.f;
        s.a = nullptr;
        s.b = nullptr;
        pf.tiles[tslot + j] = s;
      }
      for (int j = 0; j < sp; ++j) pf.short_segs[sslot + j] = segs[slot + j];
      ntiles += tt;
      nshort += ts;
    }
  }
  if (tid == 0) {
    *num_segs = nseg;
    if (pf.tiles) {
      *pf.tiles_num = ntiles;
      *pf.short_num = nshort;
    }
  }
  if (plan) {
    // plan_g: clusters of the common launch (low 16 bits) and, when nonzero,
    // of the clusters-of-4 launch of few-segment calls (high bits; plan + 1)
    __syncthreads();  // the table (global memory, written by this block) is complete
    write_cluster_plan(segs, nseg, plan, plan_g & 0xffff);
    if (plan_g >> 16) {
      __syncthreads();
      write_cluster_plan(segs, nseg, plan + 1, plan_g >> 16);
    }
  }
}

cudaError_t launch_seg_bounds(const void* idx, int idx_dtype, int T, DevSeg* segs, int* num_segs, ClusterPlan* plan,
                              int plan_g, int* run_starts, cudaStream_t stream, const int* slot_map, int map_size,
                              int* err, PrefillTables pf) {
  if (idx_dtype == 4) {
    seg_bounds_kernel<int64_t><<<1, kSegThreads, 0, stream>>>(static_cast<const int64_t*>(idx), T, segs, num_segs,
                                                               run_starts, plan, plan_g, slot_map, map_size, err, pf);
  } else {
    seg_bounds_kernel<int32_t><<<1, kSegThreads, 0, stream>>>(static_cast<const int32_t*>(idx), T, segs, num_segs,
                                                               run_starts, plan, plan_g, slot_map, map_size, err, pf);
  }
  return cudaGetLastError();
}

}  // namespace wp

// ---------------------------------------------------------------------------
// Allocation-free variant of the segmenter.
//
// Some callers cannot allocate device memory at all: a plugin that runs inside
// another inference framework's memory plan, or code that must not call
// cudaMalloc because it synchronises the device and bypasses the host
// framework's allocator. Such a caller cannot create a wp_handle (wp_create
// allocates the tables), so this entry point takes the output table from the
// caller and keeps its one scratch buffer -- the compacted run starts -- in a
// fixed array in the library's own device memory image.

// Records the message returned by wp_last_error(NULL) (defined in wp_api.cu).
extern "C" int wp_set_global_error(int code, const char* msg);
static int wp_noalloc_fail(int code, const char* msg) { return wp_set_global_error(code, msg); }

namespace {

constexpr int kNoAllocMaxTokens = 65536;  // 256 KB of run starts per device
__device__ __align__(256) int g_seg_scratch[kNoAllocMaxTokens];

// Same algorithm as seg_bounds_kernel, writing (adapter_id, token_start,
// token_count) triples of int32 to the caller's table.
template <typename I>
__global__ void __launch_bounds__(wp::kSegThreads, 1)
    seg_bounds_triples_kernel(const I* __restrict__ idx, int T, int32_t* __restrict__ table, int* __restrict__ num,
                              int* __restrict__ run_starts) {
  __shared__ int warp_buf[33];
  const int tid = threadIdx.x;
  int nruns = 0;
  for (int base = 0; base < T; base += wp::kSegThreads) {
    const int i = base + tid;
    int flag = 0;
    if (i < T) flag = (i == 0) || (idx[i] != idx[i - 1]);
    int total;
    const int pos = wp::block_exclusive_scan(flag, warp_buf, &total);
    if (flag) run_starts[nruns + pos] = i;
    nruns += total;
  }
  __syncthreads();
  int nseg = 0;
  for (int base = 0; base < nruns; base += wp::kSegThreads) {
    const int k = base + tid;
    int pieces = 0, start = 0, len = 0;
    int32_t id = -1;
    if (k < nruns) {
      start = run_starts[k];
      const int end = (k + 1 < nruns) ? run_starts[k + 1] : T;
      len = end - start;
      const I raw = idx[start];
      if (raw >= 0) {
        id = static_cast<int32_t>(raw);
        pieces = (len + wp::kSegTokens - 1) / wp::kSegTokens;
      }
    }
    int total;
    const int slot = nseg + wp::block_exclusive_scan(pieces, warp_buf, &total);
    for (int j = 0; j < pieces; ++j) {
      int32_t* e = table + 3 * (slot + j);
      e[0] = id;
      e[1] = start + j * wp::kSegTokens;
      e[2] = min(wp::kSegTokens, len - j * wp::kSegTokens);
    }
    nseg += total;
  }
  if (tid == 0) *num = nseg;
}

// Device address of g_seg_scratch, looked up once per device.
int* g_scratch_ptr[64] = {nullptr};

}  // namespace

extern "C" int wp_seg_bounds_noalloc_max_tokens(void) { return kNoAllocMaxTokens; }

// Declared in include/wp_api.h. The first call on a device looks up the
// scratch array's device address (cudaGetSymbolAddress, with that device
// current); make that first call before any stream capture. Calls on one
// device share the scratch array: calls that overlap on the GPU (different
// streams, no ordering between them) race on it.
extern "C" int wp_build_seg_bounds_noalloc(const void* token_lora_indices, int32_t idx_dtype, int32_t T,
                                           int32_t* out_table, int32_t* out_num, void* stream) {
  if (idx_dtype != 3 && idx_dtype != 4) return wp_noalloc_fail(-1, "build_seg_bounds_noalloc: ids must be int32 or int64");
  if (T < 0) return wp_noalloc_fail(-1, "build_seg_bounds_noalloc: negative token count");
  if (T > kNoAllocMaxTokens)
    return wp_noalloc_fail(-4, "build_seg_bounds_noalloc: T exceeds the fixed scratch of 65536 tokens");
  if (!out_num || (T > 0 && (!token_lora_indices || !out_table)))
    return wp_noalloc_fail(-1, "build_seg_bounds_noalloc: NULL pointer");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return wp_noalloc_fail(-2, "build_seg_bounds_noalloc: no current CUDA device");
  if (!g_scratch_ptr[dev]) {
    int* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_seg_scratch);
    if (e != cudaSuccess || !p) return wp_noalloc_fail(-2, "build_seg_bounds_noalloc: cudaGetSymbolAddress failed");
    g_scratch_ptr[dev] = p;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (idx_dtype == 4)
    seg_bounds_triples_kernel<int64_t><<<1, wp::kSegThreads, 0, s>>>(static_cast<const int64_t*>(token_lora_indices),
                                                                      T, out_table, out_num, g_scratch_ptr[dev]);
  else
    seg_bounds_triples_kernel<int32_t><<<1, wp::kSegThreads, 0, s>>>(static_cast<const int32_t*>(token_lora_indices),
                                                                      T, out_table, out_num, g_scratch_ptr[dev]);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return wp_noalloc_fail(-2, cudaGetErrorString(e));
  return 0;
}
