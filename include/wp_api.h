/* wp_api.h -- C ABI of the B200-native grouped multi-LoRA apply library
 * (libwp_b200.so).
 *
 * The library replaces the reference's pybind extension `warp_pipe_ext`
 * (csrc/pybind, csrc/dispatch, csrc/kernels, csrc/memory of
 * vac014/AdapterSlotsPlusPlus). Every entry point below names the reference
 * method it stands in for as `file:line` inside that project.
 *
 * Conventions
 *   - Plain pointers and sizes only; no torch types. Device pointers are
 *     CUDA device addresses on the handle's device; `stream` is a
 *     cudaStream_t passed as void*.
 *   - Return value: 0 = ok; >0 = "not handled" (the Python engine maps it to
 *     a False return where the reference returns False); <0 = error (the
 *     engine raises). wp_last_error() gives the message of the last error.
 *   - One handle per device and thread; calls on one handle are not
 *     thread-safe (the reference's WarpPipeExtension is not either).
 *   - Math: A is stored [r, d] (rank-major), B is stored [o, r];
 *     H[t,:] = alpha * X[t,:] . A^T  (fp32), Y[t,:] += H[t,:] . B^T, with
 *     alpha applied once, in shrink (tests/correctness/reference_bgmv.py:4-18).
 */
#ifndef WP_API_H_
#define WP_API_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define WP_OK 0
#define WP_NOT_HANDLED 1
#define WP_ERR_INVALID (-1)
#define WP_ERR_CUDA (-2)
#define WP_ERR_UNKNOWN_ADAPTER (-3)
#define WP_ERR_CAPACITY (-4)
#define WP_ERR_NCCL (-5)
#define WP_ERR_DEVICE_TIMEOUT (-6)

/* element types */
#define WP_DTYPE_F16 0
#define WP_DTYPE_BF16 1
#define WP_DTYPE_F32 2
#define WP_DTYPE_I32 3
#define WP_DTYPE_I64 4

/* which segment table wp_read_seg_table returns */
#define WP_TABLE_LIVE 0     /* built by wp_build_seg_bounds */
#define WP_TABLE_REGISTRY 1 /* built by wp_build_segments   */
#define WP_TABLE_TILES 2    /* prefill mode: 128-token tiles of the long runs */
#define WP_TABLE_SHORT 3    /* prefill mode: pieces of the short runs */

/* segment table modes of wp_build_seg_bounds_ex */
#define WP_SEG_DECODE 0  /* pieces of at most 32 tokens only (the reference's table) */
#define WP_SEG_PREFILL 1 /* also: runs of >= 128 tokens as 128-token tiles for the tcgen05 prefill kernels */
#define WP_SEG_AUTO 2    /* prefill mode when T >= wp_config.prefill_tokens > 0 (the default of wp_build_seg_bounds) */

typedef struct wp_handle wp_handle;

typedef struct wp_config {
  int32_t device;            /* CUDA device ordinal                                  */
  int32_t max_tokens;        /* capacity of the per-step tables (T), e.g. 16384       */
  int32_t num_staging_slots; /* GPU staging slots (reference: WP_MAX_STAGING = 8)     */
  int64_t slot_bytes;        /* bytes per slot for A+B together (0 = 2*64*16384*2)    */
  int32_t ctas_per_sm;       /* cap on persistent CTAs per SM of the apply kernel (0=auto) */
  int32_t use_pdl;           /* 1 = programmatic dependent launch between kernels     */
  int32_t prefetch_weights;  /* 1 = with use_pdl, start loading adapter weights before the
                                previous kernel on the stream finishes. The caller promises
                                that the kernel right before an apply call never writes the
                                adapter weights (true in serving: weights are static during
                                a step). 0 = strict stream order. */
  int32_t kernel;            /* apply kernel of fused live-mode calls: 0 = default (automatic,
                                or the WP_KERNEL environment variable: "split", "cluster"),
                                1 = clustered decode (mma.sync), 2 = balanced decode
                                ("split": one CTA per SM, equal one-stage items) */
  int32_t prefill_tokens;    /* WP_SEG_AUTO switches to prefill mode at this many tokens
                                (> 0; 0 = never, the default: on B200 the decode kernel is
                                faster on the measured prefill mixes) */
  int32_t peer_wait_ms;      /* bound of each in-kernel wait on a tensor-parallel peer
                                (wp_add_lora_row_parallel); 0 = 5000 ms. On expiry the
                                kernel sets WP_ERR_DEVICE_TIMEOUT's flag and returns. */
  int32_t prefetch_inputs;   /* with use_pdl and prefetch_weights: a fused live call loads its
                                x and runs its whole shrink phase before the previous kernel
                                on the stream finishes; only the y loads wait for it. The
                                caller promises that the kernel right before each apply call
                                never writes that call's x (serving: it is the base layer's
                                GEMM, which reads x and writes y); wp_note_input_write lifts
                                the promise for one call. Not used with tensor parallelism. */
} wp_config;

/* One entry of the segment table, as read back by wp_read_seg_table.
 * Mirrors the three fields of SegmentDescriptor the live kernels read
 * (csrc/bridge/warp_pipe_metadata.h:41-57). */
typedef struct wp_segment {
  int32_t adapter_id;
  int32_t token_start;
  int32_t token_count;
} wp_segment;

/* ---- lifetime ---------------------------------------------------------- */

/* Replaces WarpPipeExtension::WarpPipeExtension (warp_pipe_bindings.cpp:20-34):
 * allocates the device-resident segment tables, workspaces, staging slots and
 * the private prefetch stream. */
int wp_create(const wp_config* cfg, wp_handle** out);

/* Replaces ~WarpPipeExtension (warp_pipe_bindings.cpp:36-39). */
int wp_destroy(wp_handle* h);

/* Message of the last failed call on this handle (or a global message when
 * h is NULL). Never NULL. */
const char* wp_last_error(const wp_handle* h);

/* Replaces warp_pipe_rank_supported (csrc/dispatch/warp_pipe_dispatcher.cpp:18):
 * 1 for r in {8,16,32,64}, else 0. */
int wp_rank_supported(int32_t rank);

/* Kernel of the latest apply launch: 0 = balanced decode ("split_kernel"),
 * 1 = clustered decode ("apply_kernel", clusters of 2), 3 = clustered decode
 * on clusters of 4 (fused live calls with few segments), -1 = none yet.
 * For reports and profiling. */
int32_t wp_last_apply_kernel(const wp_handle* h);

/* Number of kernels this handle has launched so far (all entry points). */
int64_t wp_kernel_launch_count(const wp_handle* h);

/* ---- adapter store ----------------------------------------------------- */

/* Replaces WarpPipeExtension::register_adapter (warp_pipe_bindings.cpp:110-119)
 * and AdapterStore::register_adapter (csrc/memory/adapter_store.h:21-27).
 * A [r,d] and B [o,r] are DEVICE pointers (16-byte aligned, the caller keeps
 * them alive until eviction). Re-registering an id overwrites it. */
int wp_register_adapter(wp_handle* h, int32_t adapter_id, const void* A, const void* B, int32_t rank,
                        int32_t d_model, int32_t out_features, float alpha_scale, int32_t dtype);

/* Pinned-host adapter store (no counterpart in the reference, which keeps
 * every adapter on the device): A/B are HOST pointers; the library copies
 * them into its own page-locked store. The adapter reaches the GPU through a
 * staging slot (wp_prefetch_adapter, or on demand inside wp_build_segments). */
int wp_register_adapter_host(wp_handle* h, int32_t adapter_id, const void* A_host, const void* B_host,
                             int32_t rank, int32_t d_model, int32_t out_features, float alpha_scale,
                             int32_t dtype);

/* Replaces WarpPipeExtension::evict_adapter (warp_pipe_bindings.cpp:121-124).
 * Unknown ids are a no-op. Frees the adapter's staging slot, if any. */
int wp_evict_adapter(wp_handle* h, int32_t adapter_id);

/* ---- segment tables ---------------------------------------------------- */

/* Replaces WarpPipeExtension::build_segments (warp_pipe_bindings.cpp:128-130)
 * -> build_segment_table (csrc/dispatch/segment_builder.cpp:5-50).
 * K segments, seg_offsets has K+1 entries (host arrays). Errors on a size
 * mismatch, K > max_tokens or an unknown id, like the reference. The table is
 * uploaded on `stream`. Adapters that live only in the host store are staged
 * into a slot on the prefetch stream and `stream` waits for that copy. */
int wp_build_segments(wp_handle* h, const int32_t* sorted_adapter_ids, const int32_t* seg_offsets, int32_t K,
                      void* stream);

/* Replaces WarpPipeExtension::build_seg_bounds (warp_pipe_bindings.cpp:162-170)
 * -> build_seg_bounds_kernel (csrc/kernels/warp_pipe_r32.cu:461-512).
 * token_lora_indices: DEVICE array of T ints (idx_dtype WP_DTYPE_I32 or
 * WP_DTYPE_I64). Builds the run-length table (runs of equal ids in token
 * order, ids < 0 skipped, runs split into pieces of at most 32 tokens) on the
 * device, without a host sync. Returns WP_NOT_HANDLED (the reference's False)
 * only when T exceeds max_tokens; the reference's cap is 256. */
int wp_build_seg_bounds(wp_handle* h, const void* token_lora_indices, int32_t idx_dtype, int32_t T,
                        void* stream);

/* wp_build_seg_bounds with an explicit mode (flags: WP_SEG_DECODE,
 * WP_SEG_PREFILL, WP_SEG_AUTO). In prefill mode the full table is built as
 * usual and, besides it, the runs of at least 128 tokens of one adapter
 * become 128-token tiles; a following wp_add_lora / wp_add_lora_slices then
 * runs them as tcgen05 GEMMs (M = 128 tokens, accumulators in TMEM) and the
 * short runs on the decode kernel (calls that the prefill kernels do not
 * cover -- rank 8, d or o not a multiple of 64, unaligned y -- take
 * the full table on the decode kernel). The reference has no prefill path:
 * it caps segments at 32 tokens (csrc/bridge/warp_pipe_metadata.h:22). */
int wp_build_seg_bounds_ex(wp_handle* h, const void* token_lora_indices, int32_t idx_dtype, int32_t T, int32_t flags,
                           void* stream);

/* Allocation-free segmenter (no counterpart in the reference). For callers
 * that may not allocate device memory at all -- e.g. a plugin running inside
 * another framework's pre-planned memory, where a cudaMalloc would synchronise
 * the device and bypass that framework's allocator -- and therefore cannot
 * create a wp_handle. Same table as wp_build_seg_bounds, written by the
 * device as int32 triples (adapter_id, token_start, token_count) into the
 * caller's DEVICE buffer out_table (room for T triples) and the count into
 * the caller's DEVICE int32 *out_num, on `stream`, on the current device.
 * Its only scratch (run starts) is a fixed array of
 * wp_seg_bounds_noalloc_max_tokens() = 65536 ints inside the library's device
 * image, held on every GPU that loads the library until the process exits;
 * T above that is rejected (WP_ERR_CAPACITY, message in wp_last_error(NULL)).
 * Nothing needs to start at zero: each call writes the scratch before reading
 * it. The first call on a device looks the array's address up, so make it
 * before any stream capture. All calls on a device share the array: calls
 * that overlap on the GPU race. Calls no allocating routine. */
int wp_build_seg_bounds_noalloc(const void* token_lora_indices, int32_t idx_dtype, int32_t T, int32_t* out_table,
                                int32_t* out_num, void* stream);
/* Largest T wp_build_seg_bounds_noalloc accepts (65536). */
int wp_seg_bounds_noalloc_max_tokens(void);

/* Test readback of a segment table (the reference exposes none). Synchronises
 * the handle's device. Writes up to `cap` entries, sets *num to the table's
 * num_segments. */
int wp_read_seg_table(wp_handle* h, int32_t which, wp_segment* out, int32_t cap, int32_t* num);

/* ---- apply ------------------------------------------------------------- */

/* Replaces WarpPipeExtension::shrink (warp_pipe_bindings.cpp:132-139) ->
 * bgmv_shrink_kernel (warp_pipe_r32.cu:56-132, warp_pipe_rgen.cuh:42-135).
 * Uses the registry table (wp_build_segments). X: device [T, d] (dtype),
 * H: device [T, r] fp32, caller-zeroed; rows inside segments are written with
 * alpha_scale(adapter) * X . A^T. */
int wp_shrink(wp_handle* h, const void* X, void* H, int32_t d_model, int32_t rank, int32_t T, int32_t dtype,
              void* stream);

/* Replaces WarpPipeExtension::expand (warp_pipe_bindings.cpp:141-148) ->
 * bgmv_expand_kernel (warp_pipe_r32.cu:141-200, warp_pipe_rgen.cuh:137-189).
 * H: device [T, r] fp32; Y: device [T, o] (dtype), updated in place. */
int wp_expand(wp_handle* h, const void* H, void* Y, int32_t out_features, int32_t rank, int32_t T,
              int32_t dtype, void* stream);

/* The kernel the caller just enqueued on the stream wrote the next apply
 * call's x (e.g. a copy that made it contiguous): that call loads x only
 * after the dependency wait, whatever prefetch_inputs says. No reference
 * counterpart (the reference has no programmatic dependent launch). */
int wp_note_input_write(wp_handle* h);

/* Replaces WarpPipeExtension::add_lora_packed (warp_pipe_bindings.cpp:195-234)
 * -> bgmv_shrink_dsak_kernel + bgmv_expand_dsak_kernel (warp_pipe_r32.cu:280-423),
 * and covers the sliced-output and non-rank-32 calls the reference sends back
 * to the stock path (lora_warp_pipe/punica_wrapper.py:147-155).
 * Uses the live table (wp_build_seg_bounds). For token t in a segment of
 * adapter i:  y[t, y_offset + j] += (scale * x[t,:] . A_i^T) . B_i[j,:]
 * with A_i = wa_base + i*wa_stride0 ([r,d] row-major), B_i = wb_base +
 * i*wb_stride0 ([o,r] row-major), j < out_features. x row stride x_ld, y row
 * stride y_ld (elements). Graph-capturable: fixed grids, the segment count is
 * read on the device. */
int wp_add_lora(wp_handle* h, void* y, const void* x, const void* wa_base, int64_t wa_stride0,
                const void* wb_base, int64_t wb_stride0, int32_t num_adapters, float scale, int32_t T, int32_t d_model,
                int32_t out_features, int32_t rank, int64_t x_ld, int64_t y_ld, int32_t y_offset,
                int32_t dtype, void* stream);

/* Several output slices sharing x in one launch, the shape of vLLM's
 * PunicaWrapper.add_lora_packed_nslice (q/k/v, gate/up), which the reference
 * leaves to its FusedPunicaWrapper (lora_warp_pipe/punica_wrapper.py:8-30).
 * Slice s (s < nslices <= 3) adds (scale * x . A_s,i^T) . B_s,i^T into
 * y[:, y_offsets[s] : y_offsets[s] + out_features], with A_s,i = wa_bases[s]
 * + i*wa_strides[s] and B_s,i = wb_bases[s] + i*wb_strides[s]. All slices
 * share rank, d_model, out_features and num_adapters. Result per slice is
 * identical to nslices wp_add_lora calls. */
int wp_add_lora_slices(wp_handle* h, void* y, const void* x, int32_t nslices, const void* const* wa_bases,
                       const int64_t* wa_strides, const void* const* wb_bases, const int64_t* wb_strides,
                       const int32_t* y_offsets, int32_t num_adapters, float scale, int32_t T, int32_t d_model,
                       int32_t out_features, int32_t rank, int64_t x_ld, int64_t y_ld, int32_t dtype,
                       void* stream);

/* Shrink half of wp_add_lora, exported for tensor-parallel row-parallel
 * layers: H [T, r] fp32 (device) receives scale * x . A^T for rows inside
 * live segments; other rows are left untouched. */
int wp_add_lora_shrink(wp_handle* h, void* H, const void* x, const void* wa_base, int64_t wa_stride0,
                       int32_t num_adapters, float scale, int32_t T, int32_t d_model, int32_t rank, int64_t x_ld,
                       int32_t dtype, void* stream);

/* Expand half of wp_add_lora: y[t, y_offset + j] += H[t,:] . B_i[j,:] for the
 * num_adapters stacked B_i = wb_base + i*wb_stride0. */
int wp_add_lora_expand(wp_handle* h, void* y, const void* H, const void* wb_base, int64_t wb_stride0,
                       int32_t num_adapters, int32_t T, int32_t out_features, int32_t rank, int64_t y_ld,
                       int32_t y_offset, int32_t dtype, void* stream);

/* ---- adapter pool: the live path over a pinned-host store --------------- */

/* The reference stages host adapters only for its registry path
 * (StagingBufferPool, csrc/memory/staging_buffer.h:29-105, fed by
 * prefetch_adapter, csrc/pybind/warp_pipe_bindings.cpp:46-64); its live
 * DSAK path reads device stacks only (csrc/kernels/warp_pipe_r32.cu:263-269).
 * A pool pages whole adapters -- one tenant's A/B of every LoRA projection of
 * a model (num_proj projections, projection p: A [rank, d[p]], B [o[p], rank])
 * -- from caller-owned page-locked host blobs into num_slots GPU slots. The
 * slots of projection p are a stacked tensor that wp_add_lora takes as is
 * (wp_pool_stack); wp_build_seg_bounds_pool writes the live table with slot
 * numbers in place of adapter ids. Adapter ids are 0 .. max_adapters-1. */
typedef struct wp_pool wp_pool;
int wp_pool_create(wp_handle* h, int32_t num_slots, int32_t num_proj, int32_t rank, const int32_t* d,
                   const int32_t* o, int32_t dtype, int32_t max_adapters, wp_pool** out);
int wp_pool_destroy(wp_pool* p);
/* Byte offsets of projection proj's A and B inside one slot (and inside a
 * registered host blob, which has the slot's layout), and the slot size. */
int wp_pool_layout(wp_pool* p, int32_t proj, int64_t* a_off, int64_t* b_off, int64_t* slot_bytes);
/* Device stacks of projection proj: wa = [num_slots][1][rank][d] and wb =
 * [num_slots][1][o][rank] with adapter stride stride0 (elements). */
int wp_pool_stack(wp_pool* p, int32_t proj, void** wa, void** wb, int64_t* stride0);
/* Registers adapter_id's host blob (page-locked, slot_bytes, the caller keeps
 * it alive until wp_pool_evict). Re-registering replaces it. */
int wp_pool_register_host(wp_pool* p, int32_t adapter_id, const void* blob);
int wp_pool_evict(wp_pool* p, int32_t adapter_id);
/* Same semantics as wp_prefetch_adapter / wp_is_prefetch_ready /
 * wp_release_prefetch, for the pool: copies the adapter into a free or least
 * recently used slot (never one the current step reads) on the pool's copy
 * stream and holds it until released; -1 for an unknown id or no free slot. */
int32_t wp_pool_prefetch(wp_pool* p, int32_t adapter_id);
int32_t wp_pool_is_ready(wp_pool* p, int32_t adapter_id);
int wp_pool_release(wp_pool* p, int32_t adapter_id);
/* Starts a step on `stream`: makes every adapter in ids[0..n) resident
 * (copies for the cold ones are issued now on the copy stream), makes
 * `stream` wait for the copies it reads (no host sync), and uploads the slot
 * map. A slot is overwritten only after the kernels of the steps that read it.
 * Returns the number of adapters copied here (cold misses), or < 0. */
int wp_pool_prepare(wp_pool* p, const int32_t* ids, int32_t n, void* stream);
int wp_pool_stats(wp_pool* p, int64_t* copies, int64_t* bytes, int32_t* resident);
/* wp_build_seg_bounds with the ids translated to the pool's slots (ids that
 * are not resident are dropped and raise the device error flag). */
int wp_build_seg_bounds_pool(wp_handle* h, wp_pool* p, const void* token_lora_indices, int32_t idx_dtype, int32_t T,
                             void* stream);

/* ---- staging slots / prefetch ------------------------------------------ */

/* Replaces WarpPipeExtension::prefetch_adapter (warp_pipe_bindings.cpp:46-57)
 * and StagingBufferPool::acquire_slot (csrc/memory/staging_buffer.h:62-73):
 * copies the adapter's A/B into a staging slot on the private prefetch
 * stream. Returns the slot index, or -1 (unknown id, or no free slot). Never
 * fails otherwise. Re-prefetching an adapter returns its existing slot. */
int32_t wp_prefetch_adapter(wp_handle* h, int32_t adapter_id);

/* Same as wp_prefetch_adapter, but the copy is ordered after the work queued
 * so far on `caller_stream` (the stream that produced the adapter's tensors),
 * without blocking the host. */
int32_t wp_prefetch_adapter_on(wp_handle* h, int32_t adapter_id, void* caller_stream);

/* Replaces is_prefetch_ready (warp_pipe_bindings.cpp:59-62,
 * staging_buffer.h:89-93): non-blocking event query. */
int32_t wp_is_prefetch_ready(wp_handle* h, int32_t adapter_id);

/* Replaces release_prefetch (warp_pipe_bindings.cpp:64, staging_buffer.h:75-79).
 * Unknown ids are a no-op. */
int wp_release_prefetch(wp_handle* h, int32_t adapter_id);

/* Slot bookkeeping for tests and benches: number of slots, slots in use, and
 * the device error flag raised by a timed-out wait inside a kernel (0 = none;
 * reading it synchronises the device; `clear` resets it). */
int wp_slot_stats(wp_handle* h, int32_t* num_slots, int32_t* slots_in_use);
int wp_device_error(wp_handle* h, int32_t clear, int32_t* flag);

/* ---- scheduler bridge ----------------------------------------------------- */

/* Scheduler state for one tick, the fields of the reference's
 * SchedulerKernelBridge (csrc/bridge/warp_pipe_metadata.h:89-104): per adapter
 * slot i < num_active_adapters (at most WP_BRIDGE_MAX = 64). */
#define WP_BRIDGE_MAX 64
typedef struct wp_bridge {
  float whittle_scores[WP_BRIDGE_MAX];
  float t_remaining_ms[WP_BRIDGE_MAX];
  float gwar_pred_next3[WP_BRIDGE_MAX];
  float lambda_hat[WP_BRIDGE_MAX];
  uint8_t burst_active[WP_BRIDGE_MAX];
  uint8_t promo_eligible[WP_BRIDGE_MAX];
  uint8_t is_hot[WP_BRIDGE_MAX];
  uint8_t prefetch_ready[WP_BRIDGE_MAX];
  uint8_t tile_size_code[WP_BRIDGE_MAX];
  uint32_t step_id;
  uint32_t num_active_adapters;
  uint32_t num_segments;
  float global_load;
} wp_bridge;

/* Replaces WarpPipeExtension::write_bridge (warp_pipe_bindings.cpp, engine.py:34-42
 * of the reference): copies one tick's state into the handle's page-locked,
 * device-mapped bridge. Fails when num_active_adapters > WP_BRIDGE_MAX. */
int wp_write_bridge(wp_handle* h, const wp_bridge* b);
/* Replaces read_bridge_debug (engine.py:34-37): host read of the bridge. */
int wp_read_bridge(wp_handle* h, wp_bridge* out);
/* Replaces read_bridge_via_kernel (engine.py:39-42): a kernel reads the bridge
 * through its device mapping and writes [whittle_scores[0..n), n,
 * num_segments, step_id] (n + 3 floats) to device memory, which is copied to
 * out (cap floats); *count = n + 3. Synchronises the handle's device. */
int wp_read_bridge_kernel(wp_handle* h, float* out, int32_t cap, int32_t* count);

/* ---- tracing and launch plan (no counterpart in the reference) --------- */

/* Turns per-CTA phase tracing of the apply kernel on or off. When on, each
 * launch (kernel 0: fused or shrink-only, kernel 1: expand-only) records, per
 * CTA, 8 + 4*16 uint64: start, after the dependency wait, first stage ready,
 * end (globaltimer ns), stages consumed, ns waited for stages, 0, 0, then
 * (before wait, after wait, after compute, after hand-back) for the first 16
 * stages. */
int wp_trace_enable(wp_handle* h, int32_t enable);
/* Copies the record of the latest launch of `kernel` (synchronises). */
int wp_trace_read(wp_handle* h, int32_t kernel, uint64_t* out, int32_t cap, int32_t* n);
/* Cluster size and persistent grid the apply kernel uses for (dtype, rank). */
int wp_apply_plan(wp_handle* h, int32_t dtype, int32_t rank, int32_t* cluster, int32_t* grid);

/* ---- tensor parallel (no counterpart in the reference) ----------------- */

/* Size of the opaque NCCL unique id blob (ncclUniqueId). */
int32_t wp_tp_unique_id_bytes(void);
/* Rank 0 fills `id` (wp_tp_unique_id_bytes() bytes); the caller broadcasts it. */
int wp_tp_get_unique_id(void* id);
/* Creates this handle's NCCL communicator over NVLink (one rank per GPU). */
int wp_tp_init(wp_handle* h, const void* id, int32_t rank, int32_t world);
/* In-place fp32 sum all-reduce of n floats on `stream` (row-parallel shrink
 * partials [T, r]). Capturable in a CUDA graph. */
int wp_tp_allreduce_f32(wp_handle* h, void* buf, int64_t n, void* stream);
int wp_tp_destroy(wp_handle* h);

/* Row-parallel layers over peer memory (one process per GPU, NVLink P2P):
 * a fused alternative to wp_add_lora_shrink + wp_tp_allreduce_f32 +
 * wp_add_lora_expand for the row-parallel LoRA layers of a tensor-parallel
 * model (reference: single-GPU only; the sharding follows vLLM's
 * RowParallelLinearWithLoRA). Each rank creates a mailbox (device memory
 * for the [T, r] partials of every rank plus flags) and exports it; the
 * caller all-gathers the handles (world x wp_tp_mailbox_handle_bytes()
 * bytes, in rank order) and opens them. */
int32_t wp_tp_mailbox_handle_bytes(void);
int wp_tp_mailbox_create(wp_handle* h, int32_t rank, int32_t world, int32_t max_tokens, void* handle_out);
int wp_tp_mailbox_open(wp_handle* h, const void* handles);
int wp_tp_mailbox_close(wp_handle* h);

/* One launch per row-parallel layer: each segment's partial H over this
 * rank's d slice (x [T, d_shard], A stack sliced along d) is exchanged with
 * the peers inside the kernel (stores into their mailboxes, a release flag,
 * a bounded acquire wait), summed in rank order, and expanded with the full
 * B onto y: y[t, y_offset + j] += (scale * sum_ranks x_p[t,:] . A_p^T) . B[j,:].
 * Every rank calls it with the same segment table and T. */
int wp_add_lora_row_parallel(wp_handle* h, void* y, const void* x, const void* wa_base, int64_t wa_stride0,
                             const void* wb_base, int64_t wb_stride0, int32_t num_adapters, float scale, int32_t T,
                             int32_t d_shard, int32_t out_features, int32_t rank, int64_t x_ld, int64_t y_ld,
                             int32_t y_offset, int32_t dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WP_API_H_ */
