// wp_apply.cu -- the grouped multi-LoRA apply kernel (decode) for sm_100a.
//
// Semantics (reference: tests/correctness/reference_bgmv.py:4-18, the math of
// bgmv_shrink_kernel / bgmv_expand_kernel in csrc/kernels/warp_pipe_r32.cu:56-200
// and their DSAK twins :280-423):
//   shrink:  H[t, :] = alpha * X[t, :] . A_seg^T      (fp32)
//   expand:  Y[t, j] = round(Y[t, j] + H[t, :] . B_seg[j, :])
// for every token t inside a segment of the table; other rows are untouched.
//
// One launch does both halves of one LoRA layer call. The grid is persistent
// (a fixed number of co-resident CTAs, so the launch can be captured in a CUDA
// graph) and organised in thread-block clusters of CL CTAs (CL = 2 on B200);
// the segmenter's ClusterPlan gives each cluster its segments (when clusters
// are left over, the largest segments, at most kPlanMaxHelpers, get a helper
// cluster that takes half of their output columns; these pairs take the
// lowest clusters, the whole segments follow). For one
// segment the CL CTAs of the cluster
//   1. split d in CL slices: CTA q streams A[:, slice q] and x[segment rows,
//      slice q] and accumulates a [r x <=32] fp32 partial;
//   2. exchange the partials through distributed shared memory (st.async
//      pushes into the peers' receive slots, completed on the peer's
//      mbarrier) and add them in cluster-rank order: deterministic, and the
//      same H on every CTA; with tensor parallelism (row-parallel "fused"
//      mode) the partial then goes through the peers' mailboxes as well;
//   3. split o in CL slices: CTA q streams B[slice q, :] and y[segment rows,
//      slice q] and adds H . B^T to y, rounding once.
// H never leaves the cluster; there are no global atomics and no second launch.
// The same kernel runs the shrink alone (H written to global memory, for the
// registry-path shrink() and the NCCL row-parallel mode) or the expand alone
// (H read from global memory).
//
// Math: warp-level mma.sync m16n8k16 (bf16/fp16 in, fp32 accumulate) on
// fragments loaded with ldmatrix from the swizzled TMA boxes. Decode segments
// are at most 32 tokens, where a tcgen05.mma (M >= 64) would cost as much as a
// whole mma.sync stage; runs of >= 128 tokens of one adapter have their own
// tcgen05 GEMM kernels in wp_prefill.cu.
//   shrink: D[rank, token] += A . x^T, warp w owning 32 columns of every
//     stage, the eight warp partials added in a fixed order.
//   expand, transposed: D^T[o, t] = y + B[o, :] . H[t, :]^T with M = 16 output
//     columns and N = 8 tokens per tile; y enters the accumulator through
//     ldmatrix.trans and leaves through stmatrix.trans, rounded once. H enters
//     rounded to the weights' 16-bit type, as the stock expand takes it.
// The stage bodies are compiled for 1, 2 and 4 token tiles of 8 (a segment
// of three tiles runs the four-tile body: the rows of its fourth tile are
// computed in shared memory and never stored).
//
// Warp roles, handing off only through mbarriers:
//   warp 8 (producer): lane 0 issues every TMA load of the CTA into a ring of
//     STAGES shared-memory stages ("full" barriers) and refills a stage when
//     its "empty" barrier fires; it runs ahead across segment and phase
//     boundaries (the expand-phase loads of B and y do not depend on H).
//   warp 9 (y store): a segment that fills its y box exactly (8, 16 or 32
//     rows) leaves through one tensor store per stage; with prefetched
//     weights it also loads the first stages' activations right after the
//     dependency wait.
//   warps 0-7 (compute): the mma.sync math of every stage, the cluster
//     exchange, the y add and store, and the release of the stages.
//
// Data movement: A and x arrive as tiled tensor loads (cp.async.bulk.tensor)
// of 64-column boxes with the 128-byte swizzle -- conflict-free fragment
// loads, zero fill past the ends of d and T; x and y boxes are 8, 16 or 32
// rows high to match the segment. B arrives as tensor boxes of 256 rows whose
// swizzle matches its 2r-byte rows (rank 8: one 1-D bulk copy). One stage
// carries 256 elements of d (shrink) or 256 output columns (expand). The
// cluster's segment descriptors are cached in shared memory once per launch.
//
// Programmatic dependent launch: every thread waits on the predecessor
// (griddepcontrol.wait) before it triggers the dependents, so the pre-wait
// prologue overlaps only the immediately preceding kernel. When the host says
// the table and the weights are not written by that kernel, the prologue
// reads the table and starts the weight loads (A, B) before the wait;
// activations (x, y, H) are always loaded after it.
//
// Waits are bounded (1 s; a wait on a tensor-parallel peer by
// wp_config.peer_wait_ms). A timed-out wait raises an error bit and marks the
// CTA bad: compute stops, the producer stops issuing, the compute warps keep
// arriving on the empty barriers and keep taking part in the cluster barriers
// (so no partner is left waiting), copies in flight are drained with a short
// bounded wait, and the kernel exits.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <type_traits>

#include "wp_device.cuh"
#include "wp_internal.h"
#include "wp_kernel_common.cuh"

namespace wp {

constexpr int kComputeWarps = 8;
constexpr int kComputeThreads = kComputeWarps * 32;
constexpr int kProducerWarp = kComputeWarps;  // TMA issue
constexpr int kStoreWarp = kComputeWarps + 1;  // y tensor stores, first activations
constexpr int kThreads = kComputeThreads + 64;  // + the producer and store warps
constexpr int kBarCompute = 1;  // named barrier of the compute warps
constexpr int kDescCache = 64;  // segment descriptors cached per CTA
constexpr int kSnakeMax = 128;  // tables up to this size are dealt by decreasing token count
constexpr unsigned long long kDrainNs = 10000000ull;  // 10 ms per stage when draining after an error

constexpr int kSmemMax = 232448;  // dynamic shared memory per CTA (227 KB)

template <int N>
struct IntC {
  static constexpr int value = N;
};

// CLM: cluster ranks the receive slots serve (2; 4 for the clusters-of-4
// instantiation of few-segment calls).
template <int R, int CLM = 2>
struct ApplyCfg {
  static constexpr int KC = kStageK;  // d elements per shrink stage (4 boxes)
  static constexpr int W = kStageCols;  // output columns per expand stage (4 boxes)
  static constexpr int ABOX = R * 128;  // one A box: R rows x 128 B
  static constexpr int XBOX = 32 * 128;  // room for one 32-row x or y box
  static constexpr int STAGE = 4 * ABOX + 4 * XBOX;  // == 4 * XBOX + W * R * 2; multiple of 1024
  static_assert(STAGE == 4 * XBOX + W * R * 2, "shrink and expand stages have one size");
  static constexpr int PITCH = R + 4;  // floats per row of the P / H tiles
  static constexpr int OFF_FLAGS = 448;
  static constexpr int OFF_DESC = 512;
  static constexpr int OFF_P = OFF_DESC + kDescCache * 32;
  static constexpr int OFF_H = OFF_P + 32 * PITCH * 4;
  static constexpr int OFF_END = OFF_H + 32 * PITCH * 4;
  static constexpr bool BTMA = R >= 16;  // B as swizzled tensor boxes (rank 8: one linear bulk copy)
  static constexpr uint32_t SWZ_MASK = R == 64 ? 0x70u : (R == 32 ? 0x30u : 0x10u);
  // shrink partials of the 8 compute warps (32 tokens x PITCH floats each) for the cross-warp sum
  static constexpr int PSLOT = 32 * PITCH;  // one segment's partial (32 token rows)
  // The eight compute warps' partials are added in passes of PROWS token
  // rows (one slot of PROWS rows per warp): fewer rows per pass leave more
  // shared memory to the stage ring (rank 32: 6 stages instead of 5; rank
  // 64: 3 instead of 2), at two more barriers per extra pass.
  static constexpr int PROWS = R == 64 ? 16 : (R == 32 ? 8 : 32);
  static constexpr int PWSLOT = PROWS * PITCH;
  static constexpr int PW = 8 * PWSLOT * 4;
  // receive slots of the cluster exchange, [2 segment parities][CLMAX - 1
  // peers]: rank i's partial in slot i (i below this CTA's rank) or i - 1
  static constexpr int CLMAX = CLM;
  static constexpr int RXSLOTS = CLMAX - 1;
  static constexpr int RX = 2 * RXSLOTS * PSLOT * 4;
  static constexpr int FIXED = OFF_END + PW + RX + 1024;
  static constexpr int FIT = (kSmemMax - FIXED) / STAGE;
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr int SMEM = FIXED + STAGES * STAGE;
  static_assert(STAGES >= 2 && STAGES <= 8 && SMEM <= kSmemMax, "shared memory budget");
  static_assert(32 * PITCH * 4 >= kComputeWarps * 128, "the P tile holds one scratch row per compute warp");
  static_assert(32 * PITCH * 4 >= kTraceSlots * 8, "the P tile holds the staged trace record");
  static_assert(PW >= 4 * kSnakeMax * 4, "the partial slots hold the table-ordering scratch");
};

// Segment assignment without a plan from the segmenter (multi-slice calls, a
// plan made for another cluster count, the registry path). Out of line: the
// production path reads the plan and never runs this code, which keeps it
// out of the instruction cache. Segments per cluster, for small tables
// (decode) ordered by decreasing token count. Fewer segments than clusters:
// the largest segments (at most kPlanMaxHelpers) get a helper cluster each,
// and the pair splits the segment's output columns (both clusters run the
// shrink; the second reads A mostly from L2); the helper pairs take the
// lowest clusters, which the hardware dispatches first (with programmatic
// dependent launch they also start first), the whole segments follow. More segments than clusters: "snake" dealing (round r gives
// cluster c the segment at sorted position r*G + c or r*G + G-1-c,
// alternating, with the last, partial round running forward), pairing large
// segments with small ones. Larger tables go round robin (cluster c takes c,
// c + G, ...). Multi-slice calls: virtual segment v is segment v % nseg of
// slice v / nseg; its descriptor carries the slice in the (live-mode unused)
// alpha field. Called by every thread of the CTA.
struct TableView {
  int nmine, seg_half, oB0, nB, nseg_t;
};

template <int R>
__device__ __noinline__ void table_fallback(const ApplyArgs& a, int S_sl, bool do_ex, int G, int cid, uint32_t q,
                                            uint32_t CL, int4* sdesc, int* scratch, TableView* tv) {
  using C = ApplyCfg<R>;
  const int tid = threadIdx.x;
  const int nseg_t = __ldcg(a.num_segs);
  tv->nseg_t = nseg_t;
  const int nseg = S_sl * nseg_t;  // virtual segments
  constexpr int kSortMax = 2 * kSnakeMax;  // scratch: the partial slots
  int* cnt = scratch;
  int* order = cnt + kSortMax;
  auto put_desc = [&](int slot, int v) {
    const int seg = v % nseg_t;
    int4 x0 = __ldcg(reinterpret_cast<const int4*>(a.segs + seg));
    const int4 x1 = __ldcg(reinterpret_cast<const int4*>(a.segs + seg) + 1);
    if (S_sl > 1) x0.w = v / nseg_t;
    sdesc[2 * slot] = x0;
    sdesc[2 * slot + 1] = x1;
  };
  auto sort_by_size = [&]() {
    for (int t = tid; t < nseg; t += kThreads) cnt[t] = __ldcg(&a.segs[t % nseg_t].token_count);
    __syncthreads();
    for (int t = tid; t < nseg; t += kThreads) {
      const int ct = cnt[t];
      int p = 0;
      for (int j = 0; j < nseg; ++j) p += (cnt[j] > ct || (cnt[j] == ct && j < t)) ? 1 : 0;
      order[p] = t;
    }
    __syncthreads();
  };
  const int osplit = (((a.o + 1) / 2) + C::W - 1) / C::W * C::W;  // first column of a segment's second half
  if (do_ex && G > 1 && nseg > 0 && nseg < G && nseg <= kSortMax && a.o - osplit >= static_cast<int>(CL) * C::W) {
    sort_by_size();
    const int helpers = min(min(nseg, G - nseg), kPlanMaxHelpers);
    const int V = nseg + helpers;
    // helper pairs first (lowest clusters start first), then whole segments
    tv->nmine = cid < V ? 1 : 0;
    if (tv->nmine) {
      const bool pair = cid < 2 * helpers;
      const int pos = pair ? cid >> 1 : cid - helpers;
      const int half = pair ? (cid & 1) : -1;
      tv->seg_half = half;
      const int ob = half == 1 ? osplit : 0;
      const int olen = half < 0 ? a.o : (half == 0 ? osplit : a.o - osplit);
      const int osl = (olen + static_cast<int>(CL) - 1) / static_cast<int>(CL);
      const int oslr = (osl + C::W - 1) / C::W * C::W;
      tv->oB0 = ob + static_cast<int>(q) * oslr;
      tv->nB = (max(0, min(oslr, ob + olen - tv->oB0)) + C::W - 1) / C::W;
      if (tid == 0) put_desc(0, order[pos]);
    }
  } else if (G > 1 && nseg > G && nseg <= kSortMax) {
    sort_by_size();
    const int rounds = (nseg + G - 1) / G;
    int nm = 0;
    // snake dealing whose last (partial) round runs forward: the clusters
    // holding one segment more are the lowest, which start first
    auto pos_of = [&](int r) { return r * G + (((rounds - 1 - r) & 1) ? G - 1 - cid : cid); };
    for (int r = 0; r < rounds; ++r)
      if (pos_of(r) < nseg) nm = r + 1;  // positions grow with r, so the items are rounds 0..nm-1
    tv->nmine = nm;
    for (int r = tid; r < min(nm, kDescCache); r += kThreads) put_desc(r, order[pos_of(r)]);
  } else {
    const int nm = nseg > cid ? (nseg - cid + G - 1) / G : 0;
    tv->nmine = nm;
    for (int r = tid; r < min(nm, kDescCache); r += kThreads) put_desc(r, cid + r * G);
  }
  __syncthreads();
}

// LF: the live fused call with a tensor-map-aligned y (the serving hot path),
// compiled without the other modes' branches; 1 = one slice, 2 = several
// slices (add_lora_packed_nslice), 4 = one slice on clusters of 4 (calls
// with fewer segments than clusters of 4: each segment's shrink and expand
// spread over four CTAs). TR: per-CTA timeline trace. TPX: row-parallel
// exchange over tensor-parallel peers' memory.
template <typename T, int R, bool TR, int LF, bool TPX = false>
__global__ void __launch_bounds__(kThreads, 1) apply_kernel(const __grid_constant__ ApplyArgs a) {
  using C = ApplyCfg<R, LF == 4 ? 4 : 2>;
  using E = Elem<T>;
  constexpr int S = C::STAGES;
  constexpr int PITCH = C::PITCH;

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + 128);
  uint64_t* cbar = reinterpret_cast<uint64_t*>(smem + 256);
  volatile int* s_bad = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS);
  volatile int* s_issued = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS + 4);
  int4* sdesc = reinterpret_cast<int4*>(smem + C::OFF_DESC);
  float* Ps = reinterpret_cast<float*>(smem + C::OFF_P);
  float* Hs = reinterpret_cast<float*>(smem + C::OFF_H);
  float* Pw = reinterpret_cast<float*>(smem + C::OFF_END);  // cross-warp shrink partials
  float* Rx = reinterpret_cast<float*>(smem + C::OFF_END + C::PW);  // cluster receive slots
  uint64_t* rx_full = reinterpret_cast<uint64_t*>(smem + 352);  // [2] all peers' partials landed (tx count)
  uint64_t* rx_free = reinterpret_cast<uint64_t*>(smem + 368);  // [2] every peer has read my partial
  uint64_t* ydone = reinterpret_cast<uint64_t*>(smem + 384);  // [S] y box of the stage final (8 warps)
  uint8_t* stage_base = align1024(smem + C::OFF_END + C::PW + C::RX);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const bool producer = warp == kProducerWarp;
  const bool registry = !LF && a.registry != 0;
  const bool y_tma = LF || a.y_tma != 0;
  const int nslices = (LF == 1 || LF == 4) ? 1 : a.nslices;
  // the live fused instantiations (not the peer-exchange one) run only with
  // clusters of 2 and sliced tensor maps (the launcher sends other calls to
  // the general instantiation): their code is compiled for exactly that
  constexpr bool kFast = LF != 0 && !TPX;
  const uint32_t q = cluster_ctarank();
  const uint32_t CL = kFast ? (LF == 4 ? 4u : 2u) : cluster_nctarank();
  const int cid = static_cast<int>(cluster_id_x());
  const int G = static_cast<int>(cluster_count_x());
  std::conditional_t<TR, Trace, TraceOff> tr;
  tr.init(a.trace, tid == 0);
  // The plan words of this cluster are loaded first thing, by the store warp
  // (idle at start-up; lane 0: header, 1: count, 2: half, 3..: the
  // descriptors of the cluster's rounds): the load's latency (long while the
  // previous kernel streams at full bandwidth) overlaps the barrier set-up
  // below, and thread 0's barrier-init fence does not wait for it.
  const bool use_plan = nslices <= 1 && a.plan != nullptr;
  int4 plan_word = make_int4(0, 0, 0, 0);
  if (use_plan && cid < kPlanMaxClusters && warp == kStoreWarp) {
    if (lane == 0) plan_word = __ldcg(&a.plan->hdr);
    if (lane == 1) plan_word.x = __ldcg(&a.plan->count[cid]);
    if (lane == 2) plan_word.x = __ldcg(&a.plan->half[cid]);
    if (lane >= 3 && lane < 3 + 2 * kPlanRounds) {
      const int j = lane - 3;
      const int slot = min((j >> 1) * G + cid, kPlanRounds * kPlanMaxClusters - 1);
      plan_word = __ldcg(reinterpret_cast<const int4*>(&a.plan->seg[slot]) + (j & 1));
    }
  }

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kComputeWarps);  // every compute warp frees the stage
      mbar_init(&ydone[s], kComputeWarps);
    }
    mbar_init(cbar, CL);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&rx_full[b], 1);
      mbar_init(&rx_free[b], CL > 1 ? CL - 1 : 1);
    }
    *s_bad = 0;
    *s_issued = 0;
    fence_mbar_init();
  }
  if (producer && lane == 0) {
    if (a.mode & kModeShrink) {
      for (int i = 0; i < 3; ++i) prefetch_tmap(&a.tmap_x[i]);
      if (!registry) prefetch_tmap(&a.tmap_a);
    }
    if ((a.mode & kModeExpand) && y_tma)
      for (int i = 0; i < 3; ++i) prefetch_tmap(&a.tmap_y[i]);
    if ((a.mode & kModeExpand) && C::BTMA && !registry) prefetch_tmap(&a.tmap_b);
    for (int sl = 1; sl < nslices && sl < kMaxSlices; ++sl) {
      prefetch_tmap(&a.tmap_a_x[sl - 1]);
      if (C::BTMA) prefetch_tmap(&a.tmap_b_x[sl - 1]);
      if (y_tma)
        for (int i = 0; i < 3; ++i) prefetch_tmap(&a.tmap_y_x[sl - 1][i]);
    }
  }
  __syncthreads();
  unsigned long long t_init = 0;  // tracing: barriers initialised
  if constexpr (TR) t_init = global_timer_ns();
  // Split cluster barrier: everyone arrives now (releasing the barrier
  // initialisation); the compute warps wait only before their first remote
  // operation on a peer's barriers (the exchange, or the closing cluster
  // barrier), the producer and store warps on their way out. Waiting here
  // would cost the time the partner CTA takes to start.
  cluster_arrive();
  unsigned long long t_synced = 0;  // tracing: after the set-up
  if constexpr (TR) t_synced = global_timer_ns();

  const bool do_sh = LF || (a.mode & kModeShrink) != 0;
  const bool do_ex = LF || (a.mode & kModeExpand) != 0;
  const int kA0 = static_cast<int>(q) * a.split_len;
  const int nA = do_sh ? (max(0, min(a.split_len, a.d - kA0)) + C::KC - 1) / C::KC : 0;
  // this CTA's expand columns (a helper cluster may take half of a segment's
  // output columns; see read_table)
  int oB0 = static_cast<int>(q) * a.oslice;
  int nB = do_ex ? (max(0, min(a.oslice, a.o - oB0)) + C::W - 1) / C::W : 0;
  int ups = nA + nB;  // stages per segment for this CTA
  // decode variant: the y box of an expand stage goes back to global memory
  // with one tensor store when its rows are exactly the segment's rows
  auto y_by_tma = [&](int n) -> bool {
    return y_tma && (kFast || a.o_sliced) && (n == 8 || n == 16 || n == 32);
  };

  // ---- segment table of this cluster (all threads) -------------------------
  int nmine = 0;
  int seg_half = -1;  // helper pairs: which half of the output columns this cluster expands (0 / 1), else -1
  // The segmenter's plan (one load round: header, this cluster's count,
  // half and descriptors together) gives the cluster its segments when it was
  // made for this launch's cluster count; table_fallback deals them otherwise.
  auto helper_range = [&](int half) {
    const int osplit = (((a.o + 1) / 2) + C::W - 1) / C::W * C::W;
    const int ob = half == 1 ? osplit : 0;
    const int olen = half < 0 ? a.o : (half == 0 ? osplit : a.o - osplit);
    const int osl = (olen + static_cast<int>(CL) - 1) / static_cast<int>(CL);
    const int oslr = (osl + C::W - 1) / C::W * C::W;
    oB0 = ob + static_cast<int>(q) * oslr;
    nB = (max(0, min(oslr, ob + olen - oB0)) + C::W - 1) / C::W;
    ups = nA + nB;
  };
  auto read_plan = [&]() -> bool {
    int4* sh = reinterpret_cast<int4*>(Ps);  // scratch: header, count, half
    if (warp == kStoreWarp) {
      if (lane == 0) sh[0] = plan_word;
      if (lane == 1) reinterpret_cast<int*>(sh + 1)[0] = plan_word.x;
      if (lane == 2) reinterpret_cast<int*>(sh + 1)[1] = plan_word.x;
      if (lane >= 3 && lane < 3 + 2 * kPlanRounds) sdesc[lane - 3] = plan_word;
    }
    __syncthreads();
    const int4 hdr = sh[0];
    const int count = reinterpret_cast<const int*>(sh + 1)[0];
    const int half = reinterpret_cast<const int*>(sh + 1)[1];
    seg_half = half;
    __syncthreads();
    if (hdr.x == 0 || hdr.z != G || cid >= kPlanMaxClusters) return false;
    if (hdr.x == 1) {
      // helper halves need an expand and room for a split of the output columns
      const int osplit = (((a.o + 1) / 2) + C::W - 1) / C::W * C::W;
      if (!do_ex || a.o - osplit < static_cast<int>(CL) * C::W) return false;
      if (count > 0) helper_range(half);
    }
    nmine = min(count, kPlanRounds);  // rounds r sit at slot r * G + cid, all loaded above
    return true;
  };
  // multi-slice calls: virtual segment v is segment v % nseg of slice v / nseg
  const int S_sl = nslices > 1 ? nslices : 1;
  int nseg_t = 0;  // segments of the table (not virtual)
  auto read_table = [&]() {
    if (use_plan && read_plan()) return;
    TableView tv{0, -1, oB0, nB, 0};
    table_fallback<R>(a, S_sl, do_ex, G, cid, q, CL, sdesc, reinterpret_cast<int*>(Pw), &tv);
    nmine = tv.nmine;
    seg_half = tv.seg_half;
    oB0 = tv.oB0;
    nB = tv.nB;
    nseg_t = tv.nseg_t;
    ups = nA + nB;
  };
  auto desc = [&](int j) -> DevSeg {
    if (j >= kDescCache) {  // round robin beyond the cache (tables larger than the snake limit)
      const int v = cid + j * G;
      if (S_sl == 1) return load_seg(a.segs, v);
      DevSeg d = load_seg(a.segs, v % nseg_t);
      d.alpha = __int_as_float(v / nseg_t);
      return d;
    }
    return unpack_seg(sdesc[2 * j], sdesc[2 * j + 1]);  // shared-memory copy
  };
  // slice of a (live-mode) descriptor
  auto slice_of = [&](const DevSeg& d) -> int { return S_sl > 1 ? __float_as_int(d.alpha) : 0; };
  auto yoff_of = [&](const DevSeg& d) -> int {
    const int sl = slice_of(d);
    return sl ? a.y_off_x[sl - 1] : a.y_off;
  };

  if (a.prefetch_weights) {
    read_table();
  } else {
    pdl_wait_prior();
    pdl_launch_dependents();
    tr.dep();
    read_table();
  }
  // tracing: the record is staged in the P tile (free after the table read)
  unsigned long long* trc = nullptr;
  if constexpr (TR) {
    if (a.trace) {
      trc = reinterpret_cast<unsigned long long*>(Ps);
      for (int i = tid; i < kTraceSlots; i += kThreads) trc[i] = 0ull;
    }
    __syncthreads();
    tr.stage(trc);
    if (trc && tid == 0) {
      trc[8 + 4] = t_synced;  // mark 4: set-up done (mark 7: table read)
    }
  }
  if (tid == 0) trace_rec_mark<TR>(trc, 7);
  const int total = nmine * ups;


  // TMA issue of stage-unit u into `stage`. parts: 1 = arm the stage's
  // barrier (weights and activations) and load the weights, 2 = load the
  // activations. ef: the L2 evict-first policy of the weight loads.
  // TMA issue. The producer issues the weights of every stage-unit and, once
  // the dependency is met, the activations; with prefetched weights the store
  // thread loads the first stages' activations right after the dependency
  // wait, while the producer is still issuing weights. A single thread issues
  // for the whole CTA, so its per-unit work sits on the critical path: the
  // tensor maps, coordinates and byte counts of a segment are worked out once
  // per segment (SegTma), and a unit costs its barrier arming and one or two
  // copies.
  struct SegTma {
    const void* amap;  // A (tensor map, or the registry's per-slot map)
    const void* bmap;  // B
    const void* xmap;  // x rows, box height of the segment
    const void* ymap;  // y rows
    const T* bptr;  // rank 8: this adapter's B rows (one bulk copy per unit)
    int aid;  // adapter coordinate of the stacked maps (0 for registry maps)
    int tok;  // first token
    uint32_t box_bytes;  // one 64-column slice of x or y
  };
  auto seg_tma = [&](const DevSeg& s) -> SegTma {
    SegTma g;
    const int bi = box_index(clamp_rows(s.token_count));
    const int sl = slice_of(s);
    g.amap = registry ? s.a : static_cast<const void*>(sl ? &a.tmap_a_x[sl - 1] : &a.tmap_a);
    g.bmap = registry ? s.b : static_cast<const void*>(sl ? &a.tmap_b_x[sl - 1] : &a.tmap_b);
    g.xmap = &a.tmap_x[bi];
    g.ymap = sl ? &a.tmap_y_x[sl - 1][bi] : &a.tmap_y[bi];
    g.bptr = registry ? static_cast<const T*>(s.b)
                      : static_cast<const T*>(sl ? a.wb_base_x[sl - 1] : a.wb_base) +
                            static_cast<int64_t>(s.adapter_id) * (sl ? a.wb_stride_x[sl - 1] : a.wb_stride);
    g.aid = registry ? 0 : s.adapter_id;
    g.tok = s.token_start;
    g.box_bytes = (8u << bi) * 128u;
    return g;
  };
  // arm the stage's barrier (weights and activations) and load the weights of unit `sub`
  auto issue_w = [&](const SegTma& g, int sub, uint8_t* st, uint64_t* bar, uint64_t ef) {
    if (sub < nA) {
      const int k0 = kA0 + sub * C::KC;
      mbar_arrive_expect_tx(bar, 4 * C::ABOX + 4 * g.box_bytes);
      if (kFast || a.d_sliced) {
        tma_load_4d_ef(st, g.amap, 0, 0, k0 / kBoxCols, g.aid, bar, ef);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) tma_load_3d_ef(st + j * C::ABOX, g.amap, k0 + j * kBoxCols, 0, g.aid, bar, ef);
      }
    } else {
      const int oc = oB0 + (sub - nA) * C::W;
      if constexpr (C::BTMA) {
        // one 256-row box of B, rows past o zero-filled
        mbar_arrive_expect_tx(bar, 256 * R * 2 + (y_tma ? 4 * g.box_bytes : 0u));
        tma_load_3d_ef(st + 4 * C::XBOX, g.bmap, 0, oc, g.aid, bar, ef);
      } else {
        const int wc = min(C::W, a.o - oc);
        mbar_arrive_expect_tx(bar, wc * R * 2 + (y_tma ? 4 * g.box_bytes : 0u));
        bulk_g2s(st + 4 * C::XBOX, g.bptr + static_cast<int64_t>(oc) * R, wc * R * 2, bar);
      }
    }
  };
  // load the activations of unit `sub` (x for a shrink unit, y for an expand unit)
  auto issue_x = [&](const SegTma& g, int sub, uint8_t* st, uint64_t* bar) {
    if (sub < nA) {
      const int k0 = kA0 + sub * C::KC;
      if (kFast || a.d_sliced) {
        tma_load_3d(st + 4 * C::ABOX, g.xmap, 0, g.tok, k0 / kBoxCols, bar);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) tma_load_2d(st + 4 * C::ABOX + j * g.box_bytes, g.xmap, k0 + j * kBoxCols, g.tok, bar);
      }
    } else if (y_tma) {
      const int oc = oB0 + (sub - nA) * C::W;
      if (kFast || a.o_sliced) {
        tma_load_3d(st, g.ymap, 0, g.tok, oc / kBoxCols, bar);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) tma_load_2d(st + j * g.box_bytes, g.ymap, oc + j * kBoxCols, g.tok, bar);
      }
    }
  };
  const int first = min(S, total);  // stages issued before any is consumed
  // x of the shrink units may load before the dependency wait (fused live
  // calls whose caller promised that the previous kernel writes no x)
  const bool xpre = LF != 0 && !TPX && a.prefetch_weights && a.prefetch_inputs;
  if (warp == kProducerWarp) {
    // ======================= producer warp ===================================
    // Lanes 1-31 leave at once: a lane blocked in a dependency or cluster wait
    // holds up the whole warp, lane 0's pre-dependency issue included.
    if (lane != 0) return;
    {
      const uint64_t ef = l2_evict_first_policy();  // adapter weights stream through L2 once
      trace_rec_mark<TR>(trc, 9);
      // With prefetched weights the first `first` units get their weights
      // before the dependency wait, and their activations come from the
      // store thread once it is met; with prefetched inputs the x of every
      // shrink unit is loaded here without waiting, and only a y (expand
      // unit) needs the dependency. Without prefetch the dependency was met
      // before the table was read.
      bool met = !a.prefetch_weights;
      int u = 0, stage = 0;
      uint32_t round = 0;  // u = round * S + stage
      // The first `first` units are armed whatever happens: with prefetched
      // weights the store thread loads their activations unconditionally, and
      // the drain after an error waits for every armed stage.
      for (int sj = 0; sj < nmine && !(*s_bad && u >= first); ++sj) {
        const SegTma g = seg_tma(desc(sj));
        if constexpr (TR)
          if (trc && sj == 0) trc[8 + 11] = global_timer_ns();  // mark 11: first segment's TMA parameters
        for (int sub = 0; sub < ups; ++sub) {
          const bool x_free = xpre && sub < nA;  // activations that need no dependency wait
          if (!met && u >= first && !x_free) {
            trace_rec_mark<TR>(trc, 8);
            pdl_wait_prior();
            pdl_launch_dependents();
            trace_rec_mark<TR>(trc, 6);
            met = true;
          }
          if (u >= S) {
            if (!mbar_wait_bounded(&empty[stage], (round - 1) & 1, a.err)) *s_bad = 1;
            if (*s_bad) break;
          }
          uint8_t* st = stage_base + stage * C::STAGE;
          if constexpr (TR)
            if (trc && u == 0) trc[8 + 5] = global_timer_ns();  // mark 5: first unit's issue starts
          issue_w(g, sub, st, &full[stage], ef);
          if (met || x_free) issue_x(g, sub, st, &full[stage]);
          trace_rec_unit<TR>(trc, u, 7);
          if (u == 0) trace_rec_mark<TR>(trc, 10);
          *s_issued = u + 1;
          ++u;
          if (++stage == S) {
            stage = 0;
            ++round;
          }
        }
      }
      if (!met) {
        trace_rec_mark<TR>(trc, 8);
        pdl_wait_prior();
        pdl_launch_dependents();
        trace_rec_mark<TR>(trc, 6);
      }
    }
    cluster_wait();  // completes the start-up cluster barrier
    return;
  }

  if (warp == kStoreWarp) {
    // ===================== y store warp =======================================
    // For every expand stage whose y box is stored by TMA: wait until the
    // compute warps have written it (ydone), store it, wait until the store
    // has read shared memory, then free the stage for the producer.
    if (lane != 0) return;  // idle lanes leave (see the producer warp)
    if (a.prefetch_weights) {
      pdl_wait_prior();
      pdl_launch_dependents();
    }
    if (a.prefetch_weights) {
      // The first stages' activations, as soon as the dependency is met,
      // whether or not the producer has armed their barriers yet: bytes that
      // land first take the barrier's transaction count below zero (its
      // range is +-(2^20 - 1)), and the phase cannot complete before the
      // producer's arrival, which adds the stage's full byte count.
      // (with prefetched inputs the producer has loaded the shrink units' x)
      int u = 0;
      for (int sj = 0; sj < nmine && u < first; ++sj) {
        const SegTma g = seg_tma(desc(sj));
        for (int sub = 0; sub < ups && u < first; ++sub, ++u)
          if (!(xpre && sub < nA)) issue_x(g, sub, stage_base + u * C::STAGE, &full[u]);
      }
    }
    if (!do_ex) {
      cluster_wait();
      return;
    }
    uint32_t ypar = 0u;
    int u = 0;
    for (int sj = 0; sj < nmine; ++sj) {
      const DevSeg s = desc(sj);
      const int n = clamp_rows(s.token_count);
      u += nA;
      if (!y_by_tma(n)) {
        u += nB;
        continue;
      }
      const void* ymap = slice_of(s) ? &a.tmap_y_x[slice_of(s) - 1][box_index(n)] : &a.tmap_y[box_index(n)];
      for (int i = 0; i < nB; ++i, ++u) {
        const int stage = u % S;
        bool ok = !*s_bad;
        if (ok && !mbar_wait_bounded(&ydone[stage], (ypar >> stage) & 1u, a.err)) {
          *s_bad = 1;
          ok = false;
        }
        ypar ^= 1u << stage;
        if (ok) {
          tma_store_3d(ymap, 0, s.token_start, (oB0 + i * C::W) / kBoxCols, stage_base + stage * C::STAGE);
          bulk_commit();
          bulk_wait_read();
        }
        mbar_arrive_n(&empty[stage], kComputeWarps);
      }
    }
    bulk_wait_all();
    cluster_wait();
    return;
  }

  // ======================== compute warps ======================================
  // With prefetched inputs the shrink and the exchange run before the
  // dependency is met; it is awaited before the first expand stage.
  bool cdep = !a.prefetch_weights;
  auto compute_dep = [&]() {
    if (!cdep) {
      pdl_wait_prior();
      pdl_launch_dependents();
      tr.dep();
      cdep = true;
    }
  };
  if (!xpre) compute_dep();
  // tensor parallelism: the epoch of this launch's peer exchange (after the
  // dependency wait, so the previous launch's advance is visible)
  const int tp_epoch = TPX ? __ldcg(&a.tp_seq[0]) + 1 : 0;
  const int g = lane >> 2;
  const int c = lane & 3;
  int kc = 0;  // next stage-unit
  uint32_t cph = 0;  // cluster barrier phase
  bool peers_ready = false;  // the start-up cluster barrier has been waited for
  auto wait_peers = [&]() {
    if (!peers_ready) {
      cluster_wait();
      peers_ready = true;
    }
  };
  // Wait for stage `kc` (calling threads only), with the optional trace.
  auto wait_full = [&](int stage) -> bool {
    if (*s_bad) return false;
    const unsigned long long tw = tr.before_wait();
    const bool ok = mbar_wait_bounded(&full[stage], (kc / S) & 1, a.err);
    tr.after_wait(tw);
    if (!ok) *s_bad = 1;
    return ok;
  };

  // shared-memory offsets of this thread's ldmatrix rows, relative to a stage
  // (the same for every stage). The 128-byte swizzle XORs the 16-byte chunk
  // with the row's low three bits, so a tile 16 rows (or 8 tokens) further on
  // sits at a plain constant offset from the first: one base per k-step.
  constexpr int MT = R >= 16 ? R / 16 : 1;  // 16-row rank tiles of the shrink (rank 8: rows 8-15 unused)
  constexpr int KS = R >= 16 ? R / 16 : 1;  // expand k-steps of 16 (rank 8: one m16n8k8 step)
  uint32_t offA[2], offX[2], offB[KS];
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    {
      const int row = lane & 15;  // rank tile mt at + mt * 2048
      const int ch = (warp & 1) * 4 + 2 * ks + (lane >> 4);
      offA[ks] = (warp >> 1) * C::ABOX + row * 128 + (((ch ^ row) & 7) << 4);
    }
    {
      const int row = (lane & 7) + ((lane >> 4) << 3);  // token pair p at + p * 2048
      const int ch = (warp & 1) * 4 + 2 * ks + ((lane >> 3) & 1);
      offX[ks] = 4 * C::ABOX + row * 128 + (((ch ^ row) & 7) << 4);  // + box warp / 2 of x
    }
  }
  // expand, transposed: A operand = B rows (output columns), 16 per tile
  // (tile m at + m * 32 R: the swizzle bits of a row do not change by 16 rows)
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const int row = warp * 32 + (lane & 15);
    uint32_t lin = static_cast<uint32_t>(row * (2 * R) + (2 * ks + (lane >> 4)) * 16);
    if constexpr (C::BTMA) lin ^= (lin >> 3) & C::SWZ_MASK;
    offB[ks] = 4 * C::XBOX + lin;
  }
  // y (token rows t, this warp's 32 columns as four 8-column matrices; token
  // tile nt at + nt * 1024)
  const uint32_t offY = (lane & 7) * 128 + (((((warp & 1) * 4 + (lane >> 3)) ^ lane) & 7) << 4);  // + box warp / 2

  for (int sj = 0; sj < nmine; ++sj) {
    const DevSeg s = desc(sj);
    const int n = clamp_rows(s.token_count);
    if (tid == 0 && n == 0 && a.err) atomicOr(a.err, kErrBadSegment);
    // x / y boxes are (8 << box_index(n)) rows of 128 bytes; this warp reads box warp / 2
    const uint32_t xsl = static_cast<uint32_t>((warp >> 1) * ((8 << box_index(n)) * 128));
    const float alpha = registry ? s.alpha : a.scale;

    if (do_sh) {
      // ---- 1. shrink: D[rank, t] += A[rank, k] . x[t, k]^T. Warp w takes 32
      // columns of d of every stage (box w/2, half w%2) for all rank tiles and
      // token tiles, so no two warps read the same bytes; the 8 partials are
      // summed in a fixed order at the end of the segment.
      const bool have = nA > 0 && n > 0;
      float acc[MT][4][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.f;
      // the unit body is compiled for 1, 2 and 4 token tiles
      auto shrink_units = [&](auto ntc) {
        constexpr int nts = decltype(ntc)::value;  // 8-token tiles
        constexpr int np = (nts + 1) / 2;  // pairs of 8-token tiles
        for (int i = 0; i < nA; ++i, ++kc) {
          const int stage = kc % S;
          if (wait_full(stage) && have) {
            // all fragment loads first, then the MMAs (two warps per scheduler
            // cannot hide a load-use chain per k-step)
            const uint32_t sb = smem_u32(stage_base + stage * C::STAGE);
            uint32_t af[2][MT][4], bx[2][2][4];
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
#pragma unroll
              for (int mt = 0; mt < MT; ++mt)
                ldsm_x4(sb + offA[ks] + mt * 2048, af[ks][mt][0], af[ks][mt][1], af[ks][mt][2], af[ks][mt][3]);
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
#pragma unroll
              for (int p = 0; p < np; ++p)
                ldsm_x4(sb + xsl + offX[ks] + p * 2048, bx[ks][p][0], bx[ks][p][1], bx[ks][p][2], bx[ks][p][3]);
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
#pragma unroll
              for (int p = 0; p < np; ++p)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                  mma_k16<T>(acc[mt][2 * p], af[ks][mt], bx[ks][p][0], bx[ks][p][1]);
                  if (2 * p + 1 < nts) mma_k16<T>(acc[mt][2 * p + 1], af[ks][mt], bx[ks][p][2], bx[ks][p][3]);
                }
          }
          __syncwarp();
          tr.mark(5);
          if (lane == 0) mbar_arrive(&empty[stage]);
        }
      };
      switch ((n + 7) >> 3) {
        case 0:
        case 1: shrink_units(IntC<1>{}); break;
        case 2: shrink_units(IntC<2>{}); break;
        default: shrink_units(IntC<4>{}); break;
      }
      tr.seg(0, sj);
      // ---- 2. cross-warp sum and cluster exchange (push), in passes of
      // PROWS token rows: every warp parks the pass's rows of its partial in
      // a slot of its own; each thread adds the eight slots of its elements
      // in a fixed order and pushes the sums by st.async into this CTA's
      // receive slot on every peer, completing bytes on the peer's rx_full
      // barrier; it keeps its own sums in registers. A receive slot of a
      // segment parity is rewritten only after every peer has released it
      // (rx_free). Every CTA adds the ranks' partials in rank order, so all
      // of them get the same H.
      wait_peers();  // the peer's receive slots and barriers are initialised
      const int par = sj & 1;
      const uint32_t use = static_cast<uint32_t>(sj >> 1);  // uses of this parity so far
      float* rx = Rx + par * C::RXSLOTS * C::PSLOT;
      // this CTA's receive slot of rank i's partial (i != q), and its own slot on rank i
      auto rslot = [&](uint32_t i) -> uint32_t { return i < q ? i : i - 1; };
      auto tslot = [&](uint32_t i) -> uint32_t { return q < i ? q : q - 1; };
      if (CL > 1 && use > 0 && !*s_bad && !mbar_wait_cluster_bounded(&rx_free[par], (use - 1) & 1, a.err)) *s_bad = 1;
      constexpr int Q4 = R / 4;  // 16-byte chunks per partial row
      constexpr int PR = C::PROWS;
      constexpr int NP = 32 / PR;  // passes at most
      constexpr int KE = (PR * Q4 + kComputeThreads - 1) / kComputeThreads;  // elements per thread and pass
      const int nch = n * Q4;
      const int npass = (n + PR - 1) / PR;
      float4 own[NP][KE];
#pragma unroll
      for (int pp = 0; pp < NP; ++pp) {
        if (pp < npass) {
          if (pp > 0) named_sync(kBarCompute, kComputeThreads);  // the previous pass has read the slots
          {
            float* dst = Pw + warp * C::PWSLOT;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
              for (int jj = 0; jj < PR / 8; ++jj)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int r = mt * 16 + g + (e >> 1) * 8;
                  const int t = jj * 8 + 2 * c + (e & 1);  // row within the pass
                  if (r < R) dst[t * PITCH + r] = acc[mt][pp * (PR / 8) + jj][e];
                }
          }
          named_sync(kBarCompute, kComputeThreads);
          if (!*s_bad) {
            const int nq = min(PR, n - pp * PR) * Q4;
#pragma unroll
            for (int k = 0; k < KE; ++k) {
              const int e4 = tid + k * kComputeThreads;
              if (e4 < nq) {
                const int offw = (e4 / Q4) * PITCH + (e4 % Q4) * 4;
                float4 p[8];
#pragma unroll
                for (int w = 0; w < 8; ++w) p[w] = *reinterpret_cast<const float4*>(Pw + w * C::PWSLOT + offw);
                float4 v;
                v.x = ((p[0].x + p[1].x) + (p[2].x + p[3].x)) + ((p[4].x + p[5].x) + (p[6].x + p[7].x));
                v.y = ((p[0].y + p[1].y) + (p[2].y + p[3].y)) + ((p[4].y + p[5].y) + (p[6].y + p[7].y));
                v.z = ((p[0].z + p[1].z) + (p[2].z + p[3].z)) + ((p[4].z + p[5].z) + (p[6].z + p[7].z));
                v.w = ((p[0].w + p[1].w) + (p[2].w + p[3].w)) + ((p[4].w + p[5].w) + (p[6].w + p[7].w));
                own[pp][k] = v;
                const int off = pp * PR * PITCH + offw;  // in the segment's partial
                for (uint32_t i = 1; i < CL; ++i) {
                  const uint32_t peer = (q + i) % CL;
                  const uint32_t slot = smem_u32(rx + tslot(peer) * C::PSLOT + off);
                  st_async_v4(mapa(slot, peer), v, mapa(smem_u32(&rx_full[par]), peer));
                }
              }
            }
          }
        }
      }
      if (tid == 0) mbar_arrive_expect_tx(&rx_full[par], (CL - 1) * static_cast<uint32_t>(nch) * 16u);
      tr.seg(3, sj);
      if (CL > 1 && !*s_bad && !mbar_wait_cluster_bounded(&rx_full[par], use & 1, a.err)) *s_bad = 1;
      tr.seg(1, sj);
      if (!*s_bad) {
#pragma unroll
        for (int pp = 0; pp < NP; ++pp) {
          if (pp < npass) {
            const int nq = min(PR, n - pp * PR) * Q4;
#pragma unroll
            for (int k = 0; k < KE; ++k) {
              const int e4 = tid + k * kComputeThreads;
              if (e4 < nq) {
                const int t = pp * PR + e4 / Q4;
                const int off = t * PITCH + (e4 % Q4) * 4;
                float4 sum = q == 0 ? own[pp][k] : *reinterpret_cast<const float4*>(rx + rslot(0) * C::PSLOT + off);
                for (uint32_t i = 1; i < CL; ++i) {
                  const float4 v =
                      i == q ? own[pp][k] : *reinterpret_cast<const float4*>(rx + rslot(i) * C::PSLOT + off);
                  sum.x += v.x;
                  sum.y += v.y;
                  sum.z += v.z;
                  sum.w += v.w;
                }
                sum.x *= alpha;
                sum.y *= alpha;
                sum.z *= alpha;
                sum.w *= alpha;
                if (do_ex) {
                  *reinterpret_cast<float4*>(Hs + off) = sum;
                } else {
                  *reinterpret_cast<float4*>(a.h + static_cast<int64_t>(s.token_start + t) * R + (e4 % Q4) * 4) = sum;
                }
              }
            }
          }
        }
      }
      named_sync(kBarCompute, kComputeThreads);  // slots read, H complete
      if (TPX && do_ex) {
        // ---- 2b. tensor-parallel exchange over peer memory: H so far is
        // this rank's slice of d. The primary cluster of the segment (its
        // rank-0 CTA) writes it into every peer's mailbox, then raises its
        // flag there (the launch epoch); every CTA of the segment waits for
        // the peers' flags in its own mailbox and adds all ranks' partials in
        // rank order, so every rank gets the same H.
        const int W = a.tp_world, me = a.tp_rank, par = tp_epoch & 1;
        const int nq = n * (R / 4);
        if (q == 0 && seg_half <= 0) {
          // The rows and flag of parity(e) in a peer's mailbox were last
          // used in epoch e - 2: write them only once that peer has
          // finished its launch of epoch e - 2 (its done word, which it
          // raises in this rank's mailbox, even for a launch without
          // segments), so no rank overwrites a slot a slower peer still reads.
          if (tid < W && tid != me && tp_epoch > 2 && !*s_bad &&
              !wait_ge_sys(TpMail::done(a.tp_mail[me], W, a.tp_tmax, a.tp_smax, tid), tp_epoch - 2, a.err,
                           a.tp_wait_ns))
            *s_bad = 1;
          named_sync(kBarCompute, kComputeThreads);
          if (!*s_bad) {
            for (int e4 = tid; e4 < nq; e4 += kComputeThreads) {
              const int t = e4 / (R / 4), r0 = (e4 % (R / 4)) * 4;
              const float4 v = *reinterpret_cast<const float4*>(Hs + t * PITCH + r0);
              for (int p = 0; p < W; ++p)
                if (p != me)
                  *reinterpret_cast<float4*>(TpMail::row(a.tp_mail[p], W, a.tp_tmax, par, me, s.token_start + t) + r0) = v;
            }
          }
          __threadfence_system();  // this thread's rows reach the peers before any flag
          named_sync(kBarCompute, kComputeThreads);
          if (tid == 0)
            for (int p = 0; p < W; ++p)
              if (p != me)
                st_release_sys(TpMail::flag(a.tp_mail[p], W, a.tp_tmax, a.tp_smax, par, me, s.token_start), tp_epoch);
        }
        if (tid < W && tid != me && !*s_bad &&
            !wait_flag_sys(TpMail::flag(a.tp_mail[me], W, a.tp_tmax, a.tp_smax, par, tid, s.token_start), tp_epoch, a.err,
                           a.tp_wait_ns))
          *s_bad = 1;
        named_sync(kBarCompute, kComputeThreads);
        if (!*s_bad) {
          for (int e4 = tid; e4 < nq; e4 += kComputeThreads) {
            const int t = e4 / (R / 4), r0 = (e4 % (R / 4)) * 4;
            float4* hp = reinterpret_cast<float4*>(Hs + t * PITCH + r0);
            const float4 mine = *hp;
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p = 0; p < W; ++p) {
              const float4 v = p == me ? mine
                                       : __ldcg(reinterpret_cast<const float4*>(
                                             TpMail::row(a.tp_mail[me], W, a.tp_tmax, par, p, s.token_start + t) + r0));
              sum.x += v.x;
              sum.y += v.y;
              sum.z += v.z;
              sum.w += v.w;
            }
            *hp = sum;
          }
        }
        named_sync(kBarCompute, kComputeThreads);  // full H
      }
      // release the slots for the push two segments on (none after the last two)
      if (tid == 0 && CL > 1 && sj + 2 < nmine)
        for (uint32_t i = 1; i < CL; ++i) mbar_arrive_remote_relaxed(mapa(smem_u32(&rx_free[par]), (q + i) % CL));
      tr.seg(2, sj);
    } else if (do_ex) {
      // expand alone: H rows of the segment from global memory
      for (int e = tid; e < n * (R / 2); e += kComputeThreads) {
        const int row = e / (R / 2);
        const int col = (e % (R / 2)) * 2;
        *reinterpret_cast<float2*>(Hs + row * PITCH + col) =
            *reinterpret_cast<const float2*>(a.h + static_cast<int64_t>(s.token_start + row) * R + col);
      }
      named_sync(kBarCompute, kComputeThreads);
    }

    if (!do_ex || nB == 0) continue;
    compute_dep();
    T* yg = static_cast<T*>(a.y);
    {
      // ---- 3. expand over this CTA's slice of o. Transposed: D^T[o, t] =
      // B[o, :] . H[t, :]^T with M = 16 output columns per tile (A operand: B
      // rows from the stage, ldmatrix) and N = 8 tokens per tile (B operand:
      // H rows), so a segment of n tokens costs ceil(n / 8) token tiles. Warp
      // w owns output columns 32w..32w+31 of every stage. y comes in and goes
      // back through ldmatrix / stmatrix .trans, which turn the
      // [token][column] box into the accumulator layout and back. H enters
      // rounded to T (the weights' type, as the stock expand takes it).
      uint32_t hb[4][KS][2];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const float* hrow = Hs + (nt * 8 + g) * PITCH;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const int k0 = ks * 16 + 2 * c;
          const float2 x0 = *reinterpret_cast<const float2*>(hrow + k0);
          const float2 x1 = R >= 16 ? *reinterpret_cast<const float2*>(hrow + k0 + 8) : make_float2(0.f, 0.f);
          hb[nt][ks][0] = E::pack2(x0.x, x0.y);
          hb[nt][ks][1] = E::pack2(x1.x, x1.y);
        }
      }
      const bool tmy = y_by_tma(n);  // the store thread writes the y box back and frees the stage
      // the unit body is compiled for 1, 2 and 4 token tiles: no runtime
      // predication of the fragment loops
      auto expand_units = [&](auto ntc) {
        constexpr int ntn = decltype(ntc)::value;
        for (int i = 0; i < nB; ++i, ++kc) {
          const int stage = kc % S;
          if (wait_full(stage) && n > 0) {
            const uint8_t* st = stage_base + stage * C::STAGE;
            const int oc = oB0 + i * C::W;
            const int wc = min(C::W, a.o - oc);
            const uint32_t sb = smem_u32(st);
            // This warp's 32 columns of the y box: rows of 128 bytes, 16-byte
            // chunk ch of row t at ((ch ^ t) & 7) * 16 (the tensor map's 128-byte
            // swizzle). A y that the tensor maps cannot address (not 16-byte
            // aligned) is copied in here by the warp itself, element by element.
            uint8_t* ybox = const_cast<uint8_t*>(st) + xsl;
            const int colw0 = warp * 32;  // first column of this warp in the stage
            if (!y_tma) {
              const T* ysrc = yg + static_cast<int64_t>(s.token_start) * a.y_ld + yoff_of(s) + oc + colw0;
#pragma unroll 1
              for (int e = lane; e < n * 32; e += 32) {
                const int t = e >> 5, col = e & 31;
                const int ch = (warp & 1) * 4 + (col >> 3);
                *reinterpret_cast<T*>(ybox + t * 128 + (((ch ^ t) & 7) << 4) + (col & 7) * 2) =
                    colw0 + col < wc ? ysrc[static_cast<int64_t>(t) * a.y_ld + col] : E::from_f(0.f);
              }
              __syncwarp();
            }
            // the accumulators start at y (fp32): D = y + H . B^T, rounded
            // once; acc[m][nt] = output columns 16m.. of token tile nt
            float acc[2][ntn][4];
#pragma unroll
            for (int nt = 0; nt < ntn; ++nt) {
              uint32_t yf[4];
              ldsm_x4_t(sb + xsl + offY + nt * 1024, yf[0], yf[1], yf[2], yf[3]);
#pragma unroll
              for (int m = 0; m < 2; ++m) {
                const float2 f0 = E::unpack2(yf[2 * m]);
                const float2 f1 = E::unpack2(yf[2 * m + 1]);
                acc[m][nt][0] = f0.x;
                acc[m][nt][1] = f0.y;
                acc[m][nt][2] = f1.x;
                acc[m][nt][3] = f1.y;
              }
            }
            tr.mark(2);
            if constexpr (R >= 16) {
              constexpr int KB = KS > 2 ? 2 : KS;  // k-steps whose B fragments are loaded together
#pragma unroll
              for (int k0 = 0; k0 < KS; k0 += KB) {
                uint32_t bA[KB][2][4];
#pragma unroll
                for (int kk = 0; kk < KB; ++kk)
#pragma unroll
                  for (int m = 0; m < 2; ++m)
                    ldsm_x4(sb + offB[k0 + kk] + m * 32 * R, bA[kk][m][0], bA[kk][m][1], bA[kk][m][2], bA[kk][m][3]);
#pragma unroll
                for (int kk = 0; kk < KB; ++kk)
#pragma unroll
                  for (int nt = 0; nt < ntn; ++nt)
#pragma unroll
                    for (int m = 0; m < 2; ++m)
                      mma_k16<T>(acc[m][nt], bA[kk][m], hb[nt][k0 + kk][0], hb[nt][k0 + kk][1]);
              }
            } else {
              // rank 8: B rows of 16 bytes (linear); matrices 2m, 2m + 1 = rows 16m..16m+15
              uint32_t bf[4];
              ldsm_x4(sb + 4 * C::XBOX + (warp * 32 + lane) * 16, bf[0], bf[1], bf[2], bf[3]);
#pragma unroll
              for (int nt = 0; nt < ntn; ++nt)
#pragma unroll
                for (int m = 0; m < 2; ++m) mma_k8<T>(acc[m][nt], bf[2 * m], bf[2 * m + 1], hb[nt][0][0]);
            }
            tr.mark(3);
            // back into the y box in place; then the box goes to global memory
            // by one tensor store (store thread) or this warp's 16-byte row
            // chunks are stored directly (element by element for a y that is
            // not 16-byte addressable).
#pragma unroll
            for (int nt = 0; nt < ntn; ++nt)
              stsm_x4_t(sb + xsl + offY + nt * 1024, E::pack2(acc[0][nt][0], acc[0][nt][1]),
                        E::pack2(acc[0][nt][2], acc[0][nt][3]), E::pack2(acc[1][nt][0], acc[1][nt][1]),
                        E::pack2(acc[1][nt][2], acc[1][nt][3]));
            tr.mark(4);
            if (tmy) {
              fence_proxy_async_smem();  // the tensor store reads these writes
            } else if (y_tma) {
              __syncwarp();
              const int sub = lane & 3;
              const int colw = colw0 + sub * 8;  // column of this lane's 16-byte chunk in the stage
              const int chunk = (warp & 1) * 4 + sub;
              T* ycol = yg + static_cast<int64_t>(s.token_start) * a.y_ld + yoff_of(s) + oc + colw;
              // o and the stage columns are multiples of 8: a chunk lies
              // wholly inside the output range or wholly outside it
              if (colw < wc) {
                int4 out[ntn];
#pragma unroll
                for (int it = 0; it < ntn; ++it) {
                  const int row = (lane >> 2) + 8 * it;
                  if (row < n) out[it] = *reinterpret_cast<const int4*>(ybox + row * 128 + (((chunk ^ row) & 7) << 4));
                }
#pragma unroll
                for (int it = 0; it < ntn; ++it) {
                  const int row = (lane >> 2) + 8 * it;
                  if (row < n) *reinterpret_cast<int4*>(ycol + static_cast<int64_t>(row) * a.y_ld) = out[it];
                }
              }
            } else {
              __syncwarp();
              T* ydst = yg + static_cast<int64_t>(s.token_start) * a.y_ld + yoff_of(s) + oc + colw0;
#pragma unroll 1
              for (int e = lane; e < n * 32; e += 32) {
                const int t = e >> 5, col = e & 31;
                const int ch = (warp & 1) * 4 + (col >> 3);
                if (colw0 + col < wc)
                  ydst[static_cast<int64_t>(t) * a.y_ld + col] =
                      *reinterpret_cast<const T*>(ybox + t * 128 + (((ch ^ t) & 7) << 4) + (col & 7) * 2);
              }
            }
          }
          __syncwarp();
          tr.mark(5);
          if (lane == 0) mbar_arrive(tmy ? &ydone[stage] : &empty[stage]);
        }
      };
      switch ((n + 7) >> 3) {
        case 0:
        case 1: expand_units(IntC<1>{}); break;
        case 2: expand_units(IntC<2>{}); break;
        default: expand_units(IntC<4>{}); break;
      }
    }
  }
  // Peers arrive on this CTA's barrier until they pass this one, so the
  // shared memory must outlive it. Their other remote accesses (pushes into
  // the receive slots, slot releases) were all observed before: every push
  // was consumed, and the releases of the last two segments are not sent.
  // No data crosses this barrier, so it needs no release fence (a fence
  // would wait for this thread's outstanding y stores).
  wait_peers();
  if (CL > 1 && !cluster_barrier_relaxed_bounded(cbar, cph, CL, kBarCompute, kComputeThreads, a.err)) *s_bad = 1;
  if (*s_bad) {
    // drain: copies may still be in flight into stages issued but not consumed
    named_sync(kBarCompute, kComputeThreads);
    if (tid == 0) {
      const int issued = *s_issued;
      for (int u = max(0, issued - S); u < issued; ++u) mbar_wait_bounded(&full[u % S], (u / S) & 1, nullptr, kDrainNs);
    }
  }
  if (TPX) {
    // every wait of this CTA on the peers is over: count it; the last CTA
    // advances the epoch for the next exchange launch
    named_sync(kBarCompute, kComputeThreads);
    if (tid == 0 && atomicAdd(&a.tp_seq[1], 1) == static_cast<int>(gridDim.x) - 1) {
      a.tp_seq[1] = 0;
      __threadfence();
      atomicExch(&a.tp_seq[0], tp_epoch);
      // tell every peer that this rank has read all it will read of this
      // epoch (also for a launch without segments)
      for (int p = 0; p < a.tp_world; ++p)
        if (p != a.tp_rank) st_release_sys(TpMail::done(a.tp_mail[p], a.tp_world, a.tp_tmax, a.tp_smax, a.tp_rank), tp_epoch);
    }
  }
  tr.finish();
}

// --------------------------------------------------------------------------
// launchers

namespace {

template <typename T, int R, bool TR, int LF, bool TPX = false>
struct ApplyKernel {
  using C = ApplyCfg<R, LF == 4 ? 4 : 2>;
  static bool prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return true;
    if (cudaFuncSetAttribute(apply_kernel<T, R, TR, LF, TPX>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return false;
    done.fetch_or(bit);
    return true;
  }

  static cudaError_t launch(const ApplyArgs& a, const LaunchCfg& lc) {
    if (lc.cluster > C::CLMAX) return cudaErrorInvalidValue;
    if (!prepare()) return cudaGetLastError();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(lc.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = lc.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = lc.cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = lc.pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, apply_kernel<T, R, TR, LF, TPX>, a);
  }

  static int max_grid(int cluster) {
    if (cluster > C::CLMAX) return 0;  // receive slots exist for CLMAX ranks
    if (!prepare()) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cluster * 64);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nclusters = 0;
    if (cudaOccupancyMaxActiveClusters(&nclusters, apply_kernel<T, R, TR, LF, TPX>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return nclusters * cluster;
  }
};

template <typename T, int R>
cudaError_t apply_variant(const ApplyArgs& a, const LaunchCfg& lc) {
  const bool live_fused = a.mode == kModeFused && !a.registry && a.y_tma;
  if (a.tp_world > 1) {
    // row-parallel exchange over peer memory (untraced): live fused single-slice calls
    if (!live_fused || a.nslices > 1) return cudaErrorInvalidValue;
    return ApplyKernel<T, R, false, 1, true>::launch(a, lc);
  }
  // the live fused instantiations are compiled for clusters of 2 and sliced maps
  const bool fast = live_fused && lc.cluster == 2 && a.d_sliced && a.o_sliced;
  const int lf = fast ? (a.nslices > 1 ? 2 : 1) : 0;
  if (a.trace) return lf == 1 ? ApplyKernel<T, R, true, 1>::launch(a, lc) : ApplyKernel<T, R, true, 0>::launch(a, lc);
  // few-segment calls on clusters of 4 (ranks 8-32; the host picks it)
  if (lf == 0 && live_fused && lc.cluster == 4 && a.d_sliced && a.o_sliced && a.nslices <= 1 && R <= 32 && !a.trace)
    return ApplyKernel<T, R <= 32 ? R : 32, false, 4>::launch(a, lc);
  if (lf == 1) return ApplyKernel<T, R, false, 1>::launch(a, lc);
  if (lf == 2) return ApplyKernel<T, R, false, 2>::launch(a, lc);
  return ApplyKernel<T, R, false, 0>::launch(a, lc);
}

template <typename T>
cudaError_t apply_by_rank(int rank, const ApplyArgs& a, const LaunchCfg& lc) {
  switch (rank) {
    case 8: return apply_variant<T, 8>(a, lc);
    case 16: return apply_variant<T, 16>(a, lc);
    case 32: return apply_variant<T, 32>(a, lc);
    case 64: return apply_variant<T, 64>(a, lc);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
int max_grid_by_rank(int rank, int cluster) {
  switch (rank) {
    case 8: return ApplyKernel<T, 8, false, 0>::max_grid(cluster);
    case 16: return ApplyKernel<T, 16, false, 0>::max_grid(cluster);
    case 32: return ApplyKernel<T, 32, false, 0>::max_grid(cluster);
    case 64: return ApplyKernel<T, 64, false, 0>::max_grid(cluster);
    default: return 0;
  }
}

}  // namespace

cudaError_t launch_apply(int dtype, int rank, const ApplyArgs& a, const LaunchCfg& lc) {
  return dtype == 1 ? apply_by_rank<__nv_bfloat16>(rank, a, lc) : apply_by_rank<__half>(rank, a, lc);
}

int apply_max_grid(int dtype, int rank, int cluster) {
  return dtype == 1 ? max_grid_by_rank<__nv_bfloat16>(rank, cluster) : max_grid_by_rank<__half>(rank, cluster);
}

int apply_max_grid4(int dtype, int rank) {
  if (rank > 32) return 0;
  switch (rank) {
    case 8: return dtype == 1 ? ApplyKernel<__nv_bfloat16, 8, false, 4>::max_grid(4) : ApplyKernel<__half, 8, false, 4>::max_grid(4);
    case 16: return dtype == 1 ? ApplyKernel<__nv_bfloat16, 16, false, 4>::max_grid(4) : ApplyKernel<__half, 16, false, 4>::max_grid(4);
    case 32: return dtype == 1 ? ApplyKernel<__nv_bfloat16, 32, false, 4>::max_grid(4) : ApplyKernel<__half, 32, false, 4>::max_grid(4);
    default: return 0;
  }
}

}  // namespace wp
