// wp_apply.cu -- the grouped multi-LoRA apply kernel for sm_100a.
//
// Semantics (reference: tests/correctness/reference_bgmv.py:4-18, the math of
// bgmv_shrink_kernel / bgmv_expand_kernel in csrc/kernels/warp_pipe_r32.cu:56-200
// and their DSAK twins :280-423):
//   shrink:  H[t, :] = alpha * X[t, :] . A_seg^T      (fp32, never rounded)
//   expand:  Y[t, j] = round(Y[t, j] + H[t, :] . B_seg[j, :])
// for every token t inside a segment of the table; other rows are untouched.
//
// One launch does both halves of one LoRA layer call. The grid is persistent
// (a fixed number of co-resident CTAs, so the launch can be captured in a CUDA
// graph) and organised in thread-block clusters of CL CTAs (CL = 2 on B200);
// the segmenter's ClusterPlan gives each cluster its segments (whole
// segments on the lowest clusters, helper clusters that take half of the
// output columns of the largest segments when clusters are left over). For one
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
// Two compute variants share this skeleton (template flag DEC):
//   DEC = true, the production decode kernel: the compute warps run
//     mma.sync m16n8k16 (bf16/fp16 in, fp32 accumulate) on fragments loaded
//     with ldmatrix from the swizzled TMA boxes. Shrink: D[rank, token] +=
//     A . x^T, warp w owning 32 columns of every stage, the eight warp
//     partials added in a fixed order. Expand, transposed: D^T[o, t] = y +
//     B[o, :] . H[t, :]^T with M = 16 output columns and N = 8 tokens per
//     tile, y entering the accumulator through ldmatrix.trans and leaving
//     through stmatrix.trans. The stage bodies are compiled once per
//     token-tile count (1-4 tiles of 8 tokens). Decode segments are at most
//     32 tokens, where one tcgen05.mma costs as much as a whole mma.sync stage.
//   DEC = false, the tcgen05 variant: a dedicated MMA warp issues
//     tcgen05.mma with the accumulators in tensor memory (described below).
//     Selected by wp_config.kernel = 3; kept as the tensor-memory
//     alternative for the decode shapes.
// Prefill-sized runs of one adapter (>= 128 tokens) have their own tcgen05
// GEMM kernels in wp_prefill.cu.
//
// Warp roles, handing off only through mbarriers:
//   warp 8 (producer): lane 0 issues every TMA load of the CTA into a ring of
//     STAGES shared-memory stages ("full" barriers) and refills a stage when
//     its "empty" barrier fires; it runs ahead across segment and phase
//     boundaries (the expand-phase loads of B and y do not depend on H).
//   warp 9: DEC = true: the y-store thread (a segment that fills its box
//     exactly leaves through one tensor store); DEC = false: the MMA warp.
//     Lane 0 issues every tcgen05.mma. Shrink stages are freed by
//     the MMA commit itself; accumulators are handed to the compute warps by
//     commits ("sh_full", "acc_full") and handed back after their TMEM reads
//     ("sh_free", "acc_free"); two expand accumulators let the MMAs of the
//     next stage run while the compute warps drain the current one.
//   warps 0-7 (compute): the mma.sync math (DEC = true) or the accumulator
//     reads (DEC = false), the cluster exchange, y add and store, and the
//     release of expand stages.
//
// Data movement: A and x arrive as tiled tensor loads (cp.async.bulk.tensor)
// of 64-column boxes with the 128-byte swizzle -- conflict-free fragment
// loads, zero fill past the ends of d and T; x and y boxes are 8, 16 or 32
// rows high to match the segment. B arrives as tensor boxes of 128 rows whose
// swizzle matches its 2r-byte rows (rank 8: one 1-D bulk copy). One stage
// carries 256 elements of d (shrink) or 256 output columns (expand). The
// cluster's segment descriptors are cached in shared memory once per launch.
//
// tcgen05 variant (DEC = false), math on the 5th-generation tensor cores
// (tcgen05.mma, issued by one thread, accumulating in tensor memory):
//   shrink: D[rank, t] += A[rank, k] . x[t, k]^T per 64-column box, M = 64
//     (rows past r are never read back), N = tokens rounded up to 8, K = 16
//     per instruction, over the CTA's slice of d. The MMA commit itself frees the
//     stage for the producer, so the compute warps do no per-stage work.
//   expand (ranks 16-64): D[t, o] = H[t, :] . B[o, :]^T with M = 128 rows
//     (the segment's tokens, spread over the four TMEM lane quarters), N = 256
//     output columns (a whole stage) and K = r; B in shared memory in the TMA
//     swizzle of its 2r-byte rows. Each compute lane reads 32 consecutive
//     output columns of one token with tcgen05.ld, adds y (16-byte reads of
//     the swizzled y box) and stores 16 bytes at a time.
//   expand (rank 8, K < 16): mma.sync m16n8k8 on the CUDA-core warps.
// H enters the expand MMAs as a 16-bit high part plus a 16-bit residual,
// which keeps ~16 mantissa bits of the fp32 H; y is rounded once.
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
constexpr int kMmaWarp = kComputeWarps + 1;  // tcgen05.mma issue
constexpr int kThreads = kComputeThreads + 64;  // + the producer and MMA warps
constexpr int kBarCompute = 1;  // named barrier of the compute warps
constexpr int kDescCache = 64;  // segment descriptors cached per CTA
constexpr int kSnakeMax = 128;  // tables up to this size are dealt by decreasing token count
constexpr unsigned long long kDrainNs = 10000000ull;  // 10 ms per stage when draining after an error

constexpr int kSmemMax = 232448;  // dynamic shared memory per CTA (227 KB)

template <int N>
struct IntC {
  static constexpr int value = N;
};

// DEC = true selects the decode variant: shrink and expand on warp-level
// mma.sync in the compute warps (no tensor memory, no MMA warp); false selects
// tcgen05 (shrink always, expand for ranks 16-64).
template <int R, bool DEC>
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
  static constexpr bool TC = !DEC && R >= 16;  // expand on tcgen05 (K = r must be a multiple of 16)
  static constexpr bool BTMA = R >= 16;  // B as swizzled tensor boxes (rank 8: one linear bulk copy)
  static constexpr int HT = 32 * R * 2;  // one 16-bit H tile (hi or lo): 32 token rows, swizzled like B
  static constexpr int SWZ_BYTES = R * 2;  // B / H row bytes = swizzle span
  static constexpr uint32_t SWZ_MASK = R == 64 ? 0x70u : (R == 32 ? 0x30u : 0x10u);
  static constexpr uint32_t UMMA_LAYOUT = R == 64 ? 2u : (R == 32 ? 4u : 6u);
  static constexpr int DPITCH = 256 + 4;  // floats per row of the expand result tile Ds (bank-shifted rows)
  static constexpr int DS = TC ? 32 * DPITCH * 4 : 0;
  // decode variant: shrink partials of the 8 compute warps (32 tokens x PITCH floats each) for the cross-warp sum
  static constexpr int PSLOT = 32 * PITCH;
  static constexpr int PW = DEC ? 8 * PSLOT * 4 : 0;
  // decode variant: receive slots of the cluster exchange, [2 segment parities][CLMAX ranks]
  static constexpr int CLMAX = DEC ? 2 : 4;
  static constexpr int RX = DEC ? 2 * CLMAX * PSLOT * 4 : 0;
  static constexpr int FIXED = OFF_END + DS + PW + RX + 1024 + (TC ? 2 * HT : 0);
  static constexpr int FIT = (kSmemMax - FIXED) / STAGE;
  static constexpr int STAGES = DEC ? (FIT > 8 ? 8 : FIT) : (R == 64 ? 2 : (R == 32 ? 5 : (R == 16 ? 7 : 8)));
  static constexpr int SMEM = FIXED + STAGES * STAGE;
  static_assert(STAGES >= 2 && STAGES <= 8 && SMEM <= kSmemMax, "shared memory budget");
  static_assert(32 * PITCH * 4 >= kComputeWarps * 128, "the P tile holds one scratch row per compute warp");
  static_assert(32 * PITCH * 4 >= 2 * kSnakeMax * 4, "the H tile holds the table-ordering scratch");
  static_assert(!DEC || PW >= 4 * kSnakeMax * 4, "the partial slots hold the table-ordering scratch");
};

template <typename T, int R, bool DEC, bool TR, int LF, bool TPX = false>
__global__ void __launch_bounds__(kThreads, 1) apply_kernel(const __grid_constant__ ApplyArgs a) {
  using C = ApplyCfg<R, DEC>;
  using E = Elem<T>;
  constexpr int S = C::STAGES;
  constexpr int PITCH = C::PITCH;

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + 128);
  uint64_t* cbar = reinterpret_cast<uint64_t*>(smem + 256);
  volatile int* s_bad = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS);
  volatile int* s_issued = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS + 4);
  volatile int* s_armed = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS + 8);  // stages armed by the producer
  int4* sdesc = reinterpret_cast<int4*>(smem + C::OFF_DESC);
  float* Ps = reinterpret_cast<float*>(smem + C::OFF_P);
  float* Hs = reinterpret_cast<float*>(smem + C::OFF_H);
  // MMA warp <-> compute warps handoffs
  uint64_t* sh_full = reinterpret_cast<uint64_t*>(smem + 264);  // shrink accumulator complete (commit)
  uint64_t* sh_free = reinterpret_cast<uint64_t*>(smem + 272);  // shrink accumulator read (8 warps)
  uint64_t* ht_full = reinterpret_cast<uint64_t*>(smem + 280);  // H tiles written (8 warps)
  uint64_t* acc_full = reinterpret_cast<uint64_t*>(smem + 288);  // [2] expand accumulator complete (commit)
  uint64_t* acc_free = reinterpret_cast<uint64_t*>(smem + 304);  // [2] expand accumulator read (8 warps)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + 336);
  float* Ds = reinterpret_cast<float*>(smem + C::OFF_END);  // expand results of one stage (fp32)
  float* Pw = reinterpret_cast<float*>(smem + C::OFF_END + C::DS);  // decode: cross-warp shrink partials
  float* Rx = reinterpret_cast<float*>(smem + C::OFF_END + C::DS + C::PW);  // decode: cluster receive slots
  uint64_t* rx_full = reinterpret_cast<uint64_t*>(smem + 352);  // [2] all peers' partials landed (tx count)
  uint64_t* rx_free = reinterpret_cast<uint64_t*>(smem + 368);  // [2] every peer has read my partial
  uint64_t* ydone = reinterpret_cast<uint64_t*>(smem + 384);  // [S] decode: y box of the stage final (8 warps)
  uint8_t* ht_base = align1024(smem + C::OFF_END + C::DS + C::PW + C::RX);  // H hi / lo tiles (tcgen05 expand)
  uint8_t* stage_base = ht_base + (C::TC ? 2 * C::HT : 0);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const bool producer = warp == kProducerWarp;
  // LF: the live fused call with a tensor-map-aligned y (the serving hot
  // path), compiled without the other modes' branches; 1 = one slice,
  // 2 = several slices (add_lora_packed_nslice)
  const bool registry = !LF && a.registry != 0;
  const bool y_tma = LF || a.y_tma != 0;
  const int nslices = LF == 1 ? 1 : a.nslices;
  const uint32_t q = cluster_ctarank();
  const uint32_t CL = cluster_nctarank();
  const int cid = static_cast<int>(cluster_id_x());
  const int G = static_cast<int>(cluster_count_x());
  std::conditional_t<TR, Trace, TraceOff> tr;
  tr.init(a.trace, tid == 0);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], DEC ? kComputeWarps : 1);  // decode: every compute warp frees the stage
      mbar_init(&ydone[s], kComputeWarps);
    }
    mbar_init(cbar, CL);
    mbar_init(sh_full, 1);
    mbar_init(sh_free, kComputeWarps);
    mbar_init(ht_full, kComputeWarps);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_free[b], kComputeWarps);
      mbar_init(&rx_full[b], 1);
      mbar_init(&rx_free[b], CL > 1 ? CL - 1 : 1);
    }
    *s_bad = 0;
    *s_issued = 0;
    *s_armed = 0;
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
  // TMEM: shrink accumulator (columns 0-31) and two expand accumulators of two
  // 128 x 32 halves each (columns 64-127 and 128-191)
  const bool use_tmem = !DEC && ((a.mode & kModeShrink) || (C::TC && (a.mode & kModeExpand)));
  if (use_tmem && warp == 0) tmem_alloc(s_tmem, 256);
  if (use_tmem) tc_fence_before();
  __syncthreads();
  if (use_tmem) tc_fence_after();
  cluster_sync_hw();  // every CTA's cluster barrier is initialised before anyone arrives on it

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
    return DEC && y_tma && a.o_sliced && (n == 8 || n == 16 || n == 32);
  };

  // ---- segment table of this cluster (all threads) -------------------------
  int nmine = 0;
  int seg_half = -1;  // helper pairs: which half of the output columns this cluster expands (0 / 1), else -1
  // Segments per cluster, for small tables (decode) ordered by decreasing
  // token count. Fewer segments than clusters: the largest segments get a
  // helper cluster each, and the pair splits the segment's output columns
  // (both clusters run the shrink; the second reads A mostly from L2); the
  // whole segments take the lowest clusters, which the hardware dispatches
  // first (with programmatic dependent launch they also start first). More
  // segments than clusters: "snake" dealing (round r gives cluster c the
  // segment at sorted position r*G + c or r*G + G-1-c, alternating, with the
  // last, partial round running forward), pairing large segments with small
  // ones. Larger tables go round robin (cluster c takes c, c + G, ...).
  // The segmenter's plan (one load round: header, this cluster's count,
  // half and descriptors together) replaces all of this when it was made for
  // this launch's cluster count.
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
    if (tid == 0) sh[0] = __ldcg(&a.plan->hdr);
    if (tid == 1) reinterpret_cast<int*>(sh + 1)[0] = __ldcg(&a.plan->count[min(cid, kPlanMaxClusters - 1)]);
    if (tid == 2) reinterpret_cast<int*>(sh + 1)[1] = __ldcg(&a.plan->half[min(cid, kPlanMaxClusters - 1)]);
    if (tid >= 32 && tid < 32 + 2 * kPlanRounds) {
      const int j = tid - 32;
      const int slot = min((j >> 1) * G + cid, kPlanRounds * kPlanMaxClusters - 1);
      sdesc[j] = __ldcg(reinterpret_cast<const int4*>(&a.plan->seg[slot]) + (j & 1));
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
  // Multi-slice calls: virtual segment v is segment v % nseg of slice
  // v / nseg; its descriptor carries the slice in the (live-mode unused)
  // alpha field.
  const int S_sl = nslices > 1 ? nslices : 1;
  int nseg_t = 0;  // segments of the table (not virtual)
  auto put_desc = [&](int slot, int v) {
    const int seg = v % nseg_t;
    int4 x0 = __ldcg(reinterpret_cast<const int4*>(a.segs + seg));
    const int4 x1 = __ldcg(reinterpret_cast<const int4*>(a.segs + seg) + 1);
    if (S_sl > 1) x0.w = v / nseg_t;
    sdesc[2 * slot] = x0;
    sdesc[2 * slot + 1] = x1;
  };
  auto read_table = [&]() {
    if (S_sl == 1 && a.plan && read_plan()) return;
    nseg_t = __ldcg(a.num_segs);
    const int nseg = S_sl * nseg_t;  // virtual segments
    constexpr int kSortMax = DEC ? 2 * kSnakeMax : kSnakeMax;  // scratch: decode: the partial slots; else the H tile
    int* cnt = DEC ? reinterpret_cast<int*>(Pw) : reinterpret_cast<int*>(Hs);
    int* order = cnt + kSortMax;
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
      const int helpers = min(nseg, G - nseg);
      const int V = nseg + helpers;
      const int solo = nseg - helpers;  // whole segments first (lowest clusters start first), then helper pairs
      nmine = cid < V ? 1 : 0;
      if (nmine) {
        const int pos = cid < solo ? helpers + cid : (cid - solo) >> 1;
        const int half = cid < solo ? -1 : ((cid - solo) & 1);
        seg_half = half;
        const int ob = half == 1 ? osplit : 0;
        const int olen = half < 0 ? a.o : (half == 0 ? osplit : a.o - osplit);
        const int osl = (olen + static_cast<int>(CL) - 1) / static_cast<int>(CL);
        const int oslr = (osl + C::W - 1) / C::W * C::W;
        oB0 = ob + static_cast<int>(q) * oslr;
        nB = (max(0, min(oslr, ob + olen - oB0)) + C::W - 1) / C::W;
        ups = nA + nB;
        if (tid == 0) put_desc(0, order[pos]);
      }
    } else if (G > 1 && nseg > G && nseg <= kSortMax) {
      sort_by_size();
      const int rounds = (nseg + G - 1) / G;
      nmine = 0;
      // snake dealing whose last (partial) round runs forward: the clusters
      // holding one segment more are the lowest, which start first
      auto pos_of = [&](int r) { return r * G + (((rounds - 1 - r) & 1) ? G - 1 - cid : cid); };
      for (int r = 0; r < rounds; ++r)
        if (pos_of(r) < nseg) nmine = r + 1;  // positions grow with r, so the items are rounds 0..nmine-1
      for (int r = tid; r < min(nmine, kDescCache); r += kThreads) put_desc(r, order[pos_of(r)]);
    } else {
      nmine = nseg > cid ? (nseg - cid + G - 1) / G : 0;
      for (int r = tid; r < min(nmine, kDescCache); r += kThreads) put_desc(r, cid + r * G);
    }
    __syncthreads();
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
  if (tid == 0) trace_mark_t<TR>(a.trace, 7);
  const int total = nmine * ups;
  const uint32_t tbase = use_tmem ? *s_tmem : 0u;
  const uint32_t t_sh = tbase;
  constexpr uint32_t kAbf = E::is_bf16 ? 1u : 0u;

  // TMA issue of stage-unit u into `stage`. parts: 1 = arm the stage's
  // barrier (weights and activations) and load the weights, 2 = load the
  // activations. ef: the L2 evict-first policy of the weight loads.
  auto issue = [&](int u, int stage, int parts, uint64_t ef) {
    const DevSeg s = desc(u / ups);
    const int sub = u % ups;
    const int n = clamp_rows(s.token_count);
    const int bi = box_index(n);
    const uint32_t box_bytes = (8u << bi) * 128u;  // one 64-column slice of x or y
    uint8_t* st = stage_base + stage * C::STAGE;
    uint64_t* bar = &full[stage];
    if (sub < nA) {
      const int k0 = kA0 + sub * C::KC;
      if (parts & 1) {
        mbar_arrive_expect_tx(bar, 4 * C::ABOX + 4 * box_bytes);
        const int sl = slice_of(s);
        const void* amap = registry ? s.a : static_cast<const void*>(sl ? &a.tmap_a_x[sl - 1] : &a.tmap_a);
        const int aid = registry ? 0 : s.adapter_id;
        if (a.d_sliced) {
          tma_load_4d_ef(st, amap, 0, 0, k0 / kBoxCols, aid, bar, ef);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) tma_load_3d_ef(st + j * C::ABOX, amap, k0 + j * kBoxCols, 0, aid, bar, ef);
        }
      }
      if (parts & 2) {
        if (a.d_sliced) {
          tma_load_3d(st + 4 * C::ABOX, &a.tmap_x[bi], 0, s.token_start, k0 / kBoxCols, bar);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tma_load_2d(st + 4 * C::ABOX + j * box_bytes, &a.tmap_x[bi], k0 + j * kBoxCols, s.token_start, bar);
        }
      }
    } else {
      const int oc = oB0 + (sub - nA) * C::W;
      const int wc = min(C::W, a.o - oc);
      if (parts & 1) {
        if constexpr (C::BTMA) {
          // one 256-row box of B, rows past o zero-filled
          mbar_arrive_expect_tx(bar, 256 * R * 2 + (y_tma ? 4 * box_bytes : 0u));
          const int sl = slice_of(s);
          const void* bmap = registry ? s.b : static_cast<const void*>(sl ? &a.tmap_b_x[sl - 1] : &a.tmap_b);
          const int bid = registry ? 0 : s.adapter_id;
          tma_load_3d_ef(st + 4 * C::XBOX, bmap, 0, oc, bid, bar, ef);
        } else {
          mbar_arrive_expect_tx(bar, wc * R * 2 + (y_tma ? 4 * box_bytes : 0u));
          const int sl = slice_of(s);
          const T* B = registry ? static_cast<const T*>(s.b)
                                  : static_cast<const T*>(sl ? a.wb_base_x[sl - 1] : a.wb_base) +
                                        static_cast<int64_t>(s.adapter_id) * (sl ? a.wb_stride_x[sl - 1] : a.wb_stride);
          bulk_g2s(st + 4 * C::XBOX, B + static_cast<int64_t>(oc) * R, wc * R * 2, bar);
        }
      }
      if ((parts & 2) && y_tma) {
        if (a.o_sliced) {
          tma_load_3d(st, slice_of(s) ? &a.tmap_y_x[slice_of(s) - 1][bi] : &a.tmap_y[bi], 0, s.token_start,
                      oc / kBoxCols, bar);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tma_load_2d(st + j * box_bytes, slice_of(s) ? &a.tmap_y_x[slice_of(s) - 1][bi] : &a.tmap_y[bi],
                        oc + j * kBoxCols, s.token_start, bar);
        }
      }
    }
  };
  const int first = min(S, total);  // stages issued before any is consumed
  if (warp == kProducerWarp) {
    // ======================= producer warp ===================================
    if (lane == 0) {
      const uint64_t ef = l2_evict_first_policy();  // adapter weights stream through L2 once
      trace_mark_t<TR>(a.trace, 9);
      if (a.prefetch_weights) {
        for (int u = 0; u < first; ++u) {
          issue(u, u, 1, ef);
          if constexpr (DEC) {
            __threadfence_block();
            *s_armed = u + 1;  // the store thread may load this stage's activations
          }
          trace_unit_t<TR>(a.trace, u, 7);
          if (u == 0) trace_mark_t<TR>(a.trace, 10);
        }
        trace_mark_t<TR>(a.trace, 8);
        pdl_wait_prior();
        pdl_launch_dependents();
        trace_mark_t<TR>(a.trace, 6);
        // decode variant: the store thread loads the first stages'
        // activations right after the dependency wait, while this thread is
        // still issuing weights
        if constexpr (!DEC)
          for (int u = 0; u < first; ++u) issue(u, u, 2, ef);
      } else {
        for (int u = 0; u < first; ++u) issue(u, u, 3, ef);
      }
      *s_issued = first;
      for (int u = first; u < total; ++u) {
        const int stage = u % S;
        if (!mbar_wait_bounded(&empty[stage], ((u / S) - 1) & 1, a.err)) *s_bad = 1;
        if (*s_bad) break;
        issue(u, stage, 3, ef);
        trace_unit_t<TR>(a.trace, u, 7);
        *s_issued = u + 1;
      }
    } else if (a.prefetch_weights) {
      pdl_wait_prior();
      pdl_launch_dependents();
    }
    return;
  }

  if (warp == kMmaWarp) {
    // ========================= MMA warp ======================================
    if (a.prefetch_weights) {
      pdl_wait_prior();
      pdl_launch_dependents();
    }
    auto wait_ok = [&](uint64_t* bar, uint32_t parity) -> bool {
      if (*s_bad) return false;
      const bool ok = mbar_wait_bounded(bar, parity, a.err);
      if (!ok) *s_bad = 1;
      return ok;
    };
    if constexpr (DEC) {
      // ===================== y store thread (decode) ========================
      // For every expand stage whose y box is stored by TMA: wait until the
      // compute warps have written it (ydone), store it, wait until the store
      // has read shared memory, then free the stage for the producer.
      if (lane != 0) return;
      if (a.prefetch_weights) {
        // the first stages' activations, as soon as the dependency is met
        for (int u = 0; u < first; ++u) {
          bool armed = *s_armed > u;
          for (int spin = 0; !armed && spin < (1 << 22); ++spin) {
            __nanosleep(32);
            armed = *s_armed > u;
          }
          if (!armed) {
            *s_bad = 1;
            if (a.err) atomicOr(a.err, kErrWaitTimeout);
            break;
          }
          issue(u, u, 2, 0ull);
        }
      }
      if (!do_ex) return;
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
        for (int i = 0; i < nB; ++i, ++u) {
          const int stage = u % S;
          const bool ok = wait_ok(&ydone[stage], (ypar >> stage) & 1u);
          ypar ^= 1u << stage;
          if (ok) {
            tma_store_3d(slice_of(s) ? &a.tmap_y_x[slice_of(s) - 1][box_index(n)] : &a.tmap_y[box_index(n)], 0,
                         s.token_start, (oB0 + i * C::W) / kBoxCols,
                         stage_base + stage * C::STAGE);
            bulk_commit();
            bulk_wait_read();
          }
          mbar_arrive_n(&empty[stage], kComputeWarps);
        }
      }
      bulk_wait_all();
      return;
    }
    if (lane != 0) return;
    int u = 0;
    uint32_t sh_uses = 0, ht_uses = 0, acc_uses[2] = {0u, 0u};
    int ebuf = 0;
    for (int sj = 0; sj < nmine; ++sj) {
      const DevSeg s = desc(sj);
      const int n = clamp_rows(s.token_count);
      if (do_sh) {
        // shrink: D[rank, t] (TMEM) += A_box[rank, k] . x_box[t, k]^T, M = 64
        // (rows past r read neighbouring shared memory and are never used),
        // N = the segment's tokens rounded up to 8, K = 16 per instruction.
        // Each stage's commit frees it for the producer.
        const bool have = nA > 0 && n > 0;
        if (have && sh_uses > 0) wait_ok(sh_free, (sh_uses - 1) & 1);
        const uint32_t Nsh = static_cast<uint32_t>(max(8, (n + 7) & ~7));
        const int xsp = (8 << box_index(n)) * 128;  // bytes of one x slice
        const uint32_t idesc = umma_idesc(kAbf, 64, Nsh);
        for (int i = 0; i < nA; ++i, ++u) {
          const int stage = u % S;
          const bool ok = wait_ok(&full[stage], (u / S) & 1);
          if (sj == 0 && i == 0) trace_mark_t<TR>(a.trace, 4);
          if (ok && have) {
            tc_fence_after();
            const uint32_t st = smem_u32(stage_base + stage * C::STAGE);
            // descriptors step through the stage by adding (byte offset >> 4)
            // to their start-address field
            const uint64_t da = umma_desc(st, 1024, 2), dx = umma_desc(st + 4 * C::ABOX, 1024, 2);
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                umma_f16(t_sh, da + static_cast<uint64_t>((j * C::ABOX + ks * 32) >> 4),
                         dx + static_cast<uint64_t>((j * xsp + ks * 32) >> 4), idesc,
                         (i > 0 || j > 0 || ks > 0) ? 1u : 0u);
            umma_commit(&empty[stage]);  // the stage is free once these MMAs have read it
          } else {
            mbar_arrive(&empty[stage]);
          }
        }
        if (sj == 0) trace_mark_t<TR>(a.trace, 5);
        if (have) {
          if (!*s_bad) umma_commit(sh_full);
          ++sh_uses;
        }
      }
      if constexpr (C::TC) {
        if (do_ex && nB > 0) {
          // expand: D[o, t] (TMEM) = B[o, :] . H_hi[t, :]^T + B[o, :] . H_lo[t, :]^T,
          // two MMAs of M = 128 output columns per stage, N = 16 or 32 tokens, K = r
          const bool go = n > 0;
          if (go) {
            wait_ok(ht_full, ht_uses & 1);
            ++ht_uses;
          }
          const uint32_t N = n > 16 ? 32u : 16u;
          const uint32_t idesc = umma_idesc(kAbf, 128, N);
          const uint64_t dh = umma_desc(smem_u32(ht_base), 16 * R, C::UMMA_LAYOUT);
          const uint64_t dl = umma_desc(smem_u32(ht_base) + C::HT, 16 * R, C::UMMA_LAYOUT);
          for (int i = 0; i < nB; ++i, ++u) {
            if (!go) continue;
            const int stage = u % S;
            const int b = ebuf;
            ebuf ^= 1;
            wait_ok(&full[stage], (u / S) & 1);
            if (acc_uses[b] > 0) wait_ok(&acc_free[b], (acc_uses[b] - 1) & 1);
            ++acc_uses[b];
            if (*s_bad) continue;
            tc_fence_after();
            const uint32_t bsm = smem_u32(stage_base + stage * C::STAGE + 4 * C::XBOX);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint32_t acc = tbase + 64 + 64 * b + 32 * hh;
              const uint64_t db = umma_desc(bsm + hh * 128 * R * 2, 16 * R, C::UMMA_LAYOUT);
#pragma unroll
              for (int ks = 0; ks < R / 16; ++ks) umma_f16(acc, db + 2 * ks, dh + 2 * ks, idesc, ks > 0 ? 1u : 0u);
#pragma unroll
              for (int ks = 0; ks < R / 16; ++ks) umma_f16(acc, db + 2 * ks, dl + 2 * ks, idesc, 1u);
            }
            umma_commit(&acc_full[b]);
            if (sj == 0) trace_unit_t<TR>(a.trace, i, 6);
          }
        } else {
          u += nB;
        }
      } else {
        u += nB;
      }
    }
    return;
  }

  // ======================== epilogue / compute warps ===========================
  if (a.prefetch_weights) {
    pdl_wait_prior();
    pdl_launch_dependents();
    tr.dep();
  }
  // tensor parallelism: the epoch of this launch's peer exchange (after the
  // dependency wait, so the previous launch's advance is visible)
  const int tp_epoch = TPX ? __ldcg(&a.tp_seq[0]) + 1 : 0;
  const int g = lane >> 2;
  const int c = lane & 3;
  const int quarter = warp & 3;  // TMEM lane quarter this warp may read
  const int half = warp >> 2;
  int kc = 0;  // next stage-unit
  uint32_t cph = 0;  // cluster barrier phase
  uint32_t sh_ph = 0, acc_ph[2] = {0u, 0u};
  int ebuf = 0;
  auto wait_ok = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (*s_bad) return false;
    const bool ok = mbar_wait_bounded(bar, parity, a.err);
    if (!ok) *s_bad = 1;
    return ok;
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

  // mma.sync paths: shared-memory offsets of this thread's ldmatrix rows,
  // relative to a stage (the same for every stage).
  constexpr int MT = R >= 16 ? R / 16 : 1;  // 16-row rank tiles of the shrink (rank 8: rows 8-15 unused)
  constexpr int KS = R >= 16 ? R / 16 : 1;  // expand k-steps of 16 (rank 8: one m16n8k8 step)
  uint32_t offA[2][MT], offX[2][2], offB[KS][2], offY[4];
  if constexpr (DEC) {
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int row = mt * 16 + (lane & 15);
        const int ch = (warp & 1) * 4 + 2 * ks + (lane >> 4);
        offA[ks][mt] = (warp >> 1) * C::ABOX + row * 128 + (((ch ^ row) & 7) << 4);
      }
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int row = p * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int ch = (warp & 1) * 4 + 2 * ks + ((lane >> 3) & 1);
        offX[ks][p] = 4 * C::ABOX + row * 128 + (((ch ^ row) & 7) << 4);  // + slice (warp / 2)
      }
    }
  }
  if constexpr (!C::TC) {
    // expand, transposed: A operand = B rows (output columns) 16 per tile
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int row = warp * 32 + m * 16 + (lane & 15);
        uint32_t lin = static_cast<uint32_t>(row * (2 * R) + (2 * ks + (lane >> 4)) * 16);
        if constexpr (C::BTMA) lin ^= (lin >> 3) & C::SWZ_MASK;
        offB[ks][m] = 4 * C::XBOX + lin;
      }
    // y (token rows t, this warp's 32 columns as four 8-column matrices)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int t = nt * 8 + (lane & 7);
      const int chunk = (warp & 1) * 4 + (lane >> 3);
      offY[nt] = t * 128 + (((chunk ^ t) & 7) << 4);  // + slice (warp / 2)
    }
  }

  for (int sj = 0; sj < nmine; ++sj) {
    const DevSeg s = desc(sj);
    const int n = clamp_rows(s.token_count);
    if (tid == 0 && n == 0 && a.err) atomicOr(a.err, kErrBadSegment);
    // x / y slices are (8 << box_index(n)) rows of 128 bytes; this warp reads slice warp / 2
    const uint32_t xsl = static_cast<uint32_t>((warp >> 1) * ((8 << box_index(n)) * 128));
    const float alpha = registry ? s.alpha : a.scale;

    if (do_sh) {
      if constexpr (DEC) {
        // ---- 1. shrink on mma.sync: D[rank, t] += A[rank, k] . x[t, k]^T.
        // Warp w takes 32 columns of d of every stage (box w/2, half w%2) for
        // all rank tiles and token tiles, so no two warps read the same bytes;
        // the 8 partials are summed in a fixed order at the end of the segment.
        const bool have = nA > 0 && n > 0;
        float acc[MT][4][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.f;
        // the unit body is compiled per token-tile count (1-4)
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
                  ldsm_x4(sb + offA[ks][mt], af[ks][mt][0], af[ks][mt][1], af[ks][mt][2], af[ks][mt][3]);
  #pragma unroll
              for (int ks = 0; ks < 2; ++ks)
  #pragma unroll
                for (int p = 0; p < 2; ++p)
                  if (p < np) ldsm_x4(sb + xsl + offX[ks][p], bx[ks][p][0], bx[ks][p][1], bx[ks][p][2], bx[ks][p][3]);
  #pragma unroll
              for (int ks = 0; ks < 2; ++ks)
  #pragma unroll
                for (int p = 0; p < 2; ++p)
                  if (p < np) {
  #pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                      mma_k16<T>(acc[mt][2 * p], af[ks][mt], bx[ks][p][0], bx[ks][p][1]);
                      if (2 * p + 1 < nts) mma_k16<T>(acc[mt][2 * p + 1], af[ks][mt], bx[ks][p][2], bx[ks][p][3]);
                    }
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
          case 3: shrink_units(IntC<3>{}); break;
          default: shrink_units(IntC<4>{}); break;
        }
        tr.seg(0, sj);
        // cross-warp sum: every warp parks its partial in a slot of its own;
        // the eight slots are added per element below, in a fixed order
        {
          float* dst = Pw + warp * C::PSLOT;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int r = mt * 16 + g + (e >> 1) * 8;
                const int t = j * 8 + 2 * c + (e & 1);
                if (r < R) dst[t * PITCH + r] = acc[mt][j][e];
              }
        }
        named_sync(kBarCompute, kComputeThreads);
        // ---- 2. cluster exchange (push): each thread sums the eight slots of
        // its elements and pushes them by st.async into this CTA's slot of
        // every peer, completing bytes on the peer's rx_full barrier; it keeps
        // its own sums in registers. A slot of a segment parity is rewritten
        // only after every peer has released it (rx_free). Every CTA adds the
        // ranks' partials in rank order, so all of them get the same H.
        const int par = sj & 1;
        const uint32_t use = static_cast<uint32_t>(sj >> 1);  // uses of this parity so far
        float* rx = Rx + par * C::CLMAX * C::PSLOT;
        if (CL > 1 && use > 0 && !*s_bad && !mbar_wait_cluster_bounded(&rx_free[par], (use - 1) & 1, a.err)) *s_bad = 1;
        constexpr int Q4 = R / 4;  // 16-byte chunks per partial row
        constexpr int KE = (32 * Q4 + kComputeThreads - 1) / kComputeThreads;  // elements per thread at most
        const int nch = n * Q4;
        float4 own[KE];
        if (!*s_bad) {
#pragma unroll
          for (int k = 0; k < KE; ++k) {
            const int e4 = tid + k * kComputeThreads;
            if (e4 < nch) {
              const int off = (e4 / Q4) * PITCH + (e4 % Q4) * 4;
              float4 p[8];
#pragma unroll
              for (int w = 0; w < 8; ++w) p[w] = *reinterpret_cast<const float4*>(Pw + w * C::PSLOT + off);
              float4 v;
              v.x = ((p[0].x + p[1].x) + (p[2].x + p[3].x)) + ((p[4].x + p[5].x) + (p[6].x + p[7].x));
              v.y = ((p[0].y + p[1].y) + (p[2].y + p[3].y)) + ((p[4].y + p[5].y) + (p[6].y + p[7].y));
              v.z = ((p[0].z + p[1].z) + (p[2].z + p[3].z)) + ((p[4].z + p[5].z) + (p[6].z + p[7].z));
              v.w = ((p[0].w + p[1].w) + (p[2].w + p[3].w)) + ((p[4].w + p[5].w) + (p[6].w + p[7].w));
              own[k] = v;
              const uint32_t mine = smem_u32(rx + q * C::PSLOT + off);
              for (uint32_t i = 1; i < CL; ++i) {
                const uint32_t peer = (q + i) % CL;
                st_async_v4(mapa(mine, peer), v, mapa(smem_u32(&rx_full[par]), peer));
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
          for (int k = 0; k < KE; ++k) {
            const int e4 = tid + k * kComputeThreads;
            if (e4 < nch) {
              const int t = e4 / Q4;
              const int off = t * PITCH + (e4 % Q4) * 4;
              float4 sum = q == 0 ? own[k] : *reinterpret_cast<const float4*>(rx + off);
              for (uint32_t i = 1; i < CL; ++i) {
                const float4 v = i == q ? own[k] : *reinterpret_cast<const float4*>(rx + i * C::PSLOT + off);
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
      } else {
        kc += nA;  // shrink stages are consumed by the MMA warp
        // ---- 1. partial tile -> Ps[token][rank] (zeros when this CTA owns no slice of d)
        const bool have = nA > 0 && n > 0;
        if (have) {
          wait_ok(sh_full, sh_ph);
          sh_ph ^= 1u;
          tc_fence_after();
        }
        tr.seg(0, sj);
        // M = 64 accumulator layout: rank r sits in TMEM lane (r % 16) + 32 * (r / 16)
        if (half == 0 && quarter * 16 < R) {
          float v[32];
          // warp-uniform: the tcgen05 loads are .sync.aligned
          if (__shfl_sync(0xffffffffu, (have && !*s_bad) ? 1 : 0, 0)) {
            const uint32_t ta = t_sh + (static_cast<uint32_t>(quarter * 32) << 16);
            tmem_ld16(ta, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(ta + 16, *reinterpret_cast<float(*)[16]>(v + 16));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
          const int r = quarter * 16 + lane;
          if (lane < 16 && r < R) {
#pragma unroll
            for (int j = 0; j < 32; ++j) Ps[j * PITCH + r] = v[j];
          }
        }
        if (have) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(sh_free);  // the MMA warp may start the next shrink
        }
      }
      if constexpr (!DEC) {
      tr.mark(2);
      // ---- 2. reduce-scatter + all-gather of the partials over the cluster
      if (!cluster_barrier_bounded(cbar, cph, CL, kBarCompute, kComputeThreads, a.err)) *s_bad = 1;
      cph ^= 1u;
      tr.seg(1, sj);
      if (!*s_bad && n > 0) {
        const int per = (n + static_cast<int>(CL) - 1) / static_cast<int>(CL);
        const int r0 = static_cast<int>(q) * per;
        const int r1 = min(n, r0 + per);
        for (int e = tid; e < (r1 - r0) * (R / 2); e += kComputeThreads) {
          const int row = r0 + e / (R / 2);
          const int col = (e % (R / 2)) * 2;
          const uint32_t paddr = smem_u32(Ps + row * PITCH + col);
          float2 sum = make_float2(0.f, 0.f);
          for (uint32_t i = 0; i < CL; ++i) {
            const float2 v = ld_dsmem_f2(mapa(paddr, i));
            sum.x += v.x;
            sum.y += v.y;
          }
          sum.x *= alpha;
          sum.y *= alpha;
          if (do_ex) {
            const uint32_t haddr = smem_u32(Hs + row * PITCH + col);
            for (uint32_t i = 0; i < CL; ++i) st_dsmem_f2(mapa(haddr, i), sum);
          } else {
            *reinterpret_cast<float2*>(a.h + static_cast<int64_t>(s.token_start + row) * R + col) = sum;
          }
        }
      }
      if (!cluster_barrier_bounded(cbar, cph, CL, kBarCompute, kComputeThreads, a.err)) *s_bad = 1;
      cph ^= 1u;
      tr.seg(2, sj);
      }
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
    T* yg = static_cast<T*>(a.y);

    if constexpr (C::TC) {
      // ---- 3. expand epilogue: TMEM accumulators (issued by the MMA warp) + y -> y
      const bool go = n > 0;
      if (go) {
        // H tiles (16-bit high part + residual), rows = tokens, swizzled like B
        const int N = n > 16 ? 32 : 16;
        for (int e = tid; e < N * (R / 2); e += kComputeThreads) {
          const int j = e / (R / 2);
          const int k = (e % (R / 2)) * 2;
          float2 v = make_float2(0.f, 0.f);
          if (j < n) v = *reinterpret_cast<const float2*>(Hs + j * PITCH + k);
          const uint32_t hv = E::pack2(v.x, v.y);
          const float2 r2 = E::unpack2(hv);
          const uint32_t lv = E::pack2(v.x - r2.x, v.y - r2.y);
          uint32_t lin = static_cast<uint32_t>(j * C::SWZ_BYTES + k * 2);
          lin ^= (lin >> 3) & C::SWZ_MASK;
          *reinterpret_cast<uint32_t*>(ht_base + lin) = hv;
          *reinterpret_cast<uint32_t*>(ht_base + C::HT + lin) = lv;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(ht_full);
      }
      tr.seg(3, sj);
      const int ol = half * 128 + quarter * 32 + lane;  // this lane's output column in the stage
      for (int i = 0; i < nB; ++i, ++kc) {
        const int stage = kc % S;
        wait_full(stage);  // y box of the stage
        const uint8_t* st = stage_base + stage * C::STAGE;
        const int oc = oB0 + i * C::W;
        const int wc = min(C::W, a.o - oc);
        if (go) {
          const int b = ebuf;
          ebuf ^= 1;
          const bool ok = wait_ok(&acc_full[b], acc_ph[b]);
          acc_ph[b] ^= 1u;
          tc_fence_after();
          float v[32];
          if (__shfl_sync(0xffffffffu, (ok && !*s_bad) ? 1 : 0, 0)) {
            const uint32_t ta = tbase + 64 + 64 * b + 32 * half + (static_cast<uint32_t>(quarter * 32) << 16);
            tmem_ld16(ta, *reinterpret_cast<float(*)[16]>(v));
            if (n > 16) tmem_ld16(ta + 16, *reinterpret_cast<float(*)[16]>(v + 16));
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_free[b]);  // the MMA warp may reuse this accumulator
          tr.mark(2);
          // phase A: D column of this lane -> Ds[token][column]
          if (ol < wc) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < n) Ds[j * C::DPITCH + ol] = v[j];
          }
          named_sync(kBarCompute, kComputeThreads);
          tr.mark(3);
          // phase B: warp w takes tokens w, w + 8, ...; lane l the 8-column chunk l
          const int col = lane * 8;
          if (col < wc) {
            const int cib = lane & 7;  // 16-byte chunk inside the 128-byte box row
            const uint8_t* yb = st + (lane >> 3) * ((8 << box_index(n)) * 128);
            for (int t = warp; t < n; t += kComputeWarps) {
              const float* dr = Ds + t * C::DPITCH + col;
              const float4 d0 = reinterpret_cast<const float4*>(dr)[0];
              const float4 d1 = reinterpret_cast<const float4*>(dr)[1];
              const float dv[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
              T* yp = yg + static_cast<int64_t>(s.token_start + t) * a.y_ld + yoff_of(s) + oc + col;
              if (y_tma) {
                const int4 yv = *reinterpret_cast<const int4*>(yb + t * 128 + ((cib ^ (t & 7)) << 4));
                const uint32_t* yw = reinterpret_cast<const uint32_t*>(&yv);
                int4 out;
                uint32_t* ow = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
                for (int p2 = 0; p2 < 4; ++p2) {
                  const float2 f = E::unpack2(yw[p2]);
                  ow[p2] = E::pack2(f.x + dv[2 * p2], f.y + dv[2 * p2 + 1]);
                }
                *reinterpret_cast<int4*>(yp) = out;
              } else {
                float yv[8];
#pragma unroll
                for (int x = 0; x < 8; ++x) yv[x] = E::to_f(yp[x]);
#pragma unroll
                for (int x = 0; x < 8; ++x) yp[x] = E::from_f(yv[x] + dv[x]);
              }
            }
          }
          tr.mark(4);
        }
        named_sync(kBarCompute, kComputeThreads);
        if (tid == 0) mbar_arrive(&empty[stage]);
      }
    } else {
      // ---- 3. expand on mma.sync over this CTA's slice of o -----------------
      // Transposed: D^T[o, t] = B[o, :] . H[t, :]^T with M = 16 output columns
      // per tile (A operand: B rows from the stage, ldmatrix) and N = 8 tokens
      // per tile (B operand: H rows), so a segment of n tokens costs
      // ceil(n / 8) token tiles. Warp w owns output columns 32w..32w+31 of
      // every stage. y comes in and goes back through ldmatrix / stmatrix
      // .trans, which turn the [token][column] box into the accumulator
      // layout and back. In the decode variant H enters rounded to T (the
      // weights' type, as the stock expand does); the rank-8 path of the
      // tcgen05 kernel adds a 16-bit residual of H (~16 mantissa bits).
      uint32_t hb[4][KS][2], hl[4][KS][2];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const float* hrow = Hs + (nt * 8 + g) * PITCH;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const int k0 = ks * 16 + 2 * c;
          float2 x[2];
          x[0] = *reinterpret_cast<const float2*>(hrow + k0);
          x[1] = R >= 16 ? *reinterpret_cast<const float2*>(hrow + k0 + 8) : make_float2(0.f, 0.f);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            hb[nt][ks][e] = E::pack2(x[e].x, x[e].y);
            if constexpr (!DEC) {
              const float2 r = E::unpack2(hb[nt][ks][e]);
              hl[nt][ks][e] = E::pack2(x[e].x - r.x, x[e].y - r.y);
            }
          }
        }
      }
      const bool tmy = y_by_tma(n);  // the store thread writes the y box back and frees the stage
      // the unit body is compiled per token-tile count (1-4): no runtime
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
            // y tiles: yf[nt][ob] = y[t in tile nt][8 columns ob]
            uint32_t yf[4][4];
            float acc[2][4][4];
  #pragma unroll
            for (int nt = 0; nt < 4; ++nt)
              if (nt < ntn) ldsm_x4_t(sb + xsl + offY[nt], yf[nt][0], yf[nt][1], yf[nt][2], yf[nt][3]);
            // the accumulators start at y (fp32): D = y + H . B^T, rounded once
  #pragma unroll
            for (int m = 0; m < 2; ++m)
  #pragma unroll
              for (int nt = 0; nt < 4; ++nt) {
                float2 f0 = make_float2(0.f, 0.f), f1 = make_float2(0.f, 0.f);
                if (nt < ntn) {
                  f0 = E::unpack2(yf[nt][2 * m]);
                  f1 = E::unpack2(yf[nt][2 * m + 1]);
                }
                acc[m][nt][0] = f0.x;
                acc[m][nt][1] = f0.y;
                acc[m][nt][2] = f1.x;
                acc[m][nt][3] = f1.y;
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
                    ldsm_x4(sb + offB[k0 + kk][m], bA[kk][m][0], bA[kk][m][1], bA[kk][m][2], bA[kk][m][3]);
  #pragma unroll
                for (int kk = 0; kk < KB; ++kk)
  #pragma unroll
                  for (int nt = 0; nt < 4; ++nt)
                    if (nt < ntn) {
                      const int ks = k0 + kk;
  #pragma unroll
                      for (int m = 0; m < 2; ++m) {
                        mma_k16<T>(acc[m][nt], bA[kk][m], hb[nt][ks][0], hb[nt][ks][1]);
                        if constexpr (!DEC) mma_k16<T>(acc[m][nt], bA[kk][m], hl[nt][ks][0], hl[nt][ks][1]);
                      }
                    }
              }
            } else {
              // rank 8: B rows of 16 bytes (linear); matrices 2m, 2m + 1 = rows 16m..16m+15
              uint32_t bf[4];
              ldsm_x4(sb + 4 * C::XBOX + (warp * 32 + lane) * 16, bf[0], bf[1], bf[2], bf[3]);
  #pragma unroll
              for (int nt = 0; nt < 4; ++nt)
                if (nt < ntn) {
  #pragma unroll
                  for (int m = 0; m < 2; ++m) {
                    mma_k8<T>(acc[m][nt], bf[2 * m], bf[2 * m + 1], hb[nt][0][0]);
                    if constexpr (!DEC) mma_k8<T>(acc[m][nt], bf[2 * m], bf[2 * m + 1], hl[nt][0][0]);
                  }
                }
            }
            tr.mark(3);
            {
              // back into the y box in place; then the box goes to global memory
              // by one tensor store (store thread) or this warp's 16-byte row
              // chunks are stored directly (element by element for a y that is
              // not 16-byte addressable).
  #pragma unroll
              for (int nt = 0; nt < 4; ++nt)
                if (nt < ntn) {
                  stsm_x4_t(sb + xsl + offY[nt], E::pack2(acc[0][nt][0], acc[0][nt][1]),
                            E::pack2(acc[0][nt][2], acc[0][nt][3]), E::pack2(acc[1][nt][0], acc[1][nt][1]),
                            E::pack2(acc[1][nt][2], acc[1][nt][3]));
                }
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
                  int4 out[4];
  #pragma unroll
                  for (int it = 0; it < 4; ++it) {
                    const int row = (lane >> 2) + 8 * it;
                    if (it < ntn && row < n)
                      out[it] = *reinterpret_cast<const int4*>(ybox + row * 128 + (((chunk ^ row) & 7) << 4));
                  }
  #pragma unroll
                  for (int it = 0; it < 4; ++it) {
                    const int row = (lane >> 2) + 8 * it;
                    if (it < ntn && row < n) *reinterpret_cast<int4*>(ycol + static_cast<int64_t>(row) * a.y_ld) = out[it];
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
          }
          if constexpr (DEC) {
            __syncwarp();
            tr.mark(5);
            if (lane == 0) mbar_arrive(tmy ? &ydone[stage] : &empty[stage]);
          } else {
            named_sync(kBarCompute, kComputeThreads);
            if (tid == 0) mbar_arrive(&empty[stage]);
          }
        }
      };
      switch ((n + 7) >> 3) {
        case 0:
        case 1: expand_units(IntC<1>{}); break;
        case 2: expand_units(IntC<2>{}); break;
        case 3: expand_units(IntC<3>{}); break;
        default: expand_units(IntC<4>{}); break;
      }
    }
  }

  if constexpr (DEC) {
    // Peers arrive on this CTA's barrier until they pass this one, so the
    // shared memory must outlive it. Their other remote accesses (pushes into
    // the receive slots, slot releases) were all observed before: every push
    // was consumed, and the releases of the last two segments are not sent.
    // No data crosses this barrier, so it needs no release fence (a fence
    // would wait for this thread's outstanding y stores).
    if (CL > 1 && !cluster_barrier_relaxed_bounded(cbar, cph, CL, kBarCompute, kComputeThreads, a.err)) *s_bad = 1;
  }
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
  if (use_tmem) {
    tc_fence_before();
    named_sync(kBarCompute, kComputeThreads);  // every TMEM read and MMA is done
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(*s_tmem, 256);
    }
  }
  tr.finish();
}

// --------------------------------------------------------------------------
// launchers

namespace {

template <typename T, int R, bool DEC, bool TR, int LF, bool TPX = false>
struct ApplyKernel {
  using C = ApplyCfg<R, DEC>;
  static bool prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return true;
    if (cudaFuncSetAttribute(apply_kernel<T, R, DEC, TR, LF, TPX>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return false;
    done.fetch_or(bit);
    return true;
  }

  static cudaError_t launch(const ApplyArgs& a, const LaunchCfg& lc) {
    if (DEC && lc.cluster > C::CLMAX) return cudaErrorInvalidValue;
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
    return cudaLaunchKernelEx(&cfg, apply_kernel<T, R, DEC, TR, LF, TPX>, a);
  }

  static int max_grid(int cluster) {
    if (DEC && cluster > C::CLMAX) return 0;  // receive slots exist for CLMAX ranks
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
    if (cudaOccupancyMaxActiveClusters(&nclusters, apply_kernel<T, R, DEC, TR, LF, TPX>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return nclusters * cluster;
  }
};

template <typename T, int R>
cudaError_t apply_variant(const ApplyArgs& a, const LaunchCfg& lc) {
  const bool live_fused = lc.dec && a.mode == kModeFused && !a.registry && a.y_tma;
  const int lf = live_fused ? (a.nslices > 1 ? 2 : 1) : 0;
  if (a.tp_world > 1) {
    // row-parallel exchange over peer memory (untraced): live fused single-slice calls on the decode variant
    if (lf != 1) return cudaErrorInvalidValue;
    return ApplyKernel<T, R, true, false, 1, true>::launch(a, lc);
  }
  if (a.trace) {
    if (lf == 1) return ApplyKernel<T, R, true, true, 1>::launch(a, lc);
    return lc.dec ? ApplyKernel<T, R, true, true, 0>::launch(a, lc) : ApplyKernel<T, R, false, true, 0>::launch(a, lc);
  }
  if (lf == 1) return ApplyKernel<T, R, true, false, 1>::launch(a, lc);
  if (lf == 2) return ApplyKernel<T, R, true, false, 2>::launch(a, lc);
  return lc.dec ? ApplyKernel<T, R, true, false, 0>::launch(a, lc) : ApplyKernel<T, R, false, false, 0>::launch(a, lc);
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
int max_grid_by_rank(int rank, int cluster, bool dec) {
  switch (rank) {
    case 8: return dec ? ApplyKernel<T, 8, true, false, 0>::max_grid(cluster) : ApplyKernel<T, 8, false, false, 0>::max_grid(cluster);
    case 16: return dec ? ApplyKernel<T, 16, true, false, 0>::max_grid(cluster) : ApplyKernel<T, 16, false, false, 0>::max_grid(cluster);
    case 32: return dec ? ApplyKernel<T, 32, true, false, 0>::max_grid(cluster) : ApplyKernel<T, 32, false, false, 0>::max_grid(cluster);
    case 64: return dec ? ApplyKernel<T, 64, true, false, 0>::max_grid(cluster) : ApplyKernel<T, 64, false, false, 0>::max_grid(cluster);
    default: return 0;
  }
}

}  // namespace

cudaError_t launch_apply(int dtype, int rank, const ApplyArgs& a, const LaunchCfg& lc) {
  return dtype == 1 ? apply_by_rank<__nv_bfloat16>(rank, a, lc) : apply_by_rank<__half>(rank, a, lc);
}

int apply_max_grid(int dtype, int rank, int cluster, bool dec) {
  return dtype == 1 ? max_grid_by_rank<__nv_bfloat16>(rank, cluster, dec) : max_grid_by_rank<__half>(rank, cluster, dec);
}

}  // namespace wp
