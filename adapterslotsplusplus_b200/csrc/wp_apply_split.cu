// wp_apply_split.cu -- the balanced decode apply kernel ("split" kernel).
//
// Same semantics as wp_apply.cu (H = alpha * X . A^T per segment, then
// Y += H . B^T rounded once; reference tests/correctness/reference_bgmv.py:4-18
// and csrc/kernels/warp_pipe_r32.cu:56-200), organised for decode batches
// where a few segments are large and many are small.
//
// Work is cut into equal items of one pipeline stage each:
//   shrink item (s, c): columns [256c, 256c + 256) of d for segment s,
//   expand item (s, c): output columns [256c, 256c + 256) of o for segment s.
// Items are numbered segment-major (all shrink items first, then all expand
// items) and every CTA of a one-CTA-per-SM grid takes a contiguous block of
// each list, so every SM streams the same number of bytes of weights within
// one stage, whatever the segment sizes. A CTA accumulates its consecutive
// shrink items of one segment (a "run") in registers, writes one partial H
// (fp32) per run and publishes it with a release flag of its own (no
// round trip). For each expand run, a fetch warp waits for the flags of all
// of the segment's shrink runs (bounded), adds the partials in run order --
// deterministic -- scales by alpha and leaves H in shared memory, while the
// producer already streams the run's B and y. The last fetcher of a segment
// (an acq_rel counter) clears the segment's flags, so the kernel replays
// inside CUDA graphs.
//
// Deadlock freedom: every CTA issues and finishes all of its shrink items
// before it issues an expand item, shrink items wait on nothing, and an
// expand item waits only on shrink items; the waits are bounded (1 s) all
// the same and raise kErrWaitTimeout.
//
// Warp roles (352 threads): warps 0-7 compute (mma.sync shrink / expand,
// exactly the arithmetic of the decode variant of wp_apply.cu), warp 8 lane 0
// issues every TMA load (weights with an L2 evict-first hint), warp 9 lane 0
// stores whole y boxes with one tensor store and frees their stages, warp 10
// (all lanes) builds each expand run's H in shared memory, so the B and y
// loads of the expand stages go ahead while H is still being reduced.

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

namespace {

constexpr int kSW = 8;  // compute warps
constexpr int kSCT = kSW * 32;  // compute threads
constexpr int kSThreads = kSCT + 96;
constexpr int kSProducer = kSW;
constexpr int kSStore = kSW + 1;
constexpr int kSHFetch = kSW + 2;
constexpr int kSBar = 1;  // named barrier of the compute warps
constexpr int kSDesc = 64;  // descriptors cached per list (shrink / expand)
constexpr int kSSmemMax = 232448;
constexpr int kSMaskWords = 64;  // run-start bits of up to 2048 chunks (d <= 524288)

template <int R>
struct SplitCfg {
  static constexpr int ABOX = R * 128;  // one A box: R rows x 128 B
  static constexpr int XBOX = 32 * 128;  // room for one 32-row x or y slice
  static constexpr int STAGE = 4 * ABOX + 4 * XBOX;  // == 4 * XBOX + 256 * R * 2
  static_assert(STAGE == 4 * XBOX + 256 * R * 2, "shrink and expand stages have one size");
  static constexpr int PITCH = R + 4;  // floats per row of a partial slot
  static constexpr int PSLOT = 32 * PITCH;
  static constexpr int HSLOT = 32 * R * 4;  // one H slot: 32 dense fp32 rows
  // barriers: full[8] @0, empty[8] @64, ydone[8] @128, hread[2] @192
  static constexpr int OFF_FLAGS = 224;
  static constexpr int OFF_MASK = 256;  // kSMaskWords words
  static constexpr int OFF_DESC = 512;
  static constexpr int OFF_PW = OFF_DESC + 2 * kSDesc * 32;
  static constexpr int OFF_H = OFF_PW + 4 * PSLOT * 4;
  static constexpr int FIXED = OFF_H + HSLOT + 1024;
  static constexpr int FIT = (kSSmemMax - FIXED) / STAGE;
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr int SMEM = FIXED + STAGES * STAGE;
  static_assert(STAGES >= 2 && SMEM <= kSSmemMax, "shared memory budget");
  static_assert(HSLOT % 16 == 0, "H rows are bulk-copied");
};

// Item blocks: item i of a list of n goes to CTA f(i) = floor(i * g / n), so
// CTA k holds the contiguous items [ceil(k n / g), ceil((k + 1) n / g)) (empty
// blocks when n < g). 32-bit arithmetic: i * g stays below 2^31 for the
// lists this kernel takes (n <= 2^31 / g, enforced by the host).
__device__ __forceinline__ int blk_of(int i, int n, int g) { return i * g / n; }
__device__ __forceinline__ int blk_lo(int k, int n, int g) { return (k * n + g - 1) / g; }
// Item i starts a run of its segment (whose first item is i0).
__device__ __forceinline__ bool item_starts_run(int i, int i0, int n, int g) {
  return i == i0 || blk_of(i, n, g) != blk_of(i - 1, n, g);
}
// Runs (one per CTA holding items) over the nc items of segment s.
__device__ __forceinline__ int seg_runs(int s, int nc, int n, int g) {
  const int i0 = s * nc;
  return min(nc, blk_of(i0 + nc - 1, n, g) - blk_of(i0, n, g) + 1);
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait (1 s) for a global flag to become non-zero.
__device__ __forceinline__ bool wait_flag(const int* p, int* err) {
  if (ld_acquire_gpu(p)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    __nanosleep(64);
    if (ld_acquire_gpu(p)) return true;
    if (global_timer_ns() - t0 > kWaitTimeoutNs) {
      if (err) atomicOr(err, kErrWaitTimeout);
      return false;
    }
  }
}

template <typename T, int R, bool TR>
__global__ void __launch_bounds__(kSThreads, 1) split_kernel(const __grid_constant__ ApplyArgs a) {
  using C = SplitCfg<R>;
  using E = Elem<T>;
  constexpr int S = C::STAGES;
  constexpr int PITCH = C::PITCH;
  constexpr int MT = R >= 16 ? R / 16 : 1;  // 16-row rank tiles of the shrink (rank 8: rows 8-15 unused)
  constexpr int KS = R >= 16 ? R / 16 : 1;  // expand k-steps of 16 (rank 8: one m16n8k8 step)

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + 64);
  uint64_t* ydone = reinterpret_cast<uint64_t*>(smem + 128);
  uint64_t* hread = reinterpret_cast<uint64_t*>(smem + 192);  // [2] compute warps read a run's partials
  volatile int* s_bad = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS);
  volatile int* s_issued = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS + 4);
  volatile int* s_armed = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS + 8);  // stages armed by the producer
  int4* sdesc = reinterpret_cast<int4*>(smem + C::OFF_DESC);  // [2 lists][kSDesc][2]
  float* Pw = reinterpret_cast<float*>(smem + C::OFF_PW);
  float* Hsl = reinterpret_cast<float*>(smem + C::OFF_H);  // [32][R]: H of the current expand run
  volatile uint32_t* runmask = reinterpret_cast<volatile uint32_t*>(smem + C::OFF_MASK);  // run-start chunks
  uint8_t* stage_base = align1024(smem + C::OFF_H + C::HSLOT);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = static_cast<int>(gridDim.x);
  const int k = static_cast<int>(blockIdx.x);
  std::conditional_t<TR, Trace, TraceOff> tr;
  tr.init(a.trace, tid == 0);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSW);
      mbar_init(&ydone[s], kSW);
    }
    for (int b = 0; b < 2; ++b) mbar_init(&hread[b], 1);
    *s_bad = 0;
    *s_issued = 0;
    *s_armed = 0;
    fence_mbar_init();
  }
  if (warp == kSProducer && lane == 0) {
    for (int i = 0; i < 3; ++i) prefetch_tmap(&a.tmap_x[i]);
    prefetch_tmap(&a.tmap_a);
    if (a.y_tma)
      for (int i = 0; i < 3; ++i) prefetch_tmap(&a.tmap_y[i]);
    if (R >= 16) prefetch_tmap(&a.tmap_b);
  }

  // ---- work of this CTA ------------------------------------------------------
  const int NCD = (a.d + kStageK - 1) / kStageK;
  const int NCO = (a.o + kStageCols - 1) / kStageCols;
  int nseg = 0, sh0 = 0, nS = 0, ex0 = 0, nE = 0, s_sh0 = 0, s_ex0 = 0;
  auto read_table = [&]() {
    nseg = max(0, min(__ldcg(a.num_segs), a.sync_cap));
    const int NS = nseg * NCD, NE = nseg * NCO;
    sh0 = blk_lo(k, NS, G);
    nS = blk_lo(k + 1, NS, G) - sh0;
    ex0 = blk_lo(k, NE, G);
    nE = blk_lo(k + 1, NE, G) - ex0;
    s_sh0 = NCD ? sh0 / NCD : 0;
    s_ex0 = NCO ? ex0 / NCO : 0;
    const int nsh = nS > 0 ? (sh0 + nS - 1) / NCD - s_sh0 + 1 : 0;
    const int nex = nE > 0 ? (ex0 + nE - 1) / NCO - s_ex0 + 1 : 0;
    for (int j = tid; j < 2 * min(nsh, kSDesc); j += kSThreads)
      sdesc[j] = __ldcg(reinterpret_cast<const int4*>(a.segs + s_sh0 + (j >> 1)) + (j & 1));
    for (int j = tid; j < 2 * min(nex, kSDesc); j += kSThreads)
      sdesc[2 * kSDesc + j] = __ldcg(reinterpret_cast<const int4*>(a.segs + s_ex0 + (j >> 1)) + (j & 1));
  };
  // descriptor of segment s (list 0: shrink, 1: expand)
  auto desc = [&](int list, int s) -> DevSeg {
    const int j = s - (list ? s_ex0 : s_sh0);
    if (j >= 0 && j < kSDesc) return unpack_seg(sdesc[(list * kSDesc + j) * 2], sdesc[(list * kSDesc + j) * 2 + 1]);
    return load_seg(a.segs, s);
  };
  if (a.prefetch_weights) {
    read_table();
  } else {
    pdl_wait_prior();
    pdl_launch_dependents();
    read_table();
  }
  __syncthreads();
  const int U = nS + nE;
  // unit u -> (is shrink, segment, chunk); loops advance (segment, chunk) incrementally
  auto unit = [&](int u, int& s, int& c) -> bool {
    if (u < nS) {
      s = (sh0 + u) / NCD;
      c = (sh0 + u) - s * NCD;
      return true;
    }
    s = (ex0 + u - nS) / NCO;
    c = (ex0 + u - nS) - s * NCO;
    return false;
  };
  const int c_sh0 = sh0 - s_sh0 * NCD;  // chunk of the first shrink / expand item
  const int c_ex0 = ex0 - s_ex0 * NCO;
  const float alpha_h = a.scale;
  auto y_by_tma = [&](int n) -> bool { return a.y_tma && a.o_sliced && (n == 8 || n == 16 || n == 32); };
  int* done = a.sync;

  // TMA issue of stage-unit (sh, s, c) into `stage`; parts: 1 = arm the
  // stage and load the weights (ef: their L2 evict-first policy), 2 = the
  // activations
  auto issue = [&](bool sh, int s, int c, int stage, int parts, uint64_t ef) {
    const DevSeg g = desc(sh ? 0 : 1, s);
    const int n = clamp_rows(g.token_count);
    const int bi = box_index(n);
    const uint32_t box_bytes = (8u << bi) * 128u;  // one 64-column slice of x or y
    uint8_t* st = stage_base + stage * C::STAGE;
    uint64_t* bar = &full[stage];
    if (sh) {
      const int k0 = c * kStageK;
      if (parts & 1) {
        mbar_arrive_expect_tx(bar, 4 * C::ABOX + 4 * box_bytes);
        if (a.d_sliced) {
          tma_load_4d_ef(st, &a.tmap_a, 0, 0, k0 / kBoxCols, g.adapter_id, bar, ef);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tma_load_3d_ef(st + j * C::ABOX, &a.tmap_a, k0 + j * kBoxCols, 0, g.adapter_id, bar, ef);
        }
      }
      if (parts & 2) {
        if (a.d_sliced) {
          tma_load_3d(st + 4 * C::ABOX, &a.tmap_x[bi], 0, g.token_start, k0 / kBoxCols, bar);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tma_load_2d(st + 4 * C::ABOX + j * box_bytes, &a.tmap_x[bi], k0 + j * kBoxCols, g.token_start, bar);
        }
      }
    } else {
      const int oc = c * kStageCols;
      const int wc = min(kStageCols, a.o - oc);
      if (parts & 1) {
        if constexpr (R >= 16) {
          mbar_arrive_expect_tx(bar, 256 * R * 2 + (a.y_tma ? 4 * box_bytes : 0u));
          tma_load_3d_ef(st + 4 * C::XBOX, &a.tmap_b, 0, oc, g.adapter_id, bar, ef);
        } else {
          mbar_arrive_expect_tx(bar, wc * R * 2 + (a.y_tma ? 4 * box_bytes : 0u));
          const T* B = static_cast<const T*>(a.wb_base) + static_cast<int64_t>(g.adapter_id) * a.wb_stride;
          bulk_g2s(st + 4 * C::XBOX, B + static_cast<int64_t>(oc) * R, wc * R * 2, bar);
        }
      }
      if (parts & 2) {
        if (a.y_tma) {
          if (a.o_sliced) {
            tma_load_3d(st, &a.tmap_y[bi], 0, g.token_start, oc / kBoxCols, bar);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tma_load_2d(st + j * box_bytes, &a.tmap_y[bi], oc + j * kBoxCols, g.token_start, bar);
          }
        }
      }
    }
  };
  const int first = min(S, U);  // stages issued before any is consumed
  if (warp == kSProducer) {
    // =========================== producer ====================================
    // Lanes 1-31 leave at once: a lane blocked in the dependency wait would
    // hold up the whole warp, lane 0's pre-dependency issue included.
    if (lane != 0) return;
    {
      const uint64_t ef = l2_evict_first_policy();
      if (a.prefetch_weights) {
        // the store thread loads these stages' activations as soon as the
        // dependency wait ends, while this thread still issues weights
        for (int u = 0; u < first; ++u) {
          int s, c;
          const bool sh = unit(u, s, c);
          issue(sh, s, c, u, 1, ef);
          __threadfence_block();
          *s_armed = u + 1;
        }
        pdl_wait_prior();
        pdl_launch_dependents();
      } else {
        for (int u = 0; u < first; ++u) {
          int s, c;
          const bool sh = unit(u, s, c);
          issue(sh, s, c, u, 3, ef);
        }
      }
      *s_issued = first;
      int s = 0, c = 0;
      bool sh = true;
      if (first < U) sh = unit(first, s, c);
      for (int u = first; u < U; ++u) {
        const int stage = u % S;
        if (!mbar_wait_bounded(&empty[stage], ((u / S) - 1) & 1, a.err)) *s_bad = 1;
        if (*s_bad) break;
        issue(sh, s, c, stage, 3, ef);
        *s_issued = u + 1;
        // next unit
        if (u + 1 == nS) {
          sh = false;
          s = s_ex0;
          c = c_ex0;
        } else if (++c == (sh ? NCD : NCO)) {
          c = 0;
          ++s;
        }
      }
    }
    return;
  }

  if (warp == kSHFetch) {
    // ====================== flag bookkeeping warp ============================
    // After the compute warps have read an expand run's partials (hread), count
    // the segment's readers; the last one clears the segment's run flags for
    // the next launch. Off the compute warps' path.
    pdl_wait_prior();
    pdl_launch_dependents();
    const int NS = nseg * NCD;
    int hruns = 0;
    const int s_last = nE > 0 ? (ex0 + nE - 1) / NCO : s_ex0 - 1;
    for (int s = s_ex0; s <= s_last; ++s, ++hruns) {
      bool ok = !*s_bad && mbar_wait_bounded(&hread[hruns & 1], (hruns >> 1) & 1, a.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      int last = 0;
      if (lane == 0) last = atom_add_acq_rel_gpu(&done[s], 1) == seg_runs(s, NCO, nseg * NCO, G) - 1;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        for (int c = lane; c < NCD; c += 32)
          if (item_starts_run(s * NCD + c, s * NCD, NS, G)) a.rflag[s * NCD + c] = 0;
        __syncwarp();
        if (lane == 0) done[s] = 0;
      }
    }
    return;
  }

  if (warp == kSStore) {
    // ======================== y store thread =================================
    if (a.prefetch_weights) {
      pdl_wait_prior();
      pdl_launch_dependents();
    }
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
        int s2, c2;
        const bool sh2 = unit(u, s2, c2);
        issue(sh2, s2, c2, u, 2, 0ull);
      }
    }
    uint32_t ypar = 0u;
    int s = s_ex0, c = c_ex0;
    DevSeg g = desc(1, s);
    int n = clamp_rows(g.token_count);
    for (int u = nS; u < U; ++u, ++c) {
      if (c == NCO) {
        c = 0;
        ++s;
      }
      if (u == nS || c == 0) {
        g = desc(1, s);
        n = clamp_rows(g.token_count);
      }
      if (!y_by_tma(n)) continue;  // the compute warps store and free this stage
      const int stage = u % S;
      bool ok = !*s_bad;
      if (ok && !mbar_wait_bounded(&ydone[stage], (ypar >> stage) & 1u, a.err)) {
        *s_bad = 1;
        ok = false;
      }
      ypar ^= 1u << stage;
      if (ok) {
        tma_store_3d(&a.tmap_y[box_index(n)], 0, g.token_start, (c * kStageCols) / kBoxCols, stage_base + stage * C::STAGE);
        bulk_commit();
        bulk_wait_read();
      }
      mbar_arrive_n(&empty[stage], kSW);
    }
    bulk_wait_all();
    return;
  }

  // ============================ compute warps ==================================
  if (a.prefetch_weights) {
    pdl_wait_prior();
    pdl_launch_dependents();
  }
  const int g = lane >> 2;
  const int cq = lane & 3;
  T* yg = static_cast<T*>(a.y);
  auto wait_full = [&](int u) -> bool {
    if (*s_bad) return false;
    const unsigned long long tw = tr.before_wait();
    const bool ok = mbar_wait_bounded(&full[u % S], (u / S) & 1, a.err);
    tr.after_wait(tw);
    if (!ok) *s_bad = 1;
    return ok;
  };

  // shared-memory offsets of this thread's ldmatrix rows, relative to a stage
  uint32_t offA[2][MT], offX[2][2], offB[KS][2], offY[4];
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
#pragma unroll
  for (int ks = 0; ks < KS; ++ks)
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int row = warp * 32 + m * 16 + (lane & 15);
      uint32_t lin = static_cast<uint32_t>(row * (2 * R) + (2 * ks + (lane >> 4)) * 16);
      if constexpr (R >= 16) lin ^= (lin >> 3) & (R == 64 ? 0x70u : (R == 32 ? 0x30u : 0x10u));
      offB[ks][m] = 4 * C::XBOX + lin;
    }
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int t = nt * 8 + (lane & 7);
    const int chunk = (warp & 1) * 4 + (lane >> 3);
    offY[nt] = t * 128 + (((chunk ^ t) & 7) << 4);  // + slice (warp / 2)
  }

  float acc_s[MT][4][4];  // shrink partial of the current run
  int sh_run_first_chunk = 0;
  int s = s_sh0, c = c_sh0;
  DevSeg sg = desc(0, s);
  int n = 0, np = 0, nts = 0;
  uint32_t xsl = 0;
  for (int u = 0; u < nS; ++u, ++c) {
    if (c == NCD) {
      c = 0;
      ++s;
    }
    const bool run_start = u == 0 || c == 0;
    const bool run_end = u == nS - 1 || c == NCD - 1;
    const int stage = u % S;
    if (run_start) {
      sg = desc(0, s);
      n = clamp_rows(sg.token_count);
      np = (n + 15) >> 4;
      nts = (n + 7) >> 3;
      xsl = static_cast<uint32_t>((warp >> 1) * ((8 << box_index(n)) * 128));
      if (tid == 0 && n == 0 && a.err) atomicOr(a.err, kErrBadSegment);
    }
    {
      // ---- shrink stage: D[rank, t] += A[rank, k] . x[t, k]^T (mma.sync) ------
      if (run_start) {
        sh_run_first_chunk = c;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc_s[mt][j][e] = 0.f;
      }
      if (wait_full(u) && n > 0) {
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
                mma_k16<T>(acc_s[mt][2 * p], af[ks][mt], bx[ks][p][0], bx[ks][p][1]);
                if (2 * p + 1 < nts) mma_k16<T>(acc_s[mt][2 * p + 1], af[ks][mt], bx[ks][p][2], bx[ks][p][3]);
              }
            }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (run_end) {
        // ---- end of a shrink run: one partial per (segment, run) -------------
        // cross-warp sum in a fixed order: warps 4-7 park, warps 0-3 add and park
        auto park = [&](float* dst) {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int r = mt * 16 + g + (e >> 1) * 8;
                const int t = j * 8 + 2 * cq + (e & 1);
                if (r < R) dst[t * PITCH + r] = acc_s[mt][j][e];
              }
        };
        if (warp >= 4) park(Pw + (warp - 4) * C::PSLOT);
        named_sync(kSBar, kSCT);
        if (warp < 4) {
          const float* src = Pw + warp * C::PSLOT;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int r = mt * 16 + g + (e >> 1) * 8;
                const int t = j * 8 + 2 * cq + (e & 1);
                if (r < R) acc_s[mt][j][e] += src[t * PITCH + r];
              }
          park(Pw + warp * C::PSLOT);
        }
        named_sync(kSBar, kSCT);
        // this run's partial -> part[token][chunk of the run's first item][R]
        const int pi = sh_run_first_chunk;
        constexpr int Q4 = R / 4;
        for (int e4 = tid; e4 < n * Q4; e4 += kSCT) {
          const int t = e4 / Q4;
          const int r0 = (e4 % Q4) * 4;
          const int off = t * PITCH + r0;
          float4 v;
          const float4 p0 = *reinterpret_cast<const float4*>(Pw + off);
          const float4 p1 = *reinterpret_cast<const float4*>(Pw + C::PSLOT + off);
          const float4 p2 = *reinterpret_cast<const float4*>(Pw + 2 * C::PSLOT + off);
          const float4 p3 = *reinterpret_cast<const float4*>(Pw + 3 * C::PSLOT + off);
          v.x = (p0.x + p1.x) + (p2.x + p3.x);
          v.y = (p0.y + p1.y) + (p2.y + p3.y);
          v.z = (p0.z + p1.z) + (p2.z + p3.z);
          v.w = (p0.w + p1.w) + (p2.w + p3.w);
          *reinterpret_cast<float4*>(a.part + (static_cast<int64_t>(sg.token_start + t) * a.pmax + pi) * R + r0) = v;
        }
        named_sync(kSBar, kSCT);
        // release: this run's partial (written by every compute thread before the barrier)
        if (tid == 0) st_release_gpu(&a.rflag[s * NCD + pi], 1);
      }
    }
  }

  uint32_t hb[4][KS][2];  // H fragments of the current expand run
  int hruns = 0;
  s = s_ex0;
  c = c_ex0;
  int ntn = 0;
  bool tmy = false;
  for (int u = nS; u < U; ++u, ++c) {
    if (c == NCO) {
      c = 0;
      ++s;
    }
    const bool run_start = u == nS || c == 0;
    const int stage = u % S;
    if (run_start) {
      sg = desc(1, s);
      n = clamp_rows(sg.token_count);
      ntn = (n + 7) >> 3;
      tmy = y_by_tma(n);  // the store thread writes the y box back and frees the stage
      xsl = static_cast<uint32_t>((warp >> 1) * ((8 << box_index(n)) * 128));
    }
    // ---- expand stage: D^T[o, t] = y + B[o, :] . H[t, :]^T (mma.sync) ---------
    if (run_start) {
      // H of the run: every shrink run of the segment has published its
      // partial (each thread polls the flag of one run start), then each
      // thread adds one 4-float element of all partials in chunk order --
      // the loads of up to 8 runs in flight together -- and scales by alpha.
      const int NS = nseg * NCD;
      for (int c0 = 0; c0 < NCD; c0 += kSCT) {
        const int cc = c0 + tid;
        const bool st = cc < NCD && item_starts_run(s * NCD + cc, s * NCD, NS, G);
        const uint32_t b = __ballot_sync(0xffffffffu, st);
        if (lane == 0 && c0 / 32 + warp < kSMaskWords) runmask[c0 / 32 + warp] = b;
        if (st && !*s_bad && !wait_flag(&a.rflag[s * NCD + cc], a.err)) *s_bad = 1;
      }
      named_sync(kSBar, kSCT);
      asm volatile("fence.acq_rel.gpu;" ::: "memory");  // every thread sees every published partial
      constexpr int Q4 = R / 4;
      const int nw = min((NCD + 31) / 32, kSMaskWords);
      for (int e4 = tid; e4 < n * Q4; e4 += kSCT) {
        const int t = e4 / Q4;
        const int r0 = (e4 - t * Q4) * 4;
        const float* src = a.part + static_cast<int64_t>(sg.token_start + t) * a.pmax * R + r0;
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        int w = 0;
        uint32_t bits = nw > 0 ? runmask[0] : 0u;
        bool more = true;
        while (more) {
          // next (up to) 8 run starts in chunk order
          int pl[8];
          int np8 = 0;
          while (np8 < 8) {
            while (!bits && ++w < nw) bits = runmask[w];
            if (!bits) break;
            pl[np8++] = w * 32 + __ffs(bits) - 1;
            bits &= bits - 1;
          }
          more = np8 == 8;
          float4 v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (q < np8) v[q] = __ldcg(reinterpret_cast<const float4*>(src + pl[q] * R));
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (q < np8) {
              sum.x += v[q].x;
              sum.y += v[q].y;
              sum.z += v[q].z;
              sum.w += v[q].w;
            }
        }
        sum.x *= alpha_h;
        sum.y *= alpha_h;
        sum.z *= alpha_h;
        sum.w *= alpha_h;
        *reinterpret_cast<float4*>(Hsl + t * R + r0) = sum;
      }
      named_sync(kSBar, kSCT);
      if (tid == 0) mbar_arrive(&hread[hruns & 1]);  // partials read: the bookkeeping warp may count
      const float* Hr = Hsl;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const float* hrow = Hr + (nt * 8 + g) * R;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const int k0 = ks * 16 + 2 * cq;
          const float2 x0 = *reinterpret_cast<const float2*>(hrow + k0);
          const float2 x1 = R >= 16 ? *reinterpret_cast<const float2*>(hrow + k0 + 8) : make_float2(0.f, 0.f);
          hb[nt][ks][0] = E::pack2(x0.x, x0.y);
          hb[nt][ks][1] = E::pack2(x1.x, x1.y);
        }
      }
      ++hruns;
    }
    if (wait_full(u) && n > 0) {
      const uint8_t* st = stage_base + stage * C::STAGE;
      const int oc = c * kStageCols;
      const int wc = min(kStageCols, a.o - oc);
      const uint32_t sb = smem_u32(st);
      const bool ysm = a.y_tma != 0;
      uint32_t yf[4][4];
      float acc[2][4][4];
      if (ysm) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          if (nt < ntn) ldsm_x4_t(sb + xsl + offY[nt], yf[nt][0], yf[nt][1], yf[nt][2], yf[nt][3]);
      }
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          float2 f0 = make_float2(0.f, 0.f), f1 = make_float2(0.f, 0.f);
          if (ysm && nt < ntn) {
            f0 = E::unpack2(yf[nt][2 * m]);
            f1 = E::unpack2(yf[nt][2 * m + 1]);
          }
          acc[m][nt][0] = f0.x;
          acc[m][nt][1] = f0.y;
          acc[m][nt][2] = f1.x;
          acc[m][nt][3] = f1.y;
        }
      if constexpr (R >= 16) {
        constexpr int KB = KS > 2 ? 2 : KS;
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
#pragma unroll
                for (int m = 0; m < 2; ++m) mma_k16<T>(acc[m][nt], bA[kk][m], hb[nt][k0 + kk][0], hb[nt][k0 + kk][1]);
              }
        }
      } else {
        uint32_t bf[4];
        ldsm_x4(sb + 4 * C::XBOX + (warp * 32 + lane) * 16, bf[0], bf[1], bf[2], bf[3]);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          if (nt < ntn) {
#pragma unroll
            for (int m = 0; m < 2; ++m) mma_k8<T>(acc[m][nt], bf[2 * m], bf[2 * m + 1], hb[nt][0][0]);
          }
      }
      if (ysm) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          if (nt < ntn)
            stsm_x4_t(sb + xsl + offY[nt], E::pack2(acc[0][nt][0], acc[0][nt][1]), E::pack2(acc[0][nt][2], acc[0][nt][3]),
                      E::pack2(acc[1][nt][0], acc[1][nt][1]), E::pack2(acc[1][nt][2], acc[1][nt][3]));
        if (tmy) {
          fence_proxy_async_smem();  // the tensor store reads these writes
        } else {
          __syncwarp();
          const int sub = lane & 3;
          const int colw = warp * 32 + sub * 8;
          const int chunk = (warp & 1) * 4 + sub;
          const uint8_t* ybox = st + xsl;
          T* ycol = yg + static_cast<int64_t>(sg.token_start) * a.y_ld + a.y_off + oc + colw;
          if (colw + 8 <= wc) {
            int4 out[4];
#pragma unroll
            for (int it = 0; it < 4; ++it) {
              const int row = (lane >> 2) + 8 * it;
              if (row < n) out[it] = *reinterpret_cast<const int4*>(ybox + row * 128 + (((chunk ^ row) & 7) << 4));
            }
#pragma unroll
            for (int it = 0; it < 4; ++it) {
              const int row = (lane >> 2) + 8 * it;
              if (row < n) *reinterpret_cast<int4*>(ycol + static_cast<int64_t>(row) * a.y_ld) = out[it];
            }
          } else if (colw < wc) {
            for (int it = 0; it < 4; ++it) {
              const int row = (lane >> 2) + 8 * it;
              if (row < n) {
                const T* src = reinterpret_cast<const T*>(ybox + row * 128 + (((chunk ^ row) & 7) << 4));
                for (int x = 0; x < wc - colw; ++x) ycol[static_cast<int64_t>(row) * a.y_ld + x] = src[x];
              }
            }
          }
        }
      } else {
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int t = nt * 8 + 2 * cq + (e & 1);
              const int col = warp * 32 + m * 16 + g + (e >> 1) * 8;
              if (t < n && col < wc) {
                T* yp = yg + static_cast<int64_t>(sg.token_start + t) * a.y_ld + a.y_off + oc + col;
                *yp = E::from_f(E::to_f(*yp) + acc[m][nt][e]);
              }
            }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(tmy ? &ydone[stage] : &empty[stage]);
  }

  if (*s_bad) {
    // drain: copies may still be in flight into stages issued but not consumed
    named_sync(kSBar, kSCT);
    if (tid == 0) {
      const int issued = *s_issued;
      for (int u = max(0, issued - S); u < issued; ++u) mbar_wait_bounded(&full[u % S], (u / S) & 1, nullptr, 10000000ull);
    }
  }
  tr.finish();
}

template <typename T, int R, bool TR>
struct SplitKernel {
  static bool prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return true;
    if (cudaFuncSetAttribute(split_kernel<T, R, TR>, cudaFuncAttributeMaxDynamicSharedMemorySize, SplitCfg<R>::SMEM) !=
        cudaSuccess)
      return false;
    done.fetch_or(bit);
    return true;
  }
  static cudaError_t launch(const ApplyArgs& a, const LaunchCfg& lc) {
    if (!prepare()) return cudaGetLastError();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(lc.grid);
    cfg.blockDim = dim3(kSThreads);
    cfg.dynamicSmemBytes = SplitCfg<R>::SMEM;
    cfg.stream = lc.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = lc.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, split_kernel<T, R, TR>, a);
  }
  static int max_grid() {
    if (!prepare()) return 0;
    int per_sm = 0, dev = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, split_kernel<T, R, TR>, kSThreads, SplitCfg<R>::SMEM) !=
        cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return per_sm > 0 ? sms : 0;  // one CTA per SM
  }
};

template <typename T>
cudaError_t split_by_rank(int rank, const ApplyArgs& a, const LaunchCfg& lc) {
  switch (rank) {
    case 8: return a.trace ? SplitKernel<T, 8, true>::launch(a, lc) : SplitKernel<T, 8, false>::launch(a, lc);
    case 16: return a.trace ? SplitKernel<T, 16, true>::launch(a, lc) : SplitKernel<T, 16, false>::launch(a, lc);
    case 32: return a.trace ? SplitKernel<T, 32, true>::launch(a, lc) : SplitKernel<T, 32, false>::launch(a, lc);
    case 64: return a.trace ? SplitKernel<T, 64, true>::launch(a, lc) : SplitKernel<T, 64, false>::launch(a, lc);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
int split_grid_by_rank(int rank) {
  switch (rank) {
    case 8: return SplitKernel<T, 8, false>::max_grid();
    case 16: return SplitKernel<T, 16, false>::max_grid();
    case 32: return SplitKernel<T, 32, false>::max_grid();
    case 64: return SplitKernel<T, 64, false>::max_grid();
    default: return 0;
  }
}

}  // namespace

cudaError_t launch_apply_split(int dtype, int rank, const ApplyArgs& a, const LaunchCfg& lc) {
  return dtype == 1 ? split_by_rank<__nv_bfloat16>(rank, a, lc) : split_by_rank<__half>(rank, a, lc);
}

int apply_split_max_grid(int dtype, int rank) {
  return dtype == 1 ? split_grid_by_rank<__nv_bfloat16>(rank) : split_grid_by_rank<__half>(rank);
}

}  // namespace wp
