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
// graph) and organised in thread-block clusters of CL CTAs; cluster c takes
// segments c, c + G, c + 2G, ... of the device-resident table. For one segment
// the CL CTAs of the cluster
//   1. split d in CL slices: CTA q streams A[:, slice q] and x[segment rows,
//      slice q] and accumulates a [<=32 x r] fp32 partial with mma.sync;
//   2. reduce the partials through distributed shared memory: after a
//      cluster barrier, CTA q sums rows [q*n/CL, (q+1)*n/CL) over the CL
//      partials (fixed order: deterministic) and writes the scaled rows into
//      the H tile of every CTA of the cluster (reduce-scatter + all-gather);
//   3. split o in CL slices: CTA q streams B[slice q, :] and y[segment rows,
//      slice q] and adds H . B^T to y, rounding once.
// H never leaves the cluster; there are no global atomics and no second launch.
// The same kernel runs the shrink alone (H written to global memory, for the
// tensor-parallel all-reduce and the registry-path shrink()) or the expand
// alone (H read from global memory).
//
// Warp roles: warp 8 is the producer. Its lane 0 issues every TMA load of the
// CTA into a ring of STAGES shared-memory stages, each completing on a "full"
// mbarrier, and refills a stage as soon as the 8 compute warps have arrived
// on its "empty" mbarrier. The compute warps never wait for one another
// inside the stage loop, and the producer keeps loading (across segment and
// phase boundaries -- the expand-phase loads of B and y do not depend on H)
// while the compute warps run the cluster reduction.
//
// Data movement: A and x arrive as tiled tensor loads (cp.async.bulk.tensor)
// of 64-column boxes with the 128-byte swizzle -- conflict-free fragment
// loads, zero fill past the ends of d and T; x and y boxes are 8, 16 or 32
// rows high to match the segment. B (contiguous per column chunk) arrives as
// one 1-D bulk copy (cp.async.bulk). One stage carries 256 elements of d
// (shrink) or 256 output columns (expand). The cluster's segment descriptors
// are cached in shared memory once per launch.
//
// Math: mma.sync m16n8k16 (bf16/fp16 in, fp32 accumulate). Decode segments are
// 1..32 tokens, far below the 128-row tiles of the tcgen05 unit, and the
// kernel is bound by HBM bandwidth. In the expand, H enters the MMA split into
// a 16-bit high part and a 16-bit residual, which keeps ~16 mantissa bits of
// the fp32 H.
//
// Programmatic dependent launch: every thread waits on the predecessor
// (griddepcontrol.wait) before it triggers the dependents, so the pre-wait
// prologue overlaps only the immediately preceding kernel. When the host says
// the table and the weights are not written by that kernel, the prologue
// reads the table and starts the weight loads (A, B) before the wait;
// activations (x, y, H) are always loaded after it.
//
// Waits are bounded (1 s). A timed-out wait raises an error bit and marks the
// CTA bad: compute stops, the producer stops issuing, the compute warps keep
// arriving on the empty barriers and keep taking part in the cluster barriers
// (so no partner is left waiting), copies in flight are drained with a short
// bounded wait, and the kernel exits.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "wp_device.cuh"
#include "wp_internal.h"

namespace wp {

constexpr int kComputeWarps = 8;
constexpr int kComputeThreads = kComputeWarps * 32;
constexpr int kThreads = kComputeThreads + 32;  // + the producer warp
constexpr int kBarCompute = 1;  // named barrier of the compute warps
constexpr int kDescCache = 64;  // segment descriptors cached per CTA
constexpr unsigned long long kDrainNs = 10000000ull;  // 10 ms per stage when draining after an error

template <int R>
struct ApplyCfg {
  static constexpr int KC = kStageK;  // d elements per shrink stage (4 boxes)
  static constexpr int W = kStageCols;  // output columns per expand stage (4 boxes)
  static constexpr int ABOX = R * 128;  // one A box: R rows x 128 B
  static constexpr int XBOX = 32 * 128;  // room for one 32-row x or y box
  static constexpr int STAGE = 4 * ABOX + 4 * XBOX;  // == 4 * XBOX + W * R * 2; multiple of 1024
  static_assert(STAGE == 4 * XBOX + W * R * 2, "shrink and expand stages have one size");
  static constexpr int STAGES = R == 64 ? 3 : (R == 32 ? 5 : (R == 16 ? 7 : 8));
  static constexpr int PITCH = R + 4;  // floats per row of the P / H tiles
  static constexpr int OFF_FLAGS = 448;
  static constexpr int OFF_DESC = 512;
  static constexpr int OFF_RED = OFF_DESC + kDescCache * 32;
  static constexpr int OFF_P = OFF_RED + kComputeWarps * 8 * 32 * 4;
  static constexpr int OFF_H = OFF_P + 32 * PITCH * 4;
  static constexpr int OFF_END = OFF_H + 32 * PITCH * 4;
  static constexpr int SMEM = OFF_END + 1024 + STAGES * STAGE;
};

__device__ __forceinline__ DevSeg unpack_seg(int4 v0, int4 v1) {
  DevSeg s;
  s.adapter_id = v0.x;
  s.token_start = v0.y;
  s.token_count = v0.z;
  s.alpha = __int_as_float(v0.w);
  s.a = reinterpret_cast<const void*>((static_cast<uint64_t>(static_cast<uint32_t>(v1.y)) << 32) |
                                      static_cast<uint32_t>(v1.x));
  s.b = reinterpret_cast<const void*>((static_cast<uint64_t>(static_cast<uint32_t>(v1.w)) << 32) |
                                      static_cast<uint32_t>(v1.z));
  return s;
}

// Descriptor i of a table in global memory (read through L2: the table is
// rewritten between launches).
__device__ __forceinline__ DevSeg load_seg(const DevSeg* segs, int i) {
  const int4* p = reinterpret_cast<const int4*>(segs + i);
  return unpack_seg(__ldcg(p), __ldcg(p + 1));
}

// Rows of a segment clamped to [0, 32] (0 for a malformed entry).
__device__ __forceinline__ int clamp_rows(int n) { return (n < 1 || n > kSegTokens) ? 0 : n; }

// Index of the x / y box height (8 << i rows) covering n rows.
__device__ __forceinline__ int box_index(int n) { return n <= 8 ? 0 : (n <= 16 ? 1 : 2); }

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  const uintptr_t v = reinterpret_cast<uintptr_t>(p);
  return reinterpret_cast<uint8_t*>((v + 1023) & ~static_cast<uintptr_t>(1023));
}

// Optional phase trace (a.trace != nullptr), kept by thread 0 (compute) and by
// the producer's lane 0 (its wait time only).
struct Trace {
  unsigned long long* rec = nullptr;
  unsigned long long t_start = 0, t_dep = 0, t_first = 0, waited = 0, units = 0;
  __device__ void init(unsigned long long* base, bool me) {
    if (base && me) {
      rec = base + blockIdx.x * kTraceSlots;
      t_start = global_timer_ns();
    }
  }
  __device__ void dep() {
    if (rec) t_dep = global_timer_ns();
  }
  __device__ unsigned long long before_wait() {
    if (!rec) return 0ull;
    const unsigned long long t = global_timer_ns();
    if (units < kTraceUnits) rec[8 + 4 * units] = t;
    return t;
  }
  __device__ void after_wait(unsigned long long t0) {
    if (rec) {
      const unsigned long long t = global_timer_ns();
      if (!t_first) t_first = t;
      waited += t - t0;
      if (units < kTraceUnits) rec[8 + 4 * units + 1] = t;
      ++units;
    }
  }
  __device__ void mark(int k) {  // 2: compute done, 3: stage handed back
    if (rec && units >= 1 && units <= kTraceUnits) rec[8 + 4 * (units - 1) + k] = global_timer_ns();
  }
  __device__ void finish() {
    if (rec) {
      rec[0] = t_start;
      rec[1] = t_dep;
      rec[2] = t_first;
      rec[3] = global_timer_ns();
      rec[4] = units;
      rec[5] = waited;
    }
  }
};

template <typename T, int R>
__global__ void __launch_bounds__(kThreads, 1) apply_kernel(const __grid_constant__ ApplyArgs a) {
  using C = ApplyCfg<R>;
  using E = Elem<T>;
  constexpr int S = C::STAGES;
  constexpr int NT = R / 8;  // shrink: n-tiles of 8 rank columns
  constexpr int KP = kComputeWarps / NT;  // shrink: warps sharing one n-tile (split over k-steps)
  constexpr int KS = C::KC / 16;  // shrink: k16 steps per stage
  constexpr int NTW = C::W / 8 / kComputeWarps;  // expand: n-tiles of 8 columns per warp
  constexpr int KE = R >= 16 ? R / 16 : 1;  // expand: k-steps over the rank
  constexpr int PITCH = C::PITCH;

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + 128);
  uint64_t* cbar = reinterpret_cast<uint64_t*>(smem + 256);
  volatile int* s_bad = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS);
  volatile int* s_issued = reinterpret_cast<volatile int*>(smem + C::OFF_FLAGS + 4);
  int4* sdesc = reinterpret_cast<int4*>(smem + C::OFF_DESC);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  float* Ps = reinterpret_cast<float*>(smem + C::OFF_P);
  float* Hs = reinterpret_cast<float*>(smem + C::OFF_H);
  uint8_t* stage_base = align1024(smem + C::OFF_END);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const bool producer = warp == kComputeWarps;
  const uint32_t q = cluster_ctarank();
  const uint32_t CL = cluster_nctarank();
  const int cid = static_cast<int>(cluster_id_x());
  const int G = static_cast<int>(cluster_count_x());
  Trace tr;
  tr.init(a.trace, tid == 0);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kComputeWarps);
    }
    mbar_init(cbar, CL);
    *s_bad = 0;
    *s_issued = 0;
    fence_mbar_init();
  }
  if (producer && lane == 0) {
    if (a.mode & kModeShrink) {
      for (int i = 0; i < 3; ++i) prefetch_tmap(&a.tmap_x[i]);
      if (!a.registry) prefetch_tmap(&a.tmap_a);
    }
    if ((a.mode & kModeExpand) && a.y_tma)
      for (int i = 0; i < 3; ++i) prefetch_tmap(&a.tmap_y[i]);
  }
  __syncthreads();
  cluster_sync_hw();  // every CTA's cluster barrier is initialised before anyone arrives on it

  const bool do_sh = (a.mode & kModeShrink) != 0;
  const bool do_ex = (a.mode & kModeExpand) != 0;
  const int kA0 = static_cast<int>(q) * a.split_len;
  const int nA = do_sh ? (max(0, min(a.split_len, a.d - kA0)) + C::KC - 1) / C::KC : 0;
  const int oB0 = static_cast<int>(q) * a.oslice;
  const int nB = do_ex ? (max(0, min(a.oslice, a.o - oB0)) + C::W - 1) / C::W : 0;
  const int ups = nA + nB;  // stages per segment for this CTA

  // ---- segment table of this cluster (all threads) -------------------------
  int nmine = 0;
  auto read_table = [&]() {
    const int nseg = __ldcg(a.num_segs);
    nmine = nseg > cid ? (nseg - cid + G - 1) / G : 0;
    const int cached = min(nmine, kDescCache);
    for (int j = tid; j < 2 * cached; j += kThreads)
      sdesc[j] = __ldcg(reinterpret_cast<const int4*>(a.segs + cid + (j >> 1) * G) + (j & 1));
    __syncthreads();
  };
  auto desc = [&](int j) -> DevSeg {
    if (j >= kDescCache) return load_seg(a.segs, cid + j * G);
    return unpack_seg(sdesc[2 * j], sdesc[2 * j + 1]);  // shared-memory copy
  };

  if (a.prefetch_weights) {
    read_table();
  } else {
    pdl_wait_prior();
    pdl_launch_dependents();
    tr.dep();
    read_table();
  }
  const int total = nmine * ups;

  if (producer) {
    // ======================= producer warp ===================================
    if (lane == 0) {
      // parts: 1 = arm the stage's barrier and load the weights, 2 = load the activations
      auto issue = [&](int u, int stage, int parts) {
        const DevSeg s = desc(u / ups);
        const int sub = u % ups;
        const int n = clamp_rows(s.token_count);
        const int bi = box_index(n);
        const uint32_t box_bytes = (8u << bi) * 128u;
        uint8_t* st = stage_base + stage * C::STAGE;
        uint64_t* bar = &full[stage];
        if (sub < nA) {
          const int k0 = kA0 + sub * C::KC;
          if (parts & 1) {
            mbar_arrive_expect_tx(bar, 4 * C::ABOX + 4 * box_bytes);
            const void* amap = a.registry ? s.a : static_cast<const void*>(&a.tmap_a);
            const int aid = a.registry ? 0 : s.adapter_id;
#pragma unroll
            for (int j = 0; j < 4; ++j) tma_load_3d(st + j * C::ABOX, amap, k0 + j * kBoxCols, 0, aid, bar);
          }
          if (parts & 2) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tma_load_2d(st + 4 * C::ABOX + j * C::XBOX, &a.tmap_x[bi], k0 + j * kBoxCols, s.token_start, bar);
          }
        } else {
          const int oc = oB0 + (sub - nA) * C::W;
          const int wc = min(C::W, a.o - oc);
          if (parts & 1) {
            mbar_arrive_expect_tx(bar, wc * R * 2 + (a.y_tma ? 4 * box_bytes : 0u));
            const T* B = a.registry ? static_cast<const T*>(s.b)
                                    : static_cast<const T*>(a.wb_base) +
                                          static_cast<int64_t>(s.adapter_id) * a.wb_stride;
            bulk_g2s(st + 4 * C::XBOX, B + static_cast<int64_t>(oc) * R, wc * R * 2, bar);
          }
          if ((parts & 2) && a.y_tma) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tma_load_2d(st + j * C::XBOX, &a.tmap_y[bi], oc + j * kBoxCols, s.token_start, bar);
          }
        }
      };
      const int first = min(S, total);
      if (a.prefetch_weights) {
        for (int u = 0; u < first; ++u) issue(u, u, 1);
        pdl_wait_prior();
        pdl_launch_dependents();
        for (int u = 0; u < first; ++u) issue(u, u, 2);
      } else {
        for (int u = 0; u < first; ++u) issue(u, u, 3);
      }
      *s_issued = first;
      for (int u = first; u < total; ++u) {
        const int stage = u % S;
        if (!mbar_wait_bounded(&empty[stage], ((u / S) - 1) & 1, a.err)) *s_bad = 1;
        if (*s_bad) break;
        issue(u, stage, 3);
        *s_issued = u + 1;
      }
    } else if (a.prefetch_weights) {
      pdl_wait_prior();
      pdl_launch_dependents();
    }
    return;
  }

  // ========================= compute warps ===================================
  if (a.prefetch_weights) {
    pdl_wait_prior();
    pdl_launch_dependents();
    tr.dep();
  }
  const int g = lane >> 2;
  const int c = lane & 3;
  int kc = 0;  // next stage-unit to consume
  uint32_t cph = 0;

  // Wait for the next stage; true when its data may be used.
  auto acquire = [&](int& stage) -> bool {
    stage = kc % S;
    if (*s_bad) return false;
    const unsigned long long tw = tr.before_wait();
    const bool ok = mbar_wait_bounded(&full[stage], (kc / S) & 1, a.err);
    tr.after_wait(tw);
    if (!ok) *s_bad = 1;
    return ok;
  };
  // Hand the stage back to the producer.
  auto release = [&](int stage) {
    tr.mark(2);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    tr.mark(3);
    ++kc;
  };

  for (int sj = 0; sj < nmine; ++sj) {
    const DevSeg s = desc(sj);
    const int n = clamp_rows(s.token_count);
    if (tid == 0 && n == 0 && a.err) atomicOr(a.err, kErrBadSegment);
    const float alpha = a.registry ? s.alpha : a.scale;

    if (do_sh) {
      // ---- 1. partial shrink over this CTA's slice of d -------------------
      const int nt = warp % NT;
      const int kp = warp / NT;
      float acc[2][2][4];  // [independent chain][m-tile][fragment]
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[x][m][j] = 0.f;
      const bool m1 = n > 16;
      for (int i = 0; i < nA; ++i) {
        int stage;
        if (acquire(stage) && n > 0) {
          const uint8_t* st = stage_base + stage * C::STAGE;
          const int arow = nt * 8 + g;
#pragma unroll
          for (int it = 0; it < KS / KP; ++it) {
            const int ks = kp + it * KP;
            const int box = ks >> 2;
            const int col = (ks & 3) * 16 + 2 * c;
            const uint8_t* ab = st + box * C::ABOX;
            const uint8_t* xb = st + 4 * C::ABOX + box * C::XBOX;
            const uint32_t b0 = lds32(ab + sw128(arow, col));
            const uint32_t b1 = lds32(ab + sw128(arow, col + 8));
            uint32_t af[4];
            af[0] = lds32(xb + sw128(g, col));
            af[1] = lds32(xb + sw128(g + 8, col));
            af[2] = lds32(xb + sw128(g, col + 8));
            af[3] = lds32(xb + sw128(g + 8, col + 8));
            mma_k16<T>(acc[it & 1][0], af, b0, b1);
            if (m1) {
              af[0] = lds32(xb + sw128(g + 16, col));
              af[1] = lds32(xb + sw128(g + 24, col));
              af[2] = lds32(xb + sw128(g + 16, col + 8));
              af[3] = lds32(xb + sw128(g + 24, col + 8));
              mma_k16<T>(acc[it & 1][1], af, b0, b1);
            }
          }
        }
        release(stage);
      }
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[0][m][j] += acc[1][m][j];
      // combine the KP warps of each n-tile, then publish the partial tile
      if constexpr (KP > 1) {
        float* mine = red + warp * 8 * 32;
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int j = 0; j < 4; ++j) mine[(m * 4 + j) * 32 + lane] = acc[0][m][j];
        named_sync(kBarCompute, kComputeThreads);
        if (kp == 0) {
#pragma unroll
          for (int w2 = 1; w2 < KP; ++w2) {
            const float* other = red + (nt + w2 * NT) * 8 * 32;
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
              for (int j = 0; j < 4; ++j) acc[0][m][j] += other[(m * 4 + j) * 32 + lane];
          }
        }
      }
      if (kp == 0) {
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int row = m * 16 + g + hf * 8;
            *reinterpret_cast<float2*>(Ps + row * PITCH + nt * 8 + 2 * c) =
                make_float2(acc[0][m][hf * 2], acc[0][m][hf * 2 + 1]);
          }
      }
      // ---- 2. reduce-scatter + all-gather of the partials over the cluster
      if (!cluster_barrier_bounded(cbar, cph, CL, kBarCompute, kComputeThreads, a.err)) *s_bad = 1;
      cph ^= 1u;
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

    if (do_ex && nB > 0) {
      // ---- 3. expand over this CTA's slice of o ----------------------------
      // H fragments (16-bit high part + residual) of both 16-row tiles.
      uint32_t hi[2][KE][4], lo[2][KE][4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const float* h0 = Hs + (m * 16 + g) * PITCH;
        const float* h1 = h0 + 8 * PITCH;
#pragma unroll
        for (int ks = 0; ks < KE; ++ks) {
          const int k0 = ks * 16 + 2 * c;
          float2 x[4];
          x[0] = *reinterpret_cast<const float2*>(h0 + k0);
          x[1] = *reinterpret_cast<const float2*>(h1 + k0);
          if (R >= 16) {
            x[2] = *reinterpret_cast<const float2*>(h0 + k0 + 8);
            x[3] = *reinterpret_cast<const float2*>(h1 + k0 + 8);
          } else {
            x[2] = x[3] = make_float2(0.f, 0.f);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            hi[m][ks][e] = E::pack2(x[e].x, x[e].y);
            const float2 r = E::unpack2(hi[m][ks][e]);
            lo[m][ks][e] = E::pack2(x[e].x - r.x, x[e].y - r.y);
          }
        }
      }
      const bool m1 = n > 16;
      T* yg = static_cast<T*>(a.y);
      for (int i = 0; i < nB; ++i) {
        int stage;
        if (acquire(stage) && n > 0) {
          const uint8_t* st = stage_base + stage * C::STAGE;
          const uint8_t* Bs = st + 4 * C::XBOX;
          const int oc = oB0 + i * C::W;
          const int wc = min(C::W, a.o - oc);
          float acc[2][NTW][4];
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int j = 0; j < NTW; ++j)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[m][j][e] = 0.f;
#pragma unroll
          for (int j = 0; j < NTW; ++j) {
            const int nt = warp * NTW + j;
            if (nt * 8 < wc) {
#pragma unroll
              for (int ks = 0; ks < KE; ++ks) {
                const uint8_t* brow = Bs + (nt * 8 + g) * (R * 2) + ks * 32 + c * 4;
                const uint32_t b0 = lds32(brow);
                if constexpr (R == 8) {
                  mma_k8<T>(acc[0][j], hi[0][ks][0], hi[0][ks][1], b0);
                  mma_k8<T>(acc[0][j], lo[0][ks][0], lo[0][ks][1], b0);
                  if (m1) {
                    mma_k8<T>(acc[1][j], hi[1][ks][0], hi[1][ks][1], b0);
                    mma_k8<T>(acc[1][j], lo[1][ks][0], lo[1][ks][1], b0);
                  }
                } else {
                  const uint32_t b1 = lds32(brow + 16);
                  mma_k16<T>(acc[0][j], hi[0][ks], b0, b1);
                  mma_k16<T>(acc[0][j], lo[0][ks], b0, b1);
                  if (m1) {
                    mma_k16<T>(acc[1][j], hi[1][ks], b0, b1);
                    mma_k16<T>(acc[1][j], lo[1][ks], b0, b1);
                  }
                }
              }
            }
          }
          // y += acc, one rounding
#pragma unroll
          for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int j = 0; j < NTW; ++j)
#pragma unroll
              for (int hf = 0; hf < 2; ++hf) {
                const int row = m * 16 + g + hf * 8;
                const int col = (warp * NTW + j) * 8 + 2 * c;
                if (row < n && col < wc) {
                  T* yp = yg + static_cast<int64_t>(s.token_start + row) * a.y_ld + a.y_off + oc + col;
                  const float v0 = acc[m][j][hf * 2], v1 = acc[m][j][hf * 2 + 1];
                  if (a.y_tma) {
                    const float2 yv = E::unpack2(lds32(st + (col >> 6) * C::XBOX + sw128(row, col & 63)));
                    *reinterpret_cast<uint32_t*>(yp) = E::pack2(yv.x + v0, yv.y + v1);
                  } else {
                    yp[0] = E::from_f(E::to_f(yp[0]) + v0);
                    yp[1] = E::from_f(E::to_f(yp[1]) + v1);
                  }
                }
              }
        }
        release(stage);
      }
    }
  }

  if (*s_bad) {
    // drain: copies may still be in flight into stages issued but not consumed
    named_sync(kBarCompute, kComputeThreads);
    if (tid == 0) {
      const int issued = *s_issued;
      for (int u = kc; u < issued; ++u) mbar_wait_bounded(&full[u % S], (u / S) & 1, nullptr, kDrainNs);
    }
  }
  tr.finish();
}

// --------------------------------------------------------------------------
// launchers

namespace {

template <typename T, int R>
struct ApplyKernel {
  static bool prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return true;
    if (cudaFuncSetAttribute(apply_kernel<T, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, ApplyCfg<R>::SMEM) !=
        cudaSuccess)
      return false;
    done.fetch_or(bit);
    return true;
  }

  static cudaError_t launch(const ApplyArgs& a, const LaunchCfg& lc) {
    if (!prepare()) return cudaGetLastError();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(lc.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = ApplyCfg<R>::SMEM;
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
    return cudaLaunchKernelEx(&cfg, apply_kernel<T, R>, a);
  }

  static int max_grid(int cluster) {
    if (!prepare()) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cluster * 64);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = ApplyCfg<R>::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nclusters = 0;
    if (cudaOccupancyMaxActiveClusters(&nclusters, apply_kernel<T, R>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    return nclusters * cluster;
  }
};

template <typename T>
cudaError_t apply_by_rank(int rank, const ApplyArgs& a, const LaunchCfg& lc) {
  switch (rank) {
    case 8: return ApplyKernel<T, 8>::launch(a, lc);
    case 16: return ApplyKernel<T, 16>::launch(a, lc);
    case 32: return ApplyKernel<T, 32>::launch(a, lc);
    case 64: return ApplyKernel<T, 64>::launch(a, lc);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
int max_grid_by_rank(int rank, int cluster) {
  switch (rank) {
    case 8: return ApplyKernel<T, 8>::max_grid(cluster);
    case 16: return ApplyKernel<T, 16>::max_grid(cluster);
    case 32: return ApplyKernel<T, 32>::max_grid(cluster);
    case 64: return ApplyKernel<T, 64>::max_grid(cluster);
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

}  // namespace wp
