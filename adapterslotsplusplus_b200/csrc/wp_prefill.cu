// wp_prefill.cu -- the prefill apply: long runs of one adapter as GEMMs on
// the 5th-generation tensor cores (tcgen05.mma, accumulators in TMEM).
//
// Semantics as in wp_apply.cu (reference math: tests/correctness/reference_bgmv.py:4-18):
//   H[t, :] = alpha * x[t, :] . A^T (fp32), y[t, j] = round(y[t, j] + H[t, :] . B[j, :])
// The reference has no prefill kernel: it cuts every run into pieces of at
// most 32 tokens (WP_MAX_SEGMENT_TOKENS, csrc/bridge/warp_pipe_metadata.h:22,
// split at csrc/kernels/warp_pipe_r32.cu:498-511) and runs them through its
// decode kernels. Here the segmenter (prefill mode) cuts runs of at least
// kPrefillMinRun tokens into tiles of kPrefillTile = 128 tokens instead, and
// a call applies them with two kernels:
//
//   prefill_shrink_kernel: items (tile, 1024-column chunk of d), split evenly
//     over the grid. Per item 4 stages of 256 columns: x box [128 tokens x
//     256] and A box [r x 256] by TMA; per stage 16 tcgen05.mma with M = 128
//     tokens, N = r, K = 16 into a TMEM accumulator (two, alternating, so the
//     next item's MMAs overlap this item's read-out); the epilogue warps read
//     it with tcgen05.ld (thread = token row) and write the fp32 partial to
//     scratch part[(token) * nKC + chunk][r] -- every slot written once, no
//     atomics.
//   prefill_expand_kernel: items (tile, 64 output columns), split evenly.
//     When its tile changes a CTA adds the tile's nKC partials (fixed order),
//     scales by alpha and writes H as a bf16/fp16 [128 x r] tile in shared
//     memory in the swizzle the tensor core reads; per item one B box [64 x
//     r] and the y tile [128 x 64] by TMA into a ring of 6-8 stages, and r /
//     16 tcgen05.mma with M = 128 tokens, N = 64, K = 16 into one of four
//     TMEM accumulators [128 lanes x 64 columns]; eight epilogue warps
//     (token row = TMEM lane, 32 columns each) add y from shared memory and
//     round once into the y tile, which a store thread sends back with one
//     tensor store (a tile with fewer than 128 rows: 16-byte row stores).
//
// Warp roles (192 threads): warps 0-3 epilogue (TMEM lane quarter w), warp 4
// lane 0 TMA producer, warp 5 lane 0 MMA issuer; hand-offs only through
// mbarriers (full / empty stages, acc_full / acc_free accumulators, h_full /
// h_free for the H tile). Waits are bounded (1 s): a timed-out wait raises
// the error bit, stops issuing and lets the other roles run to their end.
// Ranks 16, 32 and 64 (K of kind::f16 is 16); d and o multiples of 64.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "wp_device.cuh"
#include "wp_internal.h"
#include "wp_kernel_common.cuh"

namespace wp {
namespace {

constexpr int kPfThreads = 192;
// expand kernel: 8 epilogue warps (two per TMEM lane quarter, 128 columns
// each), then the producer, MMA and y store warps
constexpr int kPfExEpi = 8;
constexpr int kPfExProd = 8;
constexpr int kPfExMma = 9;
constexpr int kPfExStore = 10;
constexpr int kPfExThreads = (kPfExEpi + 3) * 32;
constexpr int kPfEpi = 4;  // epilogue warps
constexpr int kPfProd = 4;  // producer warp
constexpr int kPfMma = 5;  // MMA warp
constexpr int kPfBar = 2;  // named barrier of the epilogue warps
constexpr int kPfKC = 1024;  // d columns per shrink item
constexpr int kPfStagesPerItem = kPfKC / kStageK;  // 4
constexpr int kPfN = 64;  // output columns per expand item (N of its MMAs)
constexpr int kPfAcc = 4;  // TMEM accumulators of the expand kernel (kPfN columns each)

// Optional per-CTA timeline of the expand kernel (a.trace; 64 stamps per
// CTA): 0 start, 1 epilogue past the dependency wait, 2 first H built, 3 end;
// item k < 16: 8 + 3k accumulator and y tile ready, 9 + 3k epilogue done,
// 10 + 3k stage released by the store thread.
__device__ __forceinline__ void pf_trace(const ApplyArgs& a, int slot) {
  if (a.trace && slot < 64) a.trace[static_cast<int64_t>(blockIdx.x) * 64 + slot] = global_timer_ns();
}

__device__ __forceinline__ int pf_tiles(const ApplyArgs& a) {
  const int n = __ldcg(a.num_segs);
  return n < 0 ? 0 : (n > a.sync_cap ? a.sync_cap : n);
}

template <int R>
struct PfCfg {
  // shrink stage: 4 x boxes of 128 rows (16 KB each) + 4 A boxes of R rows
  static constexpr int XST = 4 * kPrefillTile * 128;
  static constexpr int AST = 4 * R * 128;
  static constexpr int SH_STAGE = XST + AST;
  static constexpr int SH_S = 2;
  static constexpr int SH_SMEM = 1024 + SH_S * SH_STAGE + 1024;
  static constexpr uint32_t SH_ACC = R < 32 ? 32u : static_cast<uint32_t>(R);  // TMEM columns per accumulator
  // expand stage: the y tile [128 rows x 64 columns = 128 B] and one B box
  // [64 rows x 2R bytes]; H tile [128 rows x 2R bytes]
  static constexpr int YST = kPrefillTile * 128;
  static constexpr int BST = kPfN * R * 2;
  static constexpr int EX_STAGE = YST + BST;
  static constexpr int HT = kPrefillTile * R * 2;
  static constexpr int EX_S = R == 64 ? 6 : 8;
  static constexpr int EX_NAT = 1024 + HT + EX_S * EX_STAGE + 1024;
  // at least 120 KB: one expand CTA per SM, so its 512 TMEM columns never
  // wait on another CTA's allocation
  static constexpr int EX_SMEM = EX_NAT < 122880 ? 122880 : EX_NAT;
  static constexpr uint32_t LAYOUT = R == 64 ? 2u : (R == 32 ? 4u : 6u);  // swizzle of 2R-byte rows
  static constexpr uint32_t SWZ_MASK = R == 64 ? 0x70u : (R == 32 ? 0x30u : 0x10u);
  static_assert(SH_STAGE % 1024 == 0 && EX_STAGE % 1024 == 0 && HT % 1024 == 0 && YST % 1024 == 0,
                "1024-byte aligned tiles");
  static_assert(SH_SMEM <= 232448 && EX_SMEM <= 232448, "shared memory budget");
};

// ============================================================================
// shrink
// ============================================================================
template <typename T, int R>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_shrink_kernel(const __grid_constant__ ApplyArgs a) {
  using C = PfCfg<R>;
  constexpr int S = C::SH_S;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + 64);
  uint64_t* acc_full = reinterpret_cast<uint64_t*>(smem + 128);  // [2]
  uint64_t* acc_free = reinterpret_cast<uint64_t*>(smem + 144);  // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + 192);
  volatile int* s_bad = reinterpret_cast<volatile int*>(smem + 196);
  uint8_t* ring = align1024(smem + 256);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // The tile table may be the previous kernel's output (the segmenter): wait
  // for it first, unless the previous kernel is this call's decode kernel on
  // the short runs (pf_late_wait), which waited for everything before it and
  // touches other rows of x, y and the partial scratch; then the wait comes
  // only before this grid exits, so the expand kernel, which waits for this
  // grid, also follows the decode kernel.
  if (!a.pf_late_wait) pdl_wait_prior();
  pdl_launch_dependents();
  const int nt = pf_tiles(a);
  const int nKC = (a.d + kPfKC - 1) / kPfKC;
  const int nK = (a.d + kStageK - 1) / kStageK;  // 256-column stages of d
  const long long W = static_cast<long long>(nt) * nKC;
  const int G = gridDim.x, c = blockIdx.x;
  const int i0 = static_cast<int>(static_cast<long long>(c) * W / G);
  const int i1 = static_cast<int>(static_cast<long long>(c + 1) * W / G);
  if (i1 <= i0) {  // no items: no TMEM, no barriers
    if (a.pf_late_wait) pdl_wait_prior();
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_free[b], kPfEpi);
    }
    *s_bad = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(s_tmem, 2 * C::SH_ACC);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *s_tmem;
  auto stages_of = [&](int kc) { return min(kPfStagesPerItem, nK - kc * kPfStagesPerItem); };

  if (warp == kPfProd) {
    if (lane == 0) {
      prefetch_tmap(&a.tmap_a);
      prefetch_tmap(&a.tmap_x128);
      const uint64_t ef = l2_evict_first_policy();
      int u = 0;
      for (int it = i0; it < i1 && !*s_bad; ++it) {
        const DevSeg tile = load_seg(a.segs, it / nKC);
        const int kc = it % nKC;
        for (int s = 0; s < stages_of(kc); ++s, ++u) {
          const int stage = u % S;
          if (u >= S && !mbar_wait_bounded(&empty[stage], ((u / S) - 1) & 1, a.err)) {
            *s_bad = 1;
            break;
          }
          uint8_t* st = ring + stage * C::SH_STAGE;
          const int k0 = (kc * kPfStagesPerItem + s) * kStageK;
          mbar_arrive_expect_tx(&full[stage], C::SH_STAGE);
          tma_load_3d(st, &a.tmap_x128, 0, tile.token_start, k0 / kBoxCols, &full[stage]);
          tma_load_4d_ef(st + C::XST, &a.tmap_a, 0, 0, k0 / kBoxCols, tile.adapter_id, &full[stage], ef);
        }
      }
    }
    return;
  }

  if (warp == kPfMma) {
    if (lane == 0) {
      constexpr uint32_t kAb = Elem<T>::is_bf16 ? 1u : 0u;
      const uint32_t idesc = umma_idesc(kAb, kPrefillTile, R);
      int u = 0;
      for (int it = i0, k = 0; it < i1; ++it, ++k) {
        const int b = k & 1;
        if (k >= 2 && !mbar_wait_bounded(&acc_free[b], ((k >> 1) - 1) & 1, a.err)) *s_bad = 1;
        const uint32_t acc = tbase + b * C::SH_ACC;
        const int ns = stages_of(it % nKC);
        for (int s = 0; s < ns; ++s, ++u) {
          const int stage = u % S;
          const bool ok = !*s_bad && mbar_wait_bounded(&full[stage], (u / S) & 1, a.err);
          if (!ok) {
            *s_bad = 1;
            continue;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(ring + stage * C::SH_STAGE);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint64_t dx = umma_desc(st + j * (kPrefillTile * 128), 1024, 2);
            const uint64_t da = umma_desc(st + C::XST + j * (R * 128), 1024, 2);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_f16(acc, dx + 2 * ks, da + 2 * ks, idesc, (s > 0 || j > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);  // the stage is free once these MMAs have read it
        }
        umma_commit(&acc_full[b]);
      }
    }
    return;
  }

  // ============================ epilogue warps =============================
  const int t = warp * 32 + lane;  // token row of the tile = TMEM lane
  for (int it = i0, k = 0; it < i1; ++it, ++k) {
    const int b = k & 1;
    const bool ok = mbar_wait_bounded(&acc_full[b], (k >> 1) & 1, a.err);
    if (!ok) *s_bad = 1;
    tc_fence_after();
    const DevSeg tile = load_seg(a.segs, it / nKC);
    const int kc = it % nKC;
    const uint32_t taddr = tbase + b * C::SH_ACC + (static_cast<uint32_t>(warp * 32) << 16);
    float v[R];
    if constexpr (R == 16) {
      tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(v));
    } else {
#pragma unroll
      for (int h = 0; h < R / 32; ++h) tmem_ld32(taddr + 32 * h, *reinterpret_cast<float(*)[32]>(v + 32 * h));
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&acc_free[b]);
    if (ok && !*s_bad && t < tile.token_count) {
      float4* dst = reinterpret_cast<float4*>(a.part + (static_cast<int64_t>(tile.token_start + t) * nKC + kc) * R);
#pragma unroll
      for (int q = 0; q < R / 4; ++q) __stcg(dst + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
    }
  }
  tc_fence_before();
  named_sync(kPfBar, kPfEpi * 32);  // every TMEM read of this CTA is done
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 2 * C::SH_ACC);
  }
  if (a.pf_late_wait) pdl_wait_prior();
}

// ============================================================================
// expand
// ============================================================================
template <typename T, int R>
__global__ void __launch_bounds__(kPfExThreads, 1) prefill_expand_kernel(const __grid_constant__ ApplyArgs a) {
  using C = PfCfg<R>;
  using E = Elem<T>;
  constexpr int S = C::EX_S;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + 64);
  uint64_t* acc_full = reinterpret_cast<uint64_t*>(smem + 128);  // [kPfAcc]
  uint64_t* acc_free = reinterpret_cast<uint64_t*>(smem + 160);  // [kPfAcc]
  uint64_t* h_full = reinterpret_cast<uint64_t*>(smem + 192);
  uint64_t* h_free = reinterpret_cast<uint64_t*>(smem + 200);
  uint64_t* ydone = reinterpret_cast<uint64_t*>(smem + 256);  // [S] the epilogue has written the stage's y tile
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + 224);
  volatile int* s_bad = reinterpret_cast<volatile int*>(smem + 228);
  uint8_t* Ht = align1024(smem + 512);  // H tile [128 rows x 2R bytes], swizzled
  uint8_t* ring = Ht + C::HT;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // the predecessor is this call's prefill shrink, which writes neither the
  // tile table nor B; the epilogue waits for it before reading the partials
  const int nt = pf_tiles(a);
  const int nO = (a.o + kPfN - 1) / kPfN;
  const int nKC = (a.d + kPfKC - 1) / kPfKC;
  const long long V = static_cast<long long>(nt) * nO;
  const int G = gridDim.x, c = blockIdx.x;
  const int i0 = static_cast<int>(static_cast<long long>(c) * V / G);
  const int i1 = static_cast<int>(static_cast<long long>(c + 1) * V / G);
  if (i1 <= i0) {
    pdl_wait_prior();
    pdl_launch_dependents();
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);  // the MMAs have read B, the store warp is done with y
      mbar_init(&ydone[s], kPfExEpi);
    }
    for (int b = 0; b < kPfAcc; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_free[b], kPfExEpi);
    }
    mbar_init(h_full, 1);
    mbar_init(h_free, 1);
    *s_bad = 0;
    fence_mbar_init();
  }
  if (tid == 0) pf_trace(a, 0);
  if (warp == 0) tmem_alloc(s_tmem, kPfAcc * kPfN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *s_tmem;

  if (warp == kPfExProd) {
    // Lanes 1-31 leave at once: a lane blocked in the dependency wait would
    // hold up the whole warp, lane 0's pre-dependency issue included.
    if (lane != 0) return;
    {
      prefetch_tmap(&a.tmap_b64);
      prefetch_tmap(&a.tmap_y128);
      const uint64_t ef = l2_evict_first_policy();
      for (int it = i0, k = 0; it < i1 && !*s_bad; ++it, ++k) {
        const int stage = k % S;
        if (k >= S && !mbar_wait_bounded(&empty[stage], ((k / S) - 1) & 1, a.err)) {
          *s_bad = 1;
          break;
        }
        if (k == S) {  // the first stages went before the dependency wait
          pdl_wait_prior();
          pdl_launch_dependents();
        }
        const DevSeg tile = load_seg(a.segs, it / nO);
        const int oc = (it % nO) * kPfN;
        uint8_t* st = ring + stage * C::EX_STAGE;
        mbar_arrive_expect_tx(&full[stage], C::EX_STAGE);
        tma_load_3d(st, &a.tmap_y128, 0, tile.token_start, oc / kBoxCols, &full[stage]);
        tma_load_3d_ef(st + C::YST, &a.tmap_b64, 0, oc, tile.adapter_id, &full[stage], ef);
      }
      if (i1 - i0 <= S) {
        pdl_wait_prior();
        pdl_launch_dependents();
      }
    }
    return;
  }

  if (warp == kPfExMma) {
    pdl_wait_prior();
    pdl_launch_dependents();
    if (lane == 0) {
      constexpr uint32_t kAb = Elem<T>::is_bf16 ? 1u : 0u;
      const uint32_t idesc = umma_idesc(kAb, kPrefillTile, kPfN);
      const uint64_t dh = umma_desc(smem_u32(Ht), 16 * R, C::LAYOUT);
      int cur = -1, ti = -1;
      for (int it = i0, k = 0; it < i1; ++it, ++k) {
        const int tile = it / nO;
        if (tile != cur) {
          if (ti >= 0) umma_commit(h_free);  // the previous tile's MMAs have read H
          cur = tile;
          ++ti;
          if (!*s_bad && !mbar_wait_bounded(h_full, ti & 1, a.err)) *s_bad = 1;
        }
        const int b = k % kPfAcc;
        if (k >= kPfAcc && !*s_bad && !mbar_wait_bounded(&acc_free[b], ((k / kPfAcc) - 1) & 1, a.err)) *s_bad = 1;
        const int stage = k % S;
        const bool ok = !*s_bad && mbar_wait_bounded(&full[stage], (k / S) & 1, a.err);
        if (!ok) {
          *s_bad = 1;
          umma_commit(&acc_full[b]);  // let the epilogue move on
          continue;
        }
        tc_fence_after();
        const uint64_t db = umma_desc(smem_u32(ring + stage * C::EX_STAGE + C::YST), 16 * R, C::LAYOUT);
#pragma unroll
        for (int ks = 0; ks < R / 16; ++ks)
          umma_f16(tbase + b * kPfN, dh + 2 * ks, db + 2 * ks, idesc, ks > 0 ? 1u : 0u);
        umma_commit(&empty[stage]);
        umma_commit(&acc_full[b]);
      }
    }
    return;
  }

  if (warp == kPfExStore) {
    // ============================ y store thread ==========================
    // A full tile (128 rows) leaves by one tensor store of the stage's y
    // tile, which the epilogue has overwritten with the result; a partial
    // tile was stored row by row by the epilogue. Then the stage is free.
    pdl_wait_prior();
    pdl_launch_dependents();
    if (lane == 0) {
      prefetch_tmap(&a.tmap_y128);
      for (int it = i0, k = 0; it < i1; ++it, ++k) {
        const int stage = k % S;
        const bool ok = mbar_wait_bounded(&ydone[stage], (k / S) & 1, a.err);
        if (!ok) *s_bad = 1;
        const DevSeg tile = load_seg(a.segs, it / nO);
        if (ok && !*s_bad && tile.token_count == kPrefillTile) {
          tma_store_3d(&a.tmap_y128, 0, tile.token_start, ((it % nO) * kPfN) / kBoxCols, ring + stage * C::EX_STAGE);
          bulk_commit();
          bulk_wait_read();  // the store has read the stage
        }
        mbar_arrive(&empty[stage]);
        if (k < 16) pf_trace(a, 10 + 3 * k);
      }
      bulk_wait_all();
    }
    return;
  }

  // ============================ epilogue warps =============================
  // warp w reads TMEM lane quarter w % 4 (token rows 32 (w % 4) ..) and the
  // output columns [32 (w / 4), 32 (w / 4) + 32) of every item
  pdl_wait_prior();  // the shrink kernel's partials are complete and visible
  pdl_launch_dependents();
  if (tid == 0) pf_trace(a, 1);
  const int quarter = warp & 3, hf = warp >> 2;
  const int t = quarter * 32 + lane;  // token row of the tile = TMEM lane
  constexpr int RH = R / 2;  // ranks of H this thread builds
  T* yg = static_cast<T*>(a.y);
  int cur = -1, ti = -1;
  DevSeg tile{};
  for (int it = i0, k = 0; it < i1; ++it, ++k) {
    if (it / nO != cur) {
      cur = it / nO;
      ++ti;
      tile = load_seg(a.segs, cur);
      if (tid == 0 && ti == 0) pf_trace(a, 4);
      if (ti > 0 && !*s_bad && !mbar_wait_bounded(h_free, (ti - 1) & 1, a.err)) *s_bad = 1;
      // ---- H row t, ranks [hf * R/2, (hf + 1) * R/2): the nKC partials in
      // chunk order (four chunks' loads in flight at a time), times alpha,
      // rounded to the weights' 16-bit type, in the 2R-byte-row swizzle
      float h[RH];
#pragma unroll
      for (int r = 0; r < RH; ++r) h[r] = 0.f;
      if (t < tile.token_count) {
        const float4* p = reinterpret_cast<const float4*>(a.part + static_cast<int64_t>(tile.token_start + t) * nKC * R +
                                                          hf * RH);
        for (int kc0 = 0; kc0 < nKC; kc0 += 4) {
          float4 v[4][RH / 4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < RH / 4; ++q)
              v[j][q] = kc0 + j < nKC ? __ldcg(p + (kc0 + j) * (R / 4) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < RH / 4; ++q) {
              h[4 * q] += v[j][q].x;
              h[4 * q + 1] += v[j][q].y;
              h[4 * q + 2] += v[j][q].z;
              h[4 * q + 3] += v[j][q].w;
            }
        }
      }
      if (tid == 0 && ti == 0) pf_trace(a, 5);
#pragma unroll
      for (int q = 0; q < RH / 8; ++q) {  // 16-byte chunks of the row
        uint4 w;
        w.x = E::pack2(h[8 * q] * a.scale, h[8 * q + 1] * a.scale);
        w.y = E::pack2(h[8 * q + 2] * a.scale, h[8 * q + 3] * a.scale);
        w.z = E::pack2(h[8 * q + 4] * a.scale, h[8 * q + 5] * a.scale);
        w.w = E::pack2(h[8 * q + 6] * a.scale, h[8 * q + 7] * a.scale);
        uint32_t lin = static_cast<uint32_t>(t * (2 * R) + (hf * (RH / 8) + q) * 16);
        lin ^= (lin >> 3) & C::SWZ_MASK;
        *reinterpret_cast<uint4*>(Ht + lin) = w;
      }
      fence_proxy_async_smem();  // the tensor core reads these writes
      if (tid == 0 && ti == 0) pf_trace(a, 6);
      named_sync(kPfBar, kPfExEpi * 32);
      if (tid == 0) {
        mbar_arrive(h_full);
        if (ti == 0) pf_trace(a, 2);
      }
    }
    const int b = k % kPfAcc;
    const int stage = k % S;
    const bool ok = mbar_wait_bounded(&acc_full[b], (k / kPfAcc) & 1, a.err) &&
                    mbar_wait_bounded(&full[stage], (k / S) & 1, a.err);  // the y tile landed
    if (!ok) *s_bad = 1;
    if (tid == 0 && k < 16) pf_trace(a, 8 + 3 * k);
    tc_fence_after();
    const int oc = (it % nO) * kPfN;
    const int wc = min(kPfN, a.o - oc);
    const bool row_ok = ok && !*s_bad && t < tile.token_count;
    const bool full_tile = tile.token_count == kPrefillTile;  // the store thread writes the tile back
    T* yrow = yg + static_cast<int64_t>(tile.token_start + t) * a.y_ld + a.y_off + oc;
    uint8_t* yrow_s = ring + stage * C::EX_STAGE + t * 128;  // y tile row t: 128 B, 128-byte swizzle
    const uint32_t taddr = tbase + b * kPfN + 32 * hf + (static_cast<uint32_t>(quarter * 32) << 16);
    // this warp's 32 columns: y + D, rounded once, back into the y tile (full
    // tiles) or straight to y (partial tiles)
    uint32_t r[32];
    tmem_ld32_nowait(taddr, r);
    tmem_wait_ld();
    if (row_ok) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int col = hf * 32 + g * 8;
        if (col < wc) {
          const int chunk = hf * 4 + g;  // 16-byte chunk of the 128-byte row
          uint4* ps = reinterpret_cast<uint4*>(yrow_s + (((chunk ^ t) & 7) << 4));
          uint4 yv = *ps;
          uint32_t* yw = reinterpret_cast<uint32_t*>(&yv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = E::unpack2(yw[e]);
            yw[e] = E::pack2(f.x + __uint_as_float(r[g * 8 + 2 * e]), f.y + __uint_as_float(r[g * 8 + 2 * e + 1]));
          }
          if (full_tile)
            *ps = yv;
          else
            *reinterpret_cast<uint4*>(yrow + col) = yv;
        }
      }
    }
    tc_fence_before();
    fence_proxy_async_smem();  // the tensor store reads the y tile through the async proxy
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&acc_free[b]);
      mbar_arrive(&ydone[stage]);  // this warp's part of the stage is final
    }
    if (tid == 0 && k < 16) pf_trace(a, 9 + 3 * k);
  }
  tc_fence_before();
  named_sync(kPfBar, kPfExEpi * 32);  // every TMEM read of this CTA is done
  if (tid == 0) pf_trace(a, 3);
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, kPfAcc * kPfN);
  }
}

template <typename T, int R>
struct PrefillKernels {
  static bool prepare() {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load() & bit) return true;
    using C = PfCfg<R>;
    if (cudaFuncSetAttribute(prefill_shrink_kernel<T, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SH_SMEM) !=
            cudaSuccess ||
        cudaFuncSetAttribute(prefill_expand_kernel<T, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::EX_SMEM) !=
            cudaSuccess)
      return false;
    done.fetch_or(bit);
    return true;
  }
  static cudaError_t launch(const ApplyArgs& a, const LaunchCfg& lc) {
    if (!prepare()) return cudaGetLastError();
    using C = PfCfg<R>;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(lc.grid);
    cfg.blockDim = dim3(kPfThreads);
    cfg.stream = lc.stream;
    cfg.attrs = attr;
    cfg.numAttrs = lc.pdl ? 1 : 0;
    cfg.dynamicSmemBytes = C::SH_SMEM;
    cudaError_t e = cudaLaunchKernelEx(&cfg, prefill_shrink_kernel<T, R>, a);
    if (e != cudaSuccess) return e;
    cfg.dynamicSmemBytes = C::EX_SMEM;
    cfg.blockDim = dim3(kPfExThreads);
    return cudaLaunchKernelEx(&cfg, prefill_expand_kernel<T, R>, a);
  }
};

template <typename T>
cudaError_t prefill_by_rank(int rank, const ApplyArgs& a, const LaunchCfg& lc) {
  switch (rank) {
    case 16: return PrefillKernels<T, 16>::launch(a, lc);
    case 32: return PrefillKernels<T, 32>::launch(a, lc);
    case 64: return PrefillKernels<T, 64>::launch(a, lc);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_prefill(int dtype, int rank, const ApplyArgs& a, const LaunchCfg& lc) {
  return dtype == 1 ? prefill_by_rank<__nv_bfloat16>(rank, a, lc) : prefill_by_rank<__half>(rank, a, lc);
}

}  // namespace wp
