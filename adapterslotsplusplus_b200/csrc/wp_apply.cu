// wp_apply.cu -- grouped multi-LoRA shrink and expand kernels for sm_100a.
//
// Semantics (reference: tests/correctness/reference_bgmv.py:4-18, the math of
// bgmv_shrink_kernel / bgmv_expand_kernel in csrc/kernels/warp_pipe_r32.cu:56-200
// and their DSAK twins :280-423):
//   shrink:  H[t, :] = alpha * X[t, :] . A_seg^T      (fp32 result)
//   expand:  Y[t, j] = round(Y[t, j] + H[t, :] . B_seg[j, :])
// for every token t inside a segment of the table; other rows are untouched.
//
// Both kernels are persistent (one CTA per SM, a grid fixed at launch so the
// launch can be captured in a CUDA graph) and read the segment count from
// device memory. Work items are strided over the grid; CTAs without an item
// exit after the programmatic-dependency wait.
//
// Data movement: the adapter weights (the dominant HBM traffic) and the
// activation rows are streamed into a ring of shared-memory stages by the TMA
// unit's 1-D bulk copies (cp.async.bulk) completing on per-stage mbarriers,
// so several stages of loads are always in flight per SM. Every smem row is
// padded by 16 bytes, which makes the warp-level fragment loads below free of
// bank conflicts.
//
// Math: mma.sync m16n8k16 (bf16/fp16 in, fp32 accumulate). The segment tiles
// of a decode step are 1..32 tokens, far below the 64/128-row tiles of the
// tcgen05 unit; the tensor pipe is <5% busy here and the kernels are bound by
// HBM bandwidth.
//
// shrink: item = (segment, split of d). A CTA streams A[:, split] and the
//   segment's X rows through the stages in KC-wide chunks, accumulating a
//   [<=32 x R] tile in registers. With more than one split, each item stores
//   its partial tile and the last-arriving CTA of the segment (per-segment
//   arrival counter) sums the partials in split order and writes H -- a
//   deterministic split-K reduction with no memset and no float atomics. The
//   last CTA resets the counter to zero for the next call.
// expand: item = (segment, W-column chunk of o). The stage holds the B rows of
//   the chunk (one contiguous bulk copy), the segment's H rows (one copy) and
//   the segment's Y tile (one copy per row). H enters the MMA split into a
//   16-bit high part and a 16-bit residual, so the product keeps ~16 mantissa
//   bits of the fp32 H; Y is rounded once.
//
// Programmatic dependent launch: every kernel waits on its predecessor
// (griddepcontrol.wait) before it triggers its own dependents, so a kernel's
// pre-wait prologue overlaps only the immediately preceding kernel. expand
// prefetches B and Y (never written by shrink) before the wait, H after it.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "wp_device.cuh"
#include "wp_internal.h"

namespace wp {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kHeaderBytes = 1024;  // mbarriers + flags

// --------------------------------------------------------------------------
// shrink

template <int R>
struct ShrinkCfg {
  static constexpr int KC = 128;  // K elements per stage
  static constexpr int PITCH = KC * 2 + 16;  // smem row pitch (bytes)
  static constexpr int ROWS = R + kSegTokens;
  static constexpr int STAGE = ROWS * PITCH;
  static constexpr int STAGES = R == 64 ? 4 : 6;
  static constexpr int RED = kWarps * 8 * 32 * 4;  // cross-warp reduction
  static constexpr int SMEM = kHeaderBytes + RED + STAGES * STAGE;
};

struct Cursor {
  int item, chunk, nch, idx;
};

__device__ __forceinline__ int shrink_nchunks(int item, int nsplit, int split_len, int d, int kc) {
  const int split = item % nsplit;
  const int k0 = split * split_len;
  const int len = min(split_len, d - k0);
  return (len + kc - 1) / kc;
}

__device__ __forceinline__ DevSeg load_seg(const DevSeg* segs, int i) {
  DevSeg s;
  const int4* p = reinterpret_cast<const int4*>(segs + i);
  int4 v0 = __ldcg(p);
  int4 v1 = __ldcg(p + 1);
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

// Token count clamped to [0, 32]; out-of-range entries raise kErrBadSegment.
__device__ __forceinline__ int seg_rows(const DevSeg& s, int* err) {
  int n = s.token_count;
  if (n < 1 || n > kSegTokens) {
    if (threadIdx.x == 0 && err) atomicOr(err, kErrBadSegment);
    n = 0;
  }
  return n;
}

template <typename T, int R>
__global__ void __launch_bounds__(kThreads, 1) shrink_kernel(const ShrinkArgs a) {
  using C = ShrinkCfg<R>;
  constexpr int NT = R / 8;  // n-tiles of 8 rank columns
  constexpr int KP = kWarps / NT;  // warps sharing one n-tile (split over k-steps)
  constexpr int KC = C::KC;
  constexpr int PITCH = C::PITCH;

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  int* s_last = reinterpret_cast<int*>(smem + 512);
  float* red = reinterpret_cast<float*>(smem + kHeaderBytes);
  uint8_t* stage_base = smem + kHeaderBytes + C::RED;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = lane >> 2;
  const int c = lane & 3;
  const int nt = warp % NT;
  const int kp = warp / NT;

  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // X and the workspaces may be written by the previous kernel: wait first.
  pdl_wait_prior();
  pdl_launch_dependents();

  const int nseg = __ldcg(a.num_segs);
  const int nitems = nseg * a.nsplit;
  if (static_cast<int>(blockIdx.x) >= nitems) return;

  const T* xg = static_cast<const T*>(a.x);
  const int d = a.d;

  auto advance = [&](Cursor& q) {
    ++q.idx;
    if (++q.chunk == q.nch) {
      q.item += gridDim.x;
      q.chunk = 0;
      q.nch = q.item < nitems ? shrink_nchunks(q.item, a.nsplit, a.split_len, d, KC) : 0;
    }
  };

  // Issue the bulk copies of one (item, chunk) unit into `stage` (warp 0).
  auto issue = [&](const Cursor& q, int stage) {
    const int split = q.item % a.nsplit;
    const DevSeg s = load_seg(a.segs, q.item / a.nsplit);
    int n = s.token_count;
    if (n < 1 || n > kSegTokens) n = 0;
    const int k0 = split * a.split_len + q.chunk * KC;
    const int kend = min(d, split * a.split_len + a.split_len);
    const int kc = min(KC, kend - k0);
    const T* A = a.registry ? static_cast<const T*>(s.a)
                            : static_cast<const T*>(a.wa_base) + static_cast<int64_t>(s.adapter_id) * a.wa_stride;
    const uint32_t row_bytes = static_cast<uint32_t>(kc) * 2u;
    uint8_t* st = stage_base + stage * C::STAGE;
    if (lane == 0) mbar_arrive_expect_tx(&full[stage], (R + n) * row_bytes);
    __syncwarp();
    for (int row = lane; row < R + n; row += 32) {
      const T* src = row < R ? A + static_cast<int64_t>(row) * d + k0
                             : xg + static_cast<int64_t>(s.token_start + row - R) * a.x_ld + k0;
      bulk_g2s(st + row * PITCH, src, row_bytes, &full[stage]);
    }
  };

  Cursor p{static_cast<int>(blockIdx.x), 0, shrink_nchunks(blockIdx.x, a.nsplit, a.split_len, d, KC), 0};
  Cursor q = p;
  for (int s = 0; s < C::STAGES && p.item < nitems; ++s) {
    if (warp == 0) issue(p, s);
    advance(p);
  }

  float acc[2][4];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[m][j] = 0.f;

  while (q.item < nitems) {
    const int stage = q.idx % C::STAGES;
    const uint32_t parity = (q.idx / C::STAGES) & 1;
    const bool ok = mbar_wait_bounded(&full[stage], parity, a.err);
    if (__syncthreads_or(!ok)) return;  // uniform bail-out after a timeout

    const int split = q.item % a.nsplit;
    const int segi = q.item / a.nsplit;
    const DevSeg s = load_seg(a.segs, segi);
    const int n = seg_rows(s, a.err);
    const int k0 = split * a.split_len + q.chunk * KC;
    const int kend = min(d, split * a.split_len + a.split_len);
    const int kc = min(KC, kend - k0);

    if (n > 0) {
      const uint8_t* As = stage_base + stage * C::STAGE;
      const uint8_t* Xs = As + R * PITCH;
      const uint8_t* brow = As + (nt * 8 + g) * PITCH + c * 4;
      const uint8_t* xr0 = Xs + g * PITCH + c * 4;
      const bool m1 = n > 16;
      const int ks_full = kc >> 4;
      for (int ks = kp; ks < ks_full; ks += KP) {
        const int kb = ks * 32;
        const uint32_t b0 = lds32(brow + kb);
        const uint32_t b1 = lds32(brow + kb + 16);
        uint32_t af[4];
        af[0] = lds32(xr0 + kb);
        af[1] = lds32(xr0 + 8 * PITCH + kb);
        af[2] = lds32(xr0 + kb + 16);
        af[3] = lds32(xr0 + 8 * PITCH + kb + 16);
        mma_k16<T>(acc[0], af, b0, b1);
        if (m1) {
          af[0] = lds32(xr0 + 16 * PITCH + kb);
          af[1] = lds32(xr0 + 24 * PITCH + kb);
          af[2] = lds32(xr0 + 16 * PITCH + kb + 16);
          af[3] = lds32(xr0 + 24 * PITCH + kb + 16);
          mma_k16<T>(acc[1], af, b0, b1);
        }
      }
      if ((kc & 15) && (ks_full % KP) == kp) {  // 8-wide K tail
        const int kb = ks_full * 32;
        const uint32_t b0 = lds32(brow + kb);
        mma_k8<T>(acc[0], lds32(xr0 + kb), lds32(xr0 + 8 * PITCH + kb), b0);
        if (m1) mma_k8<T>(acc[1], lds32(xr0 + 16 * PITCH + kb), lds32(xr0 + 24 * PITCH + kb), b0);
      }
    }

    if (q.chunk == q.nch - 1) {
      // ---- end of item: combine the KP warps of each n-tile -------------
      if constexpr (KP > 1) {
        float* mine = red + warp * 8 * 32;
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int j = 0; j < 4; ++j) mine[(m * 4 + j) * 32 + lane] = acc[m][j];
        __syncthreads();
        if (kp == 0) {
#pragma unroll
          for (int w2 = 1; w2 < KP; ++w2) {
            const float* other = red + (nt + w2 * NT) * 8 * 32;
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
              for (int j = 0; j < 4; ++j) acc[m][j] += other[(m * 4 + j) * 32 + lane];
          }
        }
      }
      const float alpha = a.registry ? s.alpha : a.scale;
      if (kp == 0 && n > 0) {
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int row = m * 16 + g + hf * 8;
            if (row < n) {
              const int col = nt * 8 + 2 * c;
              const int64_t t = s.token_start + row;
              if (a.nsplit == 1) {
                *reinterpret_cast<float2*>(a.h + t * R + col) =
                    make_float2(acc[m][hf * 2] * alpha, acc[m][hf * 2 + 1] * alpha);
              } else {
                *reinterpret_cast<float2*>(a.partial + (static_cast<int64_t>(split) * a.cap_t + t) * R + col) =
                    make_float2(acc[m][hf * 2], acc[m][hf * 2 + 1]);
              }
            }
          }
      }
      if (a.nsplit > 1) {
        __threadfence();
        __syncthreads();
        if (tid == 0) {
          const uint32_t prev = atomicAdd(&a.counters[segi], 1u);
          *s_last = (prev == static_cast<uint32_t>(a.nsplit - 1));
        }
        __syncthreads();
        if (*s_last) {
          __threadfence();
          for (int e = tid; e < n * R; e += kThreads) {
            const int64_t t = s.token_start + e / R;
            const int col = e % R;
            float sum = 0.f;
            for (int sp = 0; sp < a.nsplit; ++sp) sum += __ldcg(a.partial + (static_cast<int64_t>(sp) * a.cap_t + t) * R + col);
            a.h[t * R + col] = sum * alpha;
          }
          if (tid == 0) a.counters[segi] = 0u;
        }
      }
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[m][j] = 0.f;
    }

    __syncthreads();  // every warp is done with `stage`
    if (p.item < nitems) {
      if (warp == 0) issue(p, stage);
      advance(p);
    }
    advance(q);
  }
}

// --------------------------------------------------------------------------
// expand

template <int R>
struct ExpandCfg {
  static constexpr int W = 128;  // output columns per item
  static constexpr int BBYTES = W * R * 2;
  static constexpr int YPITCH = W * 2 + 16;
  static constexpr int YBYTES = kSegTokens * YPITCH;
  static constexpr int HBYTES = kSegTokens * R * 4;
  static constexpr int STAGE = BBYTES + YBYTES + HBYTES;
  static constexpr int STAGES = R == 64 ? 3 : (R == 32 ? 5 : (R == 16 ? 6 : 8));
  static constexpr int SMEM = kHeaderBytes + STAGES * STAGE;
};

template <typename T, int R>
__global__ void __launch_bounds__(kThreads, 1) expand_kernel(const ExpandArgs a) {
  using C = ExpandCfg<R>;
  using E = Elem<T>;
  constexpr int W = C::W;
  constexpr int NTW = W / 8 / kWarps;  // n-tiles per warp
  constexpr int YPITCH = C::YPITCH;

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint8_t* stage_base = smem + kHeaderBytes;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = lane >> 2;
  const int c = lane & 3;

  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // The segment table, B and Y are not written by the preceding shrink, so
  // they are prefetched before the dependency wait; H is loaded after it.
  const int nseg = __ldcg(a.num_segs);
  const int nitems = nseg * a.n_ochunks;
  const bool has_work = static_cast<int>(blockIdx.x) < nitems;
  T* yg = static_cast<T*>(a.y);

  auto issue = [&](int item, int stage, int parts) {
    const DevSeg s = load_seg(a.segs, item / a.n_ochunks);
    int n = s.token_count;
    if (n < 1 || n > kSegTokens) n = 0;
    const int o0 = (item % a.n_ochunks) * W;
    const int wc = min(W, a.o - o0);
    uint8_t* st = stage_base + stage * C::STAGE;
    if (parts & 1) {
      const T* B = a.registry ? static_cast<const T*>(s.b)
                              : static_cast<const T*>(a.wb_base) + static_cast<int64_t>(s.adapter_id) * a.wb_stride;
      const uint32_t ybytes = a.y_bulk ? static_cast<uint32_t>(n * wc * 2) : 0u;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(wc * R * 2) + ybytes + n * R * 4);
        bulk_g2s(st, B + static_cast<int64_t>(o0) * R, wc * R * 2, &full[stage]);
      }
      __syncwarp();
      if (a.y_bulk) {
        for (int row = lane; row < n; row += 32)
          bulk_g2s(st + C::BBYTES + row * YPITCH, yg + (s.token_start + row) * a.y_ld + a.y_off + o0, wc * 2,
                   &full[stage]);
      }
    }
    if ((parts & 2) && lane == 0 && n > 0)
      bulk_g2s(st + C::BBYTES + C::YBYTES, a.h + static_cast<int64_t>(s.token_start) * R, n * R * 4, &full[stage]);
  };

  int issued = 0;
  if (has_work && warp == 0) {
    for (int it = blockIdx.x, s = 0; s < C::STAGES && it < nitems; ++s, it += gridDim.x) issue(it, s, 1);
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  if (!has_work) return;
  for (int it = blockIdx.x, s = 0; s < C::STAGES && it < nitems; ++s, it += gridDim.x) {
    if (warp == 0) issue(it, s, 2);
    ++issued;
  }
  int next_item = blockIdx.x + issued * gridDim.x;

  int k = 0;
  for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++k) {
    const int stage = k % C::STAGES;
    const uint32_t parity = (k / C::STAGES) & 1;
    const bool ok = mbar_wait_bounded(&full[stage], parity, a.err);
    if (__syncthreads_or(!ok)) return;

    const DevSeg s = load_seg(a.segs, item / a.n_ochunks);
    const int n = seg_rows(s, a.err);
    const int o0 = (item % a.n_ochunks) * W;
    const int wc = min(W, a.o - o0);
    const uint8_t* Bs = stage_base + stage * C::STAGE;
    const uint8_t* Ys = Bs + C::BBYTES;
    const float* Hs = reinterpret_cast<const float*>(Bs + C::BBYTES + C::YBYTES);

    float acc[2][NTW][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int j = 0; j < NTW; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[m][j][e] = 0.f;

    for (int m = 0; m < 2; ++m) {
      if (m * 16 >= n) break;
      const float* h0 = Hs + (m * 16 + g) * R;
      const float* h1 = h0 + 8 * R;
      if constexpr (R == 8) {
        const float2 x0 = *reinterpret_cast<const float2*>(h0 + 2 * c);
        const float2 x1 = *reinterpret_cast<const float2*>(h1 + 2 * c);
        const uint32_t hi0 = E::pack2(x0.x, x0.y), hi1 = E::pack2(x1.x, x1.y);
        const float2 r0 = E::unpack2(hi0), r1 = E::unpack2(hi1);
        const uint32_t lo0 = E::pack2(x0.x - r0.x, x0.y - r0.y), lo1 = E::pack2(x1.x - r1.x, x1.y - r1.y);
#pragma unroll
        for (int j = 0; j < NTW; ++j) {
          const int nt = warp * NTW + j;
          if (nt * 8 < wc) {
            const uint32_t b0 = lds32(Bs + (nt * 8 + g) * (R * 2) + c * 4);
            mma_k8<T>(acc[m][j], hi0, hi1, b0);
            mma_k8<T>(acc[m][j], lo0, lo1, b0);
          }
        }
      } else {
#pragma unroll
        for (int ks = 0; ks < R / 16; ++ks) {
          const int k0 = ks * 16 + 2 * c;
          const float2 x00 = *reinterpret_cast<const float2*>(h0 + k0);
          const float2 x10 = *reinterpret_cast<const float2*>(h1 + k0);
          const float2 x01 = *reinterpret_cast<const float2*>(h0 + k0 + 8);
          const float2 x11 = *reinterpret_cast<const float2*>(h1 + k0 + 8);
          uint32_t hi[4], lo[4];
          hi[0] = E::pack2(x00.x, x00.y);
          hi[1] = E::pack2(x10.x, x10.y);
          hi[2] = E::pack2(x01.x, x01.y);
          hi[3] = E::pack2(x11.x, x11.y);
          {
            const float2 r0 = E::unpack2(hi[0]), r1 = E::unpack2(hi[1]), r2 = E::unpack2(hi[2]),
                         r3 = E::unpack2(hi[3]);
            lo[0] = E::pack2(x00.x - r0.x, x00.y - r0.y);
            lo[1] = E::pack2(x10.x - r1.x, x10.y - r1.y);
            lo[2] = E::pack2(x01.x - r2.x, x01.y - r2.y);
            lo[3] = E::pack2(x11.x - r3.x, x11.y - r3.y);
          }
#pragma unroll
          for (int j = 0; j < NTW; ++j) {
            const int nt = warp * NTW + j;
            if (nt * 8 < wc) {
              const uint8_t* brow = Bs + (nt * 8 + g) * (R * 2) + ks * 32 + c * 4;
              const uint32_t b0 = lds32(brow);
              const uint32_t b1 = lds32(brow + 16);
              mma_k16<T>(acc[m][j], hi, b0, b1);
              mma_k16<T>(acc[m][j], lo, b0, b1);
            }
          }
        }
      }
    }

    // ---- epilogue: Y += acc, one rounding ---------------------------------
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int j = 0; j < NTW; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int row = m * 16 + g + hf * 8;
          const int col = (warp * NTW + j) * 8 + 2 * c;
          if (row < n && col < wc) {
            T* yp = yg + (s.token_start + row) * a.y_ld + a.y_off + o0 + col;
            const float v0 = acc[m][j][hf * 2], v1 = acc[m][j][hf * 2 + 1];
            if (a.y_bulk) {
              const float2 yv = E::unpack2(lds32(Ys + row * YPITCH + col * 2));
              *reinterpret_cast<uint32_t*>(yp) = E::pack2(yv.x + v0, yv.y + v1);
            } else {
              yp[0] = E::from_f(E::to_f(yp[0]) + v0);
              yp[1] = E::from_f(E::to_f(yp[1]) + v1);
            }
          }
        }

    __syncthreads();  // stage consumed by every warp
    if (next_item < nitems) {
      if (warp == 0) issue(next_item, stage, 3);
      next_item += gridDim.x;
    }
  }
}

// --------------------------------------------------------------------------
// launchers

namespace {

template <typename K>
bool ensure_smem_attr(K kernel, int bytes, std::atomic<uint64_t>& done_mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load() & bit) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  done_mask.fetch_or(bit);
  return true;
}

template <typename K, typename Args>
cudaError_t launch_persistent(K kernel, const Args& args, int smem, const LaunchCfg& lc) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(lc.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = lc.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lc.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args);
}

template <typename T, int R>
cudaError_t launch_shrink_t(const ShrinkArgs& a, const LaunchCfg& lc) {
  static std::atomic<uint64_t> mask{0};
  constexpr int smem = ShrinkCfg<R>::SMEM;
  if (!ensure_smem_attr(shrink_kernel<T, R>, smem, mask)) return cudaGetLastError();
  return launch_persistent(shrink_kernel<T, R>, a, smem, lc);
}

template <typename T, int R>
cudaError_t launch_expand_t(const ExpandArgs& a, const LaunchCfg& lc) {
  static std::atomic<uint64_t> mask{0};
  constexpr int smem = ExpandCfg<R>::SMEM;
  if (!ensure_smem_attr(expand_kernel<T, R>, smem, mask)) return cudaGetLastError();
  return launch_persistent(expand_kernel<T, R>, a, smem, lc);
}

template <typename T>
cudaError_t shrink_by_rank(int rank, const ShrinkArgs& a, const LaunchCfg& lc) {
  switch (rank) {
    case 8: return launch_shrink_t<T, 8>(a, lc);
    case 16: return launch_shrink_t<T, 16>(a, lc);
    case 32: return launch_shrink_t<T, 32>(a, lc);
    case 64: return launch_shrink_t<T, 64>(a, lc);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t expand_by_rank(int rank, const ExpandArgs& a, const LaunchCfg& lc) {
  switch (rank) {
    case 8: return launch_expand_t<T, 8>(a, lc);
    case 16: return launch_expand_t<T, 16>(a, lc);
    case 32: return launch_expand_t<T, 32>(a, lc);
    case 64: return launch_expand_t<T, 64>(a, lc);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int expand_chunk_cols(int) { return ExpandCfg<32>::W; }
int shrink_chunk_k(int) { return ShrinkCfg<32>::KC; }

cudaError_t launch_shrink(int dtype, int rank, const ShrinkArgs& a, const LaunchCfg& lc) {
  return dtype == 1 ? shrink_by_rank<__nv_bfloat16>(rank, a, lc) : shrink_by_rank<__half>(rank, a, lc);
}

cudaError_t launch_expand(int dtype, int rank, const ExpandArgs& a, const LaunchCfg& lc) {
  return dtype == 1 ? expand_by_rank<__nv_bfloat16>(rank, a, lc) : expand_by_rank<__half>(rank, a, lc);
}

}  // namespace wp
