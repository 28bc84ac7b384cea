// wp_kernel_common.cuh -- device-side helpers shared by the apply kernels:
// segment descriptors, x / y box sizing and the optional per-CTA phase trace.
#pragma once

#include <stdint.h>

#include "wp_device.cuh"
#include "wp_internal.h"

namespace wp {

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
__device__ __forceinline__ void trace_mark(unsigned long long* base, int k) {
  if (base) base[blockIdx.x * kTraceSlots + 8 + k] = global_timer_ns();
}
// Mark k (6 or 7) of stage-unit u, written by the MMA or producer warp.
__device__ __forceinline__ void trace_unit(unsigned long long* base, int u, int k) {
  if (base && u >= 0 && u < kTraceUnits)
    base[blockIdx.x * kTraceSlots + 8 + kTraceSegMarks + kTraceMarks * u + k] = global_timer_ns();
}

// Tracing is a compile-time variant of the kernels: the production
// instantiations carry none of it (its code alone slowed a launch by ~12 %,
// even when switched off at run time).
template <bool TR>
__device__ __forceinline__ void trace_mark_t(unsigned long long* base, int k) {
  if constexpr (TR) trace_mark(base, k);
}
template <bool TR>
__device__ __forceinline__ void trace_unit_t(unsigned long long* base, int u, int k) {
  if constexpr (TR) trace_unit(base, u, k);
}

// The same marks into a per-CTA record (a shared-memory staging copy).
template <bool TR>
__device__ __forceinline__ void trace_rec_mark(unsigned long long* rec, int k) {
  if constexpr (TR)
    if (rec) rec[8 + k] = global_timer_ns();
}
template <bool TR>
__device__ __forceinline__ void trace_rec_unit(unsigned long long* rec, int u, int k) {
  if constexpr (TR)
    if (rec && u >= 0 && u < kTraceUnits) rec[8 + kTraceSegMarks + kTraceMarks * u + k] = global_timer_ns();
}

struct TraceOff {
  __device__ void init(unsigned long long*, bool) {}
  __device__ void stage(unsigned long long*) {}
  __device__ void dep() {}
  __device__ unsigned long long before_wait() { return 0ull; }
  __device__ void after_wait(unsigned long long) {}
  __device__ void mark(int) {}
  __device__ void seg(int, int) {}
  __device__ void finish() {}
};

struct Trace {
  unsigned long long* rec = nullptr;
  unsigned long long* grec = nullptr;  // global record when `rec` is a shared-memory staging copy
  unsigned long long t_start = 0, t_dep = 0, t_first = 0, waited = 0, units = 0;
  __device__ void init(unsigned long long* base, bool me) {
    if (base && me) {
      rec = base + blockIdx.x * kTraceSlots;
      t_start = global_timer_ns();
    }
  }
  // Marks go to `srec` (kTraceSlots zeroed values in shared memory) from now
  // on and are copied to the global record by finish(): a global store per
  // mark would make the fences that follow marks wait for it.
  __device__ void stage(unsigned long long* srec) {
    if (rec) {
      grec = rec;
      rec = srec;
    }
  }
  __device__ void dep() {
    if (rec) t_dep = global_timer_ns();
  }
  __device__ unsigned long long before_wait() {
    if (!rec) return 0ull;
    const unsigned long long t = global_timer_ns();
    if (units < kTraceUnits) rec[8 + kTraceSegMarks + kTraceMarks * units] = t;
    return t;
  }
  __device__ void after_wait(unsigned long long t0) {
    if (rec) {
      const unsigned long long t = global_timer_ns();
      if (!t_first) t_first = t;
      waited += t - t0;
      if (units < kTraceUnits) rec[8 + kTraceSegMarks + kTraceMarks * units + 1] = t;
      ++units;
    }
  }
  __device__ void mark(int k) {  // k = 2..5: phase marks of the latest stage
    if (rec && units >= 1 && units <= kTraceUnits) rec[8 + kTraceSegMarks + kTraceMarks * (units - 1) + k] = global_timer_ns();
  }
  __device__ void seg(int k, int sj) {  // marks of the first segment
    if (rec && sj == 0) rec[8 + k] = global_timer_ns();
  }
  __device__ void finish() {
    if (rec) {
      rec[0] = t_start;
      rec[1] = t_dep;
      rec[2] = t_first;
      rec[3] = global_timer_ns();
      rec[4] = units;
      rec[5] = waited;
      if (grec) {
        __threadfence_block();
        for (int i = 0; i < kTraceSlots; ++i) grec[i] = static_cast<volatile unsigned long long*>(rec)[i];
      }
    }
  }
};


}  // namespace wp
