"""TEST INFRASTRUCTURE ONLY -- numpy restatement of the segment-table builders.

seg_bounds: build_seg_bounds_kernel (csrc/kernels/warp_pipe_r32.cu:461-512)
  - a run starts at i == 0 or where idx[i] != idx[i-1]  (:476-478)
  - runs with idx < 0 contribute nothing                  (:478)
  - a run of length L becomes ceil(L/32) pieces (:480-481) with
    token_start = start + 32*s, token_count = min(32, L - 32*s)  (:505-511)
  - slots follow token order (exclusive prefix sum, :485-495)
  - num_segments = total pieces (:497)
  The reference processes at most WP_MAX_SEGMENTS = 256 tokens
  (warp_pipe_bindings.cpp:166 returns False above it); this restatement has
  no cap.

segment_table: build_segment_table (csrc/dispatch/segment_builder.cpp:5-50)
  - K entries (adapter_id, offsets[i], offsets[i+1]-offsets[i]), unsplit;
    raises on len(offsets) != K+1 (:9-11).
"""

from __future__ import annotations

import numpy as np

SEG_TOKENS = 32  # WP_MAX_SEGMENT_TOKENS, csrc/bridge/warp_pipe_metadata.h:22


def seg_bounds(idx) -> np.ndarray:
    """int64[T] token -> adapter ids  ->  int32[n, 3] (adapter_id, token_start, token_count)."""
    idx = np.asarray(idx, dtype=np.int64).reshape(-1)
    T = idx.size
    if T == 0:
        return np.zeros((0, 3), dtype=np.int32)
    start = np.ones(T, dtype=bool)
    start[1:] = idx[1:] != idx[:-1]
    starts = np.flatnonzero(start)
    ends = np.append(starts[1:], T)
    ids = idx[starts]
    keep = ids >= 0
    starts, ends, ids = starts[keep], ends[keep], ids[keep]
    lengths = ends - starts
    pieces = (lengths + SEG_TOKENS - 1) // SEG_TOKENS
    total = int(pieces.sum())
    out = np.empty((total, 3), dtype=np.int32)
    run_of_piece = np.repeat(np.arange(starts.size), pieces)
    first_piece = np.cumsum(pieces) - pieces
    j = np.arange(total) - first_piece[run_of_piece]
    out[:, 0] = ids[run_of_piece].astype(np.int32)
    out[:, 1] = starts[run_of_piece] + SEG_TOKENS * j
    out[:, 2] = np.minimum(SEG_TOKENS, lengths[run_of_piece] - SEG_TOKENS * j)
    return out


def seg_bounds_loop(idx) -> np.ndarray:
    """Pure-Python loop form of seg_bounds for small cases (cross-check)."""
    idx = [int(v) for v in np.asarray(idx).reshape(-1)]
    out = []
    i = 0
    while i < len(idx):
        j = i + 1
        while j < len(idx) and idx[j] == idx[i]:
            j += 1
        if idx[i] >= 0:
            s = i
            while s < j:
                n = min(SEG_TOKENS, j - s)
                out.append((idx[i], s, n))
                s += n
        i = j
    return np.asarray(out, dtype=np.int32).reshape(-1, 3)


def segment_table(sorted_adapter_ids, seg_offsets) -> np.ndarray:
    K = len(sorted_adapter_ids)
    if len(seg_offsets) != K + 1:
        raise RuntimeError("build_segment_table: seg_offsets must have K+1 entries")
    out = np.empty((K, 3), dtype=np.int32)
    for i in range(K):
        out[i] = (sorted_adapter_ids[i], seg_offsets[i], seg_offsets[i + 1] - seg_offsets[i])
    return out
