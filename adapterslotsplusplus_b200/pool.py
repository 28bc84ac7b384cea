"""Adapter pool: the live grouped apply over a pinned-host adapter store.

The reference keeps host-store adapters for its registry path only
(StagingBufferPool, csrc/memory/staging_buffer.h:29-105, fed by
WarpPipeExtension::prefetch_adapter, csrc/pybind/warp_pipe_bindings.cpp:46-64);
its live add_lora_packed path reads device stacks (warp_pipe_r32.cu:263-269).
AdapterPool pages a whole tenant adapter -- its A/B for every LoRA projection
of the model -- from page-locked host memory into one of `num_slots` GPU
slots (libwp_b200.so's wp_pool_*). The slots of projection p form the stacked
tensors add_lora_packed takes, so the apply kernels run unchanged; the step's
segment table carries slot numbers (build_seg_bounds_pool).

One step:

    pool.prepare(active_ids)            # cold adapters copied now, stream waits
    pool.build_seg_bounds(token_ids)    # table in slot numbers
    for p, (y, x) in enumerate(calls):  # one call per projection
        pool.add_lora(p, y, x, scale)

Prefetching (`prefetch`, `is_prefetch_ready`, `release_prefetch`, the
reference's staging-slot semantics) copies on the pool's own stream while the
current step runs; a slot is overwritten only after the kernels of the steps
that read it.
"""

from __future__ import annotations

import ctypes
from typing import List, Sequence

import torch

from . import _lib
from .engine import WarpPipeEngine, _DTYPES, _stream_ptr


class AdapterPool:
    def __init__(self, engine: WarpPipeEngine, num_slots: int, dims: Sequence[tuple], rank: int,
                 dtype=torch.bfloat16, max_adapters: int = 4096):
        """dims: (d_in, d_out) of every LoRA projection, in call order."""
        self.engine = engine
        self._lib = _lib.load()
        self.rank = int(rank)
        self.dtype = dtype
        self.dims = [(int(d), int(o)) for d, o in dims]
        self.num_slots = int(num_slots)
        self.max_adapters = int(max_adapters)
        n = len(self.dims)
        d_arr = (ctypes.c_int32 * n)(*[d for d, _ in self.dims])
        o_arr = (ctypes.c_int32 * n)(*[o for _, o in self.dims])
        h = ctypes.c_void_p()
        _lib.check(self._lib.wp_pool_create(engine.handle, self.num_slots, n, self.rank, d_arr, o_arr,
                                            _DTYPES[dtype], self.max_adapters, ctypes.byref(h)), engine.handle)
        self._p = h
        a_off, b_off, sb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        self.layout: List[tuple] = []
        for p in range(n):
            _lib.check(self._lib.wp_pool_layout(self._p, p, ctypes.byref(a_off), ctypes.byref(b_off), ctypes.byref(sb)),
                       engine.handle)
            self.layout.append((a_off.value, b_off.value))
        self.slot_bytes = sb.value
        self._stacks = []
        wa, wb, st = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int64()
        for p in range(n):
            _lib.check(self._lib.wp_pool_stack(self._p, p, ctypes.byref(wa), ctypes.byref(wb), ctypes.byref(st)),
                       engine.handle)
            self._stacks.append((wa.value, wb.value, st.value))
        self._blobs = {}

    # -- host store ------------------------------------------------------------
    def pack(self, adapter: Sequence[tuple]) -> torch.Tensor:
        """A page-locked host blob in the slot layout from per-projection
        (A [rank, d], B [o, rank]) tensors."""
        blob = torch.zeros(self.slot_bytes, dtype=torch.uint8).pin_memory()
        self.fill(blob, adapter)
        return blob

    def fill(self, blob: torch.Tensor, adapter: Sequence[tuple]) -> None:
        if len(adapter) != len(self.dims):
            raise ValueError(f"expected {len(self.dims)} projections, got {len(adapter)}")
        for (d, o), (a_off, b_off), (A, B) in zip(self.dims, self.layout, adapter):
            if tuple(A.shape) != (self.rank, d) or tuple(B.shape) != (o, self.rank):
                raise ValueError("adapter projection shapes do not match the pool")
            blob[a_off:a_off + A.numel() * 2].copy_(A.to(self.dtype).contiguous().view(-1).view(torch.uint8))
            blob[b_off:b_off + B.numel() * 2].copy_(B.to(self.dtype).contiguous().view(-1).view(torch.uint8))

    def register_host(self, adapter_id: int, blob: torch.Tensor) -> None:
        """Registers a page-locked blob of slot_bytes (kept referenced here)."""
        if blob.device.type != "cpu" or not blob.is_pinned() or blob.numel() * blob.element_size() < self.slot_bytes:
            raise RuntimeError("register_host: the blob must be a pinned CPU tensor of slot_bytes")
        _lib.check(self._lib.wp_pool_register_host(self._p, int(adapter_id), blob.data_ptr()), self.engine.handle)
        self._blobs[int(adapter_id)] = blob

    def evict(self, adapter_id: int) -> None:
        _lib.check(self._lib.wp_pool_evict(self._p, int(adapter_id)), self.engine.handle)
        self._blobs.pop(int(adapter_id), None)

    # -- staging (reference semantics) -------------------------------------------
    def prefetch(self, adapter_id: int) -> int:
        return int(self._lib.wp_pool_prefetch(self._p, int(adapter_id)))

    def is_prefetch_ready(self, adapter_id: int) -> bool:
        return bool(self._lib.wp_pool_is_ready(self._p, int(adapter_id)))

    def release_prefetch(self, adapter_id: int) -> None:
        self._lib.wp_pool_release(self._p, int(adapter_id))

    # -- one step ----------------------------------------------------------------
    def prepare(self, adapter_ids) -> int:
        """Makes the step's adapters resident on the current stream; returns
        the number of cold misses (copies issued by this call)."""
        ids = sorted({int(i) for i in adapter_ids if int(i) >= 0})
        arr = (ctypes.c_int32 * max(1, len(ids)))(*ids)
        return _lib.check(self._lib.wp_pool_prepare(self._p, arr, len(ids), _stream_ptr(self.engine.device)),
                          self.engine.handle)

    def build_seg_bounds(self, token_lora_indices: torch.Tensor) -> bool:
        idx = token_lora_indices.reshape(-1)
        if not idx.is_cuda:
            raise RuntimeError("build_seg_bounds: token_lora_indices must be a CUDA tensor")
        if idx.dtype not in (torch.int32, torch.int64):
            idx = idx.to(torch.int64)
        idx = idx.contiguous()
        dt = _lib.WP_DTYPE_I64 if idx.dtype == torch.int64 else _lib.WP_DTYPE_I32
        rc = _lib.check(self._lib.wp_build_seg_bounds_pool(self.engine.handle, self._p, idx.data_ptr(), dt,
                                                           int(idx.numel()), _stream_ptr(self.engine.device)),
                        self.engine.handle)
        return rc == 0

    def add_lora(self, proj: int, y: torch.Tensor, x: torch.Tensor, scale: float) -> bool:
        """y += (x . A^T * scale) . B^T with the adapters of projection `proj`."""
        wa, wb, stride0 = self._stacks[proj]
        d, o = self.dims[proj]
        x2 = x.reshape(-1, x.size(-1))
        y2 = y.view(-1, y.size(-1))
        if x2.size(1) != d or y2.size(1) != o or x.dtype != self.dtype or y.dtype != self.dtype:
            raise RuntimeError("add_lora: x / y do not match the projection")
        h = self.engine.handle
        _lib.check(self._lib.wp_add_lora(h, y2.data_ptr(), x2.data_ptr(), wa, stride0, wb, stride0, self.num_slots,
                                         float(scale), int(x2.size(0)), d, o, self.rank, int(x2.stride(0)),
                                         int(y2.stride(0)), 0, _DTYPES[self.dtype], _stream_ptr(self.engine.device)), h)
        return True

    def stats(self) -> dict:
        c, b, r = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int32()
        self._lib.wp_pool_stats(self._p, ctypes.byref(c), ctypes.byref(b), ctypes.byref(r))
        return {"copies": c.value, "bytes": b.value, "resident": r.value}

    def close(self) -> None:
        if self._p:
            self._lib.wp_pool_destroy(self._p)
            self._p = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
