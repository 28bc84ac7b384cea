"""Tensor-parallel grouped LoRA apply (one process per GPU, NCCL over NVLink).

The reference is single-GPU; this is the sharding of the apply path for a
tensor-parallel base model, following vLLM's LoRA layers
(vllm/lora/layers/column_parallel_linear.py, row_parallel_linear.py):

  column-parallel layers (q, k, v, gate, up): x and A are replicated, B and
    the output y are split along out_features. Each rank shrinks the full
    [T, r] H and expands only its own output columns -- no collective.
  row-parallel layers (o, down): x and A are split along d_model; B is full.
    Three ways to combine the ranks, chosen by ``row_mode``:

    "partial" (default; vLLM's RowParallelLinearWithLoRA): each rank adds
      (scale * x_p . A_p^T) . B^T into its own *partial* output, the base
      layer's row-parallel partial sum. The base layer's all-reduce of that
      output, which a tensor-parallel model runs anyway, sums the ranks'
      LoRA terms with the base terms: by linearity the sum over ranks is
      (scale * x . A^T) . B^T. The LoRA path itself moves no bytes between
      GPUs and waits on no peer.
    "fused": ONE launch (wp_add_lora_row_parallel) that produces the full
      LoRA term on every rank: each segment's partial H is written straight
      into the peers' mailboxes (device memory mapped over NVLink through
      CUDA IPC), released with a flag, waited for (bounded) and summed in
      rank order inside the apply kernel.
    "nccl": three launches (wp_add_lora_shrink, wp_tp_allreduce_f32 of the
      fp32 [T, r] partials, wp_add_lora_expand), the S-LoRA form.

Everything runs on the caller's stream, so a whole step can be captured in
one CUDA graph.

The sharding helpers are pure tensor slicing and run anywhere; the apply
methods need the CUDA engine.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib


def _span(n: int, rank: int, world: int) -> tuple[int, int]:
    if n % world:
        raise ValueError(f"dimension {n} does not split over {world} ranks")
    step = n // world
    return rank * step, (rank + 1) * step


def shard_column(wb_t_all: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's out_features slice of B ([L, 1, o, r] -> [L, 1, o/world, r]), contiguous."""
    a, b = _span(wb_t_all.size(-2), rank, world)
    return wb_t_all[..., a:b, :].contiguous()


def shard_column_output(y: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    a, b = _span(y.size(-1), rank, world)
    return y[..., a:b]


def shard_row(wa_t_all: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's d_model slice of A ([L, 1, r, d] -> [L, 1, r, d/world]), contiguous."""
    a, b = _span(wa_t_all.size(-1), rank, world)
    return wa_t_all[..., a:b].contiguous()


def shard_row_input(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    a, b = _span(x.size(-1), rank, world)
    return x[..., a:b].contiguous()


class TensorParallelApply:
    """Grouped LoRA apply over a tensor-parallel group of `world` GPUs.

    Needs torch.distributed initialised (any backend; it only carries the
    NCCL unique id) and one WarpPipeEngine on this rank's device. Every rank
    runs build_seg_bounds on identical indices (the table is replicated, not
    exchanged)."""

    def __init__(self, engine, rank: Optional[int] = None, world: Optional[int] = None, group=None,
                 fused: Optional[bool] = None, row_mode: str = "partial"):
        import torch.distributed as dist

        if fused is not None:  # older spelling: fused=True -> "fused", fused=False -> "nccl"
            row_mode = "fused" if fused else "nccl"
        if row_mode not in ("partial", "fused", "nccl"):
            raise ValueError(f"row_mode must be 'partial', 'fused' or 'nccl', not {row_mode!r}")
        self.row_mode = row_mode

        self.engine = engine
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        lib = _lib.load()
        self._lib = lib
        nbytes = int(lib.wp_tp_unique_id_bytes())
        uid = (ctypes.c_char * nbytes)()
        if self.rank == 0:
            _lib.check(lib.wp_tp_get_unique_id(uid), None)
        obj = [bytes(uid)] if self.rank == 0 else [None]
        dist.broadcast_object_list(obj, src=0, group=group)
        uid = (ctypes.c_char * nbytes).from_buffer_copy(obj[0])
        _lib.check(lib.wp_tp_init(engine.handle, uid, self.rank, self.world), engine.handle)
        self._H = torch.empty(engine.config.max_tokens * 64, dtype=torch.float32, device=engine.device)
        self.fused = row_mode == "fused" and self.world > 1
        if self.fused:
            # every rank's mailbox, mapped into every process (CUDA IPC over NVLink)
            hb = int(lib.wp_tp_mailbox_handle_bytes())
            mine = (ctypes.c_char * hb)()
            _lib.check(lib.wp_tp_mailbox_create(engine.handle, self.rank, self.world, engine.config.max_tokens, mine),
                       engine.handle)
            got = [None] * self.world
            dist.all_gather_object(got, bytes(mine), group=group)
            allh = (ctypes.c_char * (hb * self.world)).from_buffer_copy(b"".join(got))
            _lib.check(lib.wp_tp_mailbox_open(engine.handle, allh), engine.handle)
        # every rank is past its set-up before any rank's first exchange
        # launch (a peer still initialising would otherwise eat into the
        # exchange's bounded wait)
        dist.barrier(group=group)

    def close(self):
        import torch.distributed as dist

        if self.fused:
            # no rank unmaps a mailbox while a peer may still write into it
            torch.cuda.synchronize(self.engine.device)
            dist.barrier()
            self._lib.wp_tp_mailbox_close(self.engine.handle)
        self._lib.wp_tp_destroy(self.engine.handle)

    def column_parallel(self, y_shard, x, wa_t_all, wb_shard, scale) -> bool:
        """y_shard[t] += (x[t] . A^T * scale) . B_shard^T; no collective.
        y_shard may be a column slice of a wider y."""
        full = y_shard
        if y_shard.stride(0) != y_shard.size(-1):
            return self.engine.add_lora_strided(y_shard, x, wa_t_all, wb_shard, scale)
        return self.engine.add_lora_packed(full, x, wa_t_all, wb_shard, scale)

    def row_parallel(self, y, x_shard, wa_shard, wb_t_all, scale) -> bool:
        """Row-parallel LoRA term from this rank's d slice of x and A and the
        full B. row_mode "partial": y is this rank's partial output and
        receives this rank's share (the caller's all-reduce of y completes
        it). "fused" / "nccl": y is the replicated output and receives the
        full term (sum of the ranks' H, then the expand)."""
        eng, lib = self.engine, self._lib
        r = int(wb_t_all.size(-1))
        if not eng.rank_supported(r):
            return False
        if self.row_mode == "partial" or self.world == 1:
            return self.engine.add_lora_packed(y, x_shard, wa_shard, wb_t_all, scale)
        x2d = x_shard.reshape(-1, x_shard.size(-1))
        y2d = y.view(-1, y.size(-1))
        T, d = int(x2d.size(0)), int(x2d.size(1))
        dt = _lib.WP_DTYPE_BF16 if x2d.dtype == torch.bfloat16 else _lib.WP_DTYPE_F16
        if self.fused:
            h = eng.handle
            stream = torch.cuda.current_stream(eng.device).cuda_stream
            _lib.check(lib.wp_add_lora_row_parallel(
                h, y2d.data_ptr(), x2d.data_ptr(), wa_shard.data_ptr(), wa_shard.stride(0), wb_t_all.data_ptr(),
                wb_t_all.stride(0), int(wa_shard.size(0)), float(scale), T, d, int(wb_t_all.size(-2)), r,
                x2d.stride(0), y2d.stride(0), 0, dt, stream), h)
            return True
        H = self._H[:T * r].view(T, r)
        stream = torch.cuda.current_stream(eng.device).cuda_stream
        h = eng.handle
        _lib.check(lib.wp_add_lora_shrink(h, H.data_ptr(), x2d.data_ptr(), wa_shard.data_ptr(), wa_shard.stride(0),
                                          int(wa_shard.size(0)), float(scale), T, d, r, x2d.stride(0), dt, stream), h)
        _lib.check(lib.wp_tp_allreduce_f32(h, H.data_ptr(), T * r, stream), h)
        _lib.check(lib.wp_add_lora_expand(h, y2d.data_ptr(), H.data_ptr(), wb_t_all.data_ptr(), wb_t_all.stride(0),
                                          int(wb_t_all.size(0)), T, int(wb_t_all.size(-2)), r, y2d.stride(0), 0, dt, stream), h)
        return True
