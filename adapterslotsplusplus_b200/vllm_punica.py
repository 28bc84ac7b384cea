"""vLLM-current hook: the container's vLLM (0.22) PunicaWrapperGPU routed to
the B200 kernels.

The reference hooks vLLM 0.6.3's ``PunicaWrapper.add_lora``
(lora_warp_pipe/punica_wrapper.py:119-159), which vLLM 0.22 no longer has:
its LoRA linear layers call ``add_lora_linear`` (vllm/lora/layers/
base_linear.py), which runs ``add_shrink`` then ``add_expand`` over the
layer's slices (vllm/lora/punica_wrapper/punica_gpu.py). This module keeps the
reference's mechanism -- reassigning ``__class__`` of the live wrapper -- and
maps those three entry points onto one engine:

  update_metadata  -> build_seg_bounds (once per step, eager, before replay)
  add_lora_linear  -> one launch per group of up to three equal-width slices
                      (add_lora_packed_nslice), else one launch per slice
                      (add_lora with y_offset); add_inputs=False writes the
                      LoRA-only output into a zeroed y, as vLLM's dual-stream
                      path expects;
  add_shrink       -> add_lora_shrink per slice into vLLM's fp32 buffer;
  add_expand       -> add_lora_expand per slice at its column offset.

Layouts match vLLM's stacks: lora_a_stacked[i] is [max_loras, 1, rank, in],
lora_b_stacked[i] is [max_loras, 1, out_i, rank]. The embedding and logits
entry points are not LoRA linear layers and keep vLLM's implementation.
Like the reference's hook, nothing falls back to the stock kernels on the
linear path: an unsupported call raises.
"""

from __future__ import annotations

import os
from typing import Optional, Sequence

import torch

_engine = None


def _get_engine():
    """Lazy singleton (the engine allocates device memory). Runs with
    prefetch_weights and prefetch_inputs: vLLM writes the LoRA stacks only
    between steps, and the kernel right before a LoRA call is the base
    layer's GEMM (it reads x and writes y), so an apply launch may stream
    adapter weights and x, and run its shrink, while that GEMM finishes; y is
    read after it."""
    global _engine
    if _engine is None:
        from .config import WarpPipeConfig
        from .engine import WarpPipeEngine

        _engine = WarpPipeEngine(WarpPipeConfig(prefetch_weights=True, prefetch_inputs=True))
    return _engine


def apply_lora_linear(engine, y: torch.Tensor, x: torch.Tensor, lora_a_stacked: Sequence[torch.Tensor],
                      lora_b_stacked: Sequence[torch.Tensor], scale: float, output_slices: Sequence[int],
                      add_inputs: bool = True) -> None:
    """vLLM's add_lora_linear semantics on the engine: for every slice i,
    y[:, off_i : off_i + out_i] += (x . A_i^T * scale) . B_i^T with the
    per-token adapter of the last build_seg_bounds; off_i = sum(out_<i)."""
    if not (len(lora_a_stacked) == len(lora_b_stacked) == len(output_slices)) or not output_slices:
        raise RuntimeError("add_lora_linear: slice lists differ in length")
    y2 = y.view(-1, y.size(-1))
    x2 = x.reshape(-1, x.size(-1))
    if not add_inputs:
        y2.zero_()
    if x2.data_ptr() != x.data_ptr():
        engine.note_input_write()  # the reshape copied x right before the apply (prefetch_inputs)
    widths = [int(w) for w in output_slices]
    if len(set(widths)) == 1 and len(widths) > 1 and sum(widths) == y2.size(1):
        if not engine.add_lora_packed_nslice(y2, x2, list(lora_a_stacked), list(lora_b_stacked), scale, widths):
            raise RuntimeError(f"add_lora_linear: rank {lora_b_stacked[0].size(-1)} is not supported")
        return
    off = 0
    for a, b, w in zip(lora_a_stacked, lora_b_stacked, widths):
        if not engine.add_lora(y2, x2, a, b, scale, off, w):
            raise RuntimeError(f"add_lora_linear: rank {b.size(-1)} is not supported")
        off += w


def apply_shrink(engine, y: torch.Tensor, x: torch.Tensor, lora_a_stacked: Sequence[torch.Tensor], scale: float) -> None:
    """vLLM's add_shrink: y[i] = (x . A_i^T) * scale for the rows with an
    adapter, 0 elsewhere (y fp32 [slices, T, rank], zeroed here as vLLM's
    shrink op zeroes its buffer)."""
    x2 = x.reshape(-1, x.size(-1))
    y.zero_()
    for i, a in enumerate(lora_a_stacked):
        if not engine.add_lora_shrink(y[i], x2, a, scale):
            raise RuntimeError(f"add_shrink: rank {a.size(-2)} is not supported")


def apply_expand(engine, y: torch.Tensor, x: torch.Tensor, lora_b_stacked: Sequence[torch.Tensor],
                 output_slices: Sequence[int], offset_start: int = 0, add_inputs: bool = True) -> None:
    """vLLM's add_expand: y[:, off : off + out_i] += x[i] . B_i^T, off from
    offset_start (x fp32 [slices, T, rank])."""
    y2 = y.view(-1, y.size(-1))
    if x.ndim != 3 or x.size(0) != len(output_slices):
        raise RuntimeError("add_expand: x must be [slices, T, rank]")
    off = int(offset_start)
    if not add_inputs:
        y2[:, off:off + sum(int(w) for w in output_slices)].zero_()
    for i, (b, w) in enumerate(zip(lora_b_stacked, output_slices)):
        if not engine.add_lora_expand(y2, x[i].contiguous(), b, off):
            raise RuntimeError(f"add_expand: rank {b.size(-1)} is not supported")
        off += int(w)


_CLASS = None


def wrapper_class():
    """The PunicaWrapperGPU subclass whose LoRA linear path runs the B200
    kernels, created on first use (importing vLLM takes seconds), or None
    when vLLM's GPU wrapper does not import here."""
    global _CLASS
    if _CLASS is not None:
        return _CLASS
    try:
        from vllm.lora.punica_wrapper.punica_gpu import PunicaWrapperGPU  # type: ignore
    except Exception:  # vLLM absent or not importable
        return None

    class WarpPipePunicaWrapperGPU(PunicaWrapperGPU):
        """vLLM PunicaWrapperGPU whose LoRA linear path runs the B200 kernels."""

        def update_metadata(self, mapping, lora_index_to_id, max_loras, vocab_size, **kwargs):
            super().update_metadata(mapping, lora_index_to_id, max_loras, vocab_size, **kwargs)
            eng = _get_engine()
            if not eng.build_seg_bounds(self.token_lora_indices):
                raise RuntimeError(
                    f"build_seg_bounds: {self.token_lora_indices.numel()} tokens exceed the engine's max_tokens "
                    f"({eng.config.max_tokens}); raise WarpPipeConfig.max_tokens")

        def add_lora_linear(self, y, x, lora_a_stacked, lora_b_stacked, scale, output_slices, *, buffer=None,
                            **kwargs):
            add_inputs = kwargs.pop("add_inputs", True)
            apply_lora_linear(_get_engine(), y, x, lora_a_stacked, lora_b_stacked, float(scale), output_slices,
                              add_inputs)
            return y

        def add_shrink(self, y, x, lora_a_stacked, scale, **kwargs):
            apply_shrink(_get_engine(), y, x, lora_a_stacked, float(scale))

        def add_expand(self, y, x, lora_b_stacked, output_slices, offset_start=0, add_inputs=True, **kwargs):
            apply_expand(_get_engine(), y, x, lora_b_stacked, output_slices, offset_start, add_inputs)

    _CLASS = WarpPipePunicaWrapperGPU
    return _CLASS


def install_warp_pipe_punica(wrapper) -> bool:
    """Reassign the live PunicaWrapperGPU instance's __class__ (the
    reference's mechanism, punica_wrapper.py:219-238). Returns False when
    AS_WARP_PIPE is not "1", vLLM's GPU wrapper is unavailable, or the
    instance is not a PunicaWrapperGPU (or is already installed)."""
    if os.environ.get("AS_WARP_PIPE", "0") != "1" or wrapper is None:
        return False
    cls = wrapper_class()
    if cls is None or isinstance(wrapper, cls) or not isinstance(wrapper, cls.__mro__[1]):
        return False
    wrapper.__class__ = cls
    return True


def find_punica_wrapper(lora_manager) -> Optional[object]:
    """The PunicaWrapper of a vLLM LoRA model manager (its ``punica_wrapper``
    attribute, or the one of its ``_adapter_manager``)."""
    for obj in (lora_manager, getattr(lora_manager, "_adapter_manager", None)):
        w = getattr(obj, "punica_wrapper", None) if obj is not None else None
        if w is not None:
            return w
    return None
