"""vLLM hook: the reference's FusedPunicaWrapperWarpPipe over libwp_b200.so.

Mirrors lora_warp_pipe/punica_wrapper.py:86-159,219-238 of the reference:
``update_metadata`` builds the step's segment table once (eager, before any
graph replay) and ``add_lora`` runs the grouped shrink+expand of one LoRA
layer. The class is installed by reassigning ``__class__`` of vLLM's
PunicaWrapper instance, like the reference.

Unlike the reference there is no stock-path fallback once installed: prefill
steps (any token count up to the engine's max_tokens), sliced outputs
(``y_offset``/``y_slice_size``) and ranks 8/16/32/64 all run on the B200
kernels. A call outside that envelope raises. The AS_WARP_PIPE=1 opt-in gate
is checked when the hook is installed.

AdapterSlots' FusedPunicaWrapper (the reference's base class) is an empty
submodule in the reference checkout; when it is not importable the hook
derives from a minimal base that carries the two attributes the hook reads
(``is_prefill``, ``token_lora_indices``).
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from .engine import WarpPipeEngine

try:  # the AdapterSlots serving system, when installed
    from adapter_slots.kernel.fused_punica_wrapper import FusedPunicaWrapper, _VLLM_PUNICA_AVAILABLE  # type: ignore
except Exception:  # pragma: no cover - AdapterSlots is not part of this build
    _VLLM_PUNICA_AVAILABLE = True

    class FusedPunicaWrapper:  # minimal stand-in base
        is_prefill: bool = False
        token_lora_indices: Optional[torch.Tensor] = None

        def update_metadata(self, mapping, lora_index_to_id, max_loras, vocab_size, extra_vocab_size,
                            long_lora_context=None) -> None:
            pass


_engine: Optional[WarpPipeEngine] = None


def _get_engine() -> WarpPipeEngine:
    """Lazy singleton: the engine allocates device memory, so it is created
    on first use, after the CUDA context exists.

    Serving contract: adapter weights are not written while a step runs
    (vLLM loads them between steps), and the kernel right before a LoRA call
    is the base layer's GEMM, which reads x and writes y. So the engine runs
    with prefetch_weights and prefetch_inputs: each apply launch streams its
    adapter weights and x, and runs its shrink, while the preceding kernel
    finishes (programmatic dependent launch); y is read after that kernel
    completes."""
    global _engine
    if _engine is None:
        from .config import WarpPipeConfig

        _engine = WarpPipeEngine(WarpPipeConfig(prefetch_weights=True, prefetch_inputs=True))
    return _engine


def warp_pipe_available() -> bool:
    return os.environ.get("AS_WARP_PIPE", "0") == "1"


class FusedPunicaWrapperWarpPipe(FusedPunicaWrapper):
    """PunicaWrapper whose add_lora runs the grouped B200 apply."""

    def update_metadata(self, mapping, lora_index_to_id, max_loras, vocab_size, extra_vocab_size,
                        long_lora_context=None) -> None:
        super().update_metadata(mapping, lora_index_to_id, max_loras, vocab_size, extra_vocab_size,
                                long_lora_context)
        if not _get_engine().build_seg_bounds(self.token_lora_indices):
            raise RuntimeError(
                f"build_seg_bounds: {self.token_lora_indices.numel()} tokens exceed the engine's max_tokens "
                f"({_get_engine().config.max_tokens}); raise WarpPipeConfig.max_tokens")

    def add_lora(self, y: torch.Tensor, x: torch.Tensor, wa_t_all: torch.Tensor, wb_t_all: torch.Tensor,
                 scale: float, y_offset: Optional[int] = None, y_slice_size: Optional[int] = None, *,
                 buffer: Optional[torch.Tensor] = None) -> None:
        handled = _get_engine().add_lora(y, x, wa_t_all, wb_t_all, float(scale), y_offset, y_slice_size)
        if not handled:
            raise RuntimeError(f"add_lora: rank {wb_t_all.size(-1)} is not supported (8/16/32/64)")


def install_warp_pipe_add_lora(lora_manager) -> bool:
    """Reassign the shared PunicaWrapper instance's __class__ to
    FusedPunicaWrapperWarpPipe. Returns False (a no-op) when AS_WARP_PIPE is
    not "1", vLLM LoRA support is unavailable, lora_manager is None, or the
    wrapper is already installed."""
    if not warp_pipe_available() or not _VLLM_PUNICA_AVAILABLE or lora_manager is None:
        return False
    adapter_manager = getattr(lora_manager, "_adapter_manager", None)
    if adapter_manager is None:
        return False
    wrapper = getattr(adapter_manager, "punica_wrapper", None)
    if wrapper is None or isinstance(wrapper, FusedPunicaWrapperWarpPipe):
        return False
    wrapper.__class__ = FusedPunicaWrapperWarpPipe
    return True
