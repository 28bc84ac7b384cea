"""Engine configuration (mirror of lora_warp_pipe/config.py:4-9 of the reference).

The reference fields keep their meaning: ``rank`` is the default rank of
register_adapter; ``num_staging_slots`` is the size of the staging pool (the
reference hard-codes WP_MAX_STAGING = 8; here the field is honoured). The
remaining fields size the device tables and tune the kernels.
"""

from dataclasses import dataclass


@dataclass
class WarpPipeConfig:
    enabled: bool = True
    rank: int = 32
    num_staging_slots: int = 8
    min_segment_tokens: int = 4  # kept for signature parity; the reference never reads it either
    # capacity of the per-step tables: the largest token count of one step
    max_tokens: int = 16384
    # bytes of one staging slot (A and B of one adapter); 0 = rank 64 x 16384 x 2 matrices
    slot_bytes: int = 0
    # programmatic dependent launch between consecutive apply kernels
    use_pdl: bool = True
    # with use_pdl: load adapter weights before the previous kernel on the
    # stream has finished. Only valid when that kernel never writes the
    # weights (serving: weights are static while a step runs).
    prefetch_weights: bool = False
    # cap on persistent CTAs per SM of the apply kernel (0 = as many as fit)
    ctas_per_sm: int = 0
    # apply kernel of fused live-mode calls: "auto", "cluster" (clustered,
    # mma.sync), "split" (balanced: one CTA per SM, equal one-stage items)
    kernel: str = "auto"
    # build_seg_bounds(prefill=None) sends runs of >= 128 tokens to the
    # tcgen05 prefill kernels when the step has at least this many tokens
    # (0 = never, the default: the decode kernel is faster on the measured
    # prefill mixes; prefill=True selects the prefill kernels explicitly)
    prefill_tokens: int = 0
    # bound of each in-kernel wait on a tensor-parallel peer (the fused
    # row-parallel exchange), in ms; 0 = 5000
    peer_wait_ms: int = 0
    # with prefetch_weights: a fused live call loads x and runs its shrink
    # before the previous kernel on the stream has finished (only its y
    # loads wait). Only valid when that kernel never writes the call's x
    # (serving: it is the base layer's GEMM, which writes y).
    prefetch_inputs: bool = False
