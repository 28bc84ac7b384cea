"""WarpPipeEngine: the reference's Python engine surface over libwp_b200.so.

Mirrors lora_warp_pipe/engine.py:7-69 of vac014/AdapterSlotsPlusPlus method by
method (same names, argument meaning, return values and error behaviour),
with the pybind extension replaced by the C ABI of include/wp_api.h. Every
compute call runs a CUDA kernel of libwp_b200.so on the caller's current
torch stream; there is no CPU or stock-kernel fallback.

Differences from the reference, all widening what is handled:
  * fp16 and bf16 (the reference is fp16 only);
  * ranks 8/16/32/64 on every path (the live path of the reference is rank 32);
  * any token count up to ``config.max_tokens`` (the reference returns False
    from build_seg_bounds above 256 tokens), any d_model/out_features that are
    multiples of 8 (the reference needs multiples of 256), segments of any
    length on the registry path (the reference covers 32 tokens per segment);
  * ``shrink`` returns H in fp32 (the reference rounds H to fp16);
  * sliced outputs (``y_offset``/``y_slice_size``) through ``add_lora``;
  * CPU tensors given to ``register_adapter`` go to a pinned-host store and
    reach the GPU through the staging slots.
"""

from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib
from .config import WarpPipeConfig

_DTYPES = {torch.float16: _lib.WP_DTYPE_F16, torch.bfloat16: _lib.WP_DTYPE_BF16}


def _dtype_code(t: torch.Tensor, what: str) -> int:
    code = _DTYPES.get(t.dtype)
    if code is None:
        raise RuntimeError(f"{what} must be fp16 or bf16, got {t.dtype}")
    return code


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class WarpPipeEngine:
    """Grouped multi-LoRA apply engine (one per device)."""

    def __init__(self, config: Optional[WarpPipeConfig] = None, device=None):
        self.config = config or WarpPipeConfig()
        if not torch.cuda.is_available():
            raise RuntimeError("WarpPipeEngine needs a CUDA device (libwp_b200.so has no CPU path)")
        self._lib = _lib.load()
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index or 0)
        cfg = _lib.WpConfig(
            device=self.device.index,
            max_tokens=int(self.config.max_tokens),
            num_staging_slots=int(self.config.num_staging_slots),
            slot_bytes=int(self.config.slot_bytes),
            ctas_per_sm=int(self.config.ctas_per_sm),
            use_pdl=1 if self.config.use_pdl else 0,
            prefetch_weights=1 if self.config.prefetch_weights else 0,
            kernel={"auto": 0, "cluster": 1, "split": 2}[self.config.kernel],
            prefill_tokens=int(self.config.prefill_tokens),
            peer_wait_ms=int(self.config.peer_wait_ms),
            prefetch_inputs=1 if self.config.prefetch_inputs else 0,
        )
        handle = ctypes.c_void_p()
        _lib.check(self._lib.wp_create(ctypes.byref(cfg), ctypes.byref(handle)), None)
        self._h = handle
        self._held: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}
        self._bridge: Optional[dict] = None
        # the reference exposes rank_supported on its extension object (engine._ext)
        self._ext = self

    # -- lifetime ----------------------------------------------------------
    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._lib.wp_destroy(h)
            self._h = ctypes.c_void_p()
        self._held.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int) -> int:
        return _lib.check(rc, self._h)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    # -- adapter store (engine.py:12-17) ---------------------------------------
    def register_adapter(self, adapter_id, A, B, alpha_scale, rank=None):
        rank = rank or self.config.rank
        if A.dtype != B.dtype:
            raise RuntimeError("A/B must have the same dtype")
        dt = _dtype_code(A, "A/B")
        if not (A.is_contiguous() and B.is_contiguous()):
            raise RuntimeError("A/B must be contiguous")
        d_model = int(A.size(-1))
        out_features = int(B.size(-2))
        if A.numel() != rank * d_model or B.numel() != out_features * rank:
            raise RuntimeError(f"A must be [rank={rank}, d_model] and B [out_features, rank={rank}]")
        if A.is_cuda != B.is_cuda:
            raise RuntimeError("A/B must both be CUDA tensors or both be CPU tensors")
        if A.is_cuda:
            self._check(self._lib.wp_register_adapter(self._h, int(adapter_id), A.data_ptr(), B.data_ptr(), rank,
                                                      d_model, out_features, float(alpha_scale), dt))
            self._held[int(adapter_id)] = (A, B)
        else:
            self._check(self._lib.wp_register_adapter_host(self._h, int(adapter_id), A.data_ptr(), B.data_ptr(),
                                                           rank, d_model, out_features, float(alpha_scale), dt))
            self._held.pop(int(adapter_id), None)

    def evict_adapter(self, adapter_id):
        self._check(self._lib.wp_evict_adapter(self._h, int(adapter_id)))
        self._held.pop(int(adapter_id), None)

    def rank_supported(self, rank) -> bool:
        return bool(self._lib.wp_rank_supported(int(rank)))

    # -- registry path (engine.py:19-26) ---------------------------------------
    def build_segments(self, sorted_adapter_ids: Sequence[int], seg_offsets: Sequence[int]):
        K = len(sorted_adapter_ids)
        if len(seg_offsets) != K + 1:
            raise RuntimeError("build_segment_table: seg_offsets must have K+1 entries")
        ids = (ctypes.c_int32 * max(K, 1))(*[int(i) for i in sorted_adapter_ids])
        offs = (ctypes.c_int32 * (K + 1))(*[int(o) for o in seg_offsets])
        self._check(self._lib.wp_build_segments(self._h, ids, offs, K, _stream_ptr(self.device)))

    def shrink(self, X, d_model, rank, total_tokens):
        if not (X.is_cuda and X.is_contiguous()):
            raise RuntimeError("X must be contiguous fp16/bf16 CUDA")
        dt = _dtype_code(X, "X")
        H = torch.zeros(int(total_tokens), int(rank), dtype=torch.float32, device=X.device)
        self._check(self._lib.wp_shrink(self._h, X.data_ptr(), H.data_ptr(), int(d_model), int(rank),
                                        int(total_tokens), dt, _stream_ptr(X.device)))
        return H

    def expand(self, H, Y, out_features, rank):
        if not (H.is_cuda and Y.is_cuda):
            raise RuntimeError("H/Y must be CUDA tensors")
        if not (H.is_contiguous() and Y.is_contiguous()):
            raise RuntimeError("H/Y must be contiguous")
        dt = _dtype_code(Y, "Y")
        if H.dtype != torch.float32:
            H = H.float()
        self._check(self._lib.wp_expand(self._h, H.data_ptr(), Y.data_ptr(), int(out_features), int(rank),
                                        int(H.size(0)), dt, _stream_ptr(Y.device)))

    # -- live path (engine.py:28-32, 56-62) --------------------------------------
    def build_seg_bounds(self, token_lora_indices, prefill: Optional[bool] = None) -> bool:
        """Builds the step's segment table on the device, once per step, ahead
        of every add_lora call of that step. Returns False only when the token
        count exceeds config.max_tokens. prefill: True sends runs of >= 128
        tokens of one adapter to the tcgen05 prefill kernels, False keeps the
        decode table only, None (default) decides by the token count
        (config.prefill_tokens)."""
        if not token_lora_indices.is_cuda:
            raise RuntimeError("build_seg_bounds: token_lora_indices must be a CUDA tensor")
        idx = token_lora_indices
        if idx.dtype not in (torch.int32, torch.int64):
            idx = idx.to(torch.int64)
        idx = idx.contiguous()
        code = _lib.WP_DTYPE_I64 if idx.dtype == torch.int64 else _lib.WP_DTYPE_I32
        flags = _lib.WP_SEG_AUTO if prefill is None else (_lib.WP_SEG_PREFILL if prefill else _lib.WP_SEG_DECODE)
        rc = self._check(self._lib.wp_build_seg_bounds_ex(self._h, idx.data_ptr(), code, int(idx.numel()), flags,
                                                          _stream_ptr(idx.device)))
        return rc == _lib.WP_OK

    def add_lora_packed(self, y, x, wa_t_all, wb_t_all, scale) -> bool:
        """Live-serving apply mirroring vLLM's PunicaWrapper.add_lora(): for
        every row i of x whose adapter id (from the last build_seg_bounds) is
        >= 0, y[i] += (x[i] @ wa_t_all[id].T * scale) @ wb_t_all[id].T.
        Returns False only for a rank outside {8, 16, 32, 64}."""
        return self.add_lora(y, x, wa_t_all, wb_t_all, scale)

    def add_lora(self, y, x, wa_t_all, wb_t_all, scale, y_offset: Optional[int] = None,
                 y_slice_size: Optional[int] = None) -> bool:
        """add_lora_packed plus a column slice of y: the update lands in
        y[:, y_offset : y_offset + y_slice_size] (vLLM's sliced add_lora)."""
        rank = int(wb_t_all.size(-1))
        if not self.rank_supported(rank):
            return False
        if not (x.is_cuda and y.is_cuda):
            raise RuntimeError("add_lora_packed: x/y must be CUDA tensors")
        dt = _dtype_code(x, "add_lora_packed: x/y")
        if y.dtype != x.dtype or wa_t_all.dtype != x.dtype or wb_t_all.dtype != x.dtype:
            raise RuntimeError("add_lora_packed: x, y, wa_t_all and wb_t_all must share one dtype")
        x2d = x.reshape(-1, x.size(-1))
        y2d = y.view(-1, y.size(-1))
        if x2d.stride(-1) != 1 or y2d.stride(-1) != 1:
            raise RuntimeError("add_lora_packed: x/y must be contiguous")
        if not (wa_t_all.is_contiguous() and wb_t_all.is_contiguous()):
            raise RuntimeError("add_lora_packed: wa_t_all/wb_t_all must be contiguous")
        T = int(x2d.size(0))
        d_model = int(x2d.size(1))
        if int(wa_t_all.size(-1)) != d_model or int(wa_t_all.size(-2)) != rank:
            raise RuntimeError("add_lora_packed: wa_t_all must be [L, 1, rank, d_model]")
        out_features = int(wb_t_all.size(-2))
        off = 0 if y_offset is None else int(y_offset)
        if y_slice_size is not None and int(y_slice_size) != out_features:
            raise RuntimeError("add_lora: y_slice_size must equal wb_t_all.size(-2)")
        if y_offset is None and y_slice_size is None and out_features != int(y2d.size(1)):
            raise RuntimeError("add_lora_packed: y.size(-1) must equal wb_t_all.size(-2)")
        if x2d.data_ptr() != x.data_ptr():
            self.note_input_write()  # reshape copied x: the copy is the kernel right before the apply
        self._check(self._lib.wp_add_lora(
            self._h, y2d.data_ptr(), x2d.data_ptr(), wa_t_all.data_ptr(), int(wa_t_all.stride(0)),
            wb_t_all.data_ptr(), int(wb_t_all.stride(0)), int(wa_t_all.size(0)), float(scale), T, d_model,
            out_features, rank,
            int(x2d.stride(0)), int(y2d.stride(0)), off, dt, _stream_ptr(x.device)))
        return True

    def note_input_write(self) -> None:
        """The kernel just enqueued on the current stream wrote the next apply
        call's x (e.g. a copy): with prefetch_inputs that call still loads x
        only after the preceding kernel has finished."""
        self._check(self._lib.wp_note_input_write(self._h))

    def add_lora_packed_nslice(self, y, x, lora_a_stacked, lora_b_stacked, scale, output_slices) -> bool:
        """vLLM's PunicaWrapper.add_lora_packed_nslice in one launch: slice s
        (lora_a_stacked[s] [L, 1, rank, d], lora_b_stacked[s] [L, 1, o, rank])
        adds into y[:, sum(output_slices[:s]) : ... + output_slices[s]]. The
        slices must share rank and width; up to three slices go in one launch,
        more are issued in groups of three."""
        n = len(lora_a_stacked)
        if n != len(lora_b_stacked) or n != len(output_slices) or n == 0:
            raise RuntimeError("add_lora_packed_nslice: slice lists differ in length")
        rank = int(lora_b_stacked[0].size(-1))
        if not self.rank_supported(rank):
            return False
        widths = {int(w) for w in output_slices}
        if len(widths) != 1 or any(int(b.size(-1)) != rank for b in lora_b_stacked):
            raise RuntimeError("add_lora_packed_nslice: slices must share rank and width")
        dt = _dtype_code(x, "add_lora_packed_nslice: x/y")
        x2d = x.reshape(-1, x.size(-1))
        y2d = y.view(-1, y.size(-1))
        if x2d.stride(-1) != 1 or y2d.stride(-1) != 1:
            raise RuntimeError("add_lora_packed_nslice: x/y must be contiguous")
        for t in (*lora_a_stacked, *lora_b_stacked):
            if t.dtype != x.dtype or not t.is_contiguous():
                raise RuntimeError("add_lora_packed_nslice: stacks must be contiguous and of x's dtype")
        T, d_model = int(x2d.size(0)), int(x2d.size(1))
        o = widths.pop()
        if sum(int(w) for w in output_slices) > int(y2d.size(1)):
            raise RuntimeError("add_lora_packed_nslice: output_slices exceed y's width")
        offs = [sum(int(w) for w in output_slices[:s]) for s in range(n)]
        if x2d.data_ptr() != x.data_ptr():
            self.note_input_write()  # reshape copied x right before the apply
        for g in range(0, n, 3):
            k = min(3, n - g)
            A, B = lora_a_stacked[g:g + k], lora_b_stacked[g:g + k]
            if any(int(a.size(-1)) != d_model or int(a.size(-2)) != rank for a in A):
                raise RuntimeError("add_lora_packed_nslice: lora_a must be [L, 1, rank, d_model]")
            if any(int(b.size(-2)) != o for b in B):
                raise RuntimeError("add_lora_packed_nslice: lora_b width must equal output_slices")
            self._check(self._lib.wp_add_lora_slices(
                self._h, y2d.data_ptr(), x2d.data_ptr(), k,
                (ctypes.c_void_p * k)(*[a.data_ptr() for a in A]),
                (ctypes.c_int64 * k)(*[int(a.stride(0)) for a in A]),
                (ctypes.c_void_p * k)(*[b.data_ptr() for b in B]),
                (ctypes.c_int64 * k)(*[int(b.stride(0)) for b in B]),
                (ctypes.c_int32 * k)(*offs[g:g + k]), int(A[0].size(0)), float(scale), T, d_model, o, rank,
                int(x2d.stride(0)), int(y2d.stride(0)), dt, _stream_ptr(x.device)))
        return True

    def add_lora_shrink(self, H, x, wa_t_all, scale) -> bool:
        """Shrink half of add_lora: H[t] = scale * x[t] . A_id(t)^T (fp32 H
        [T, rank]) for the rows of the live segments; other rows are left as
        they are."""
        rank = int(wa_t_all.size(-2))
        if not self.rank_supported(rank):
            return False
        dt = _dtype_code(x, "add_lora_shrink: x")
        x2d = x.reshape(-1, x.size(-1))
        if H.dtype != torch.float32 or not H.is_contiguous() or tuple(H.shape) != (x2d.size(0), rank):
            raise RuntimeError("add_lora_shrink: H must be contiguous fp32 [T, rank]")
        if wa_t_all.dtype != x.dtype or not wa_t_all.is_contiguous():
            raise RuntimeError("add_lora_shrink: wa_t_all must be contiguous, of x's dtype")
        self._check(self._lib.wp_add_lora_shrink(
            self._h, H.data_ptr(), x2d.data_ptr(), wa_t_all.data_ptr(), int(wa_t_all.stride(0)),
            int(wa_t_all.size(0)), float(scale), int(x2d.size(0)), int(x2d.size(1)), rank, int(x2d.stride(0)), dt,
            _stream_ptr(x.device)))
        return True

    def add_lora_expand(self, y, H, wb_t_all, y_offset: int = 0) -> bool:
        """Expand half of add_lora: y[t, y_offset + j] += H[t] . B_id(t)[j] for
        the rows of the live segments (H fp32 [T, rank])."""
        rank = int(wb_t_all.size(-1))
        if not self.rank_supported(rank):
            return False
        dt = _dtype_code(y, "add_lora_expand: y")
        y2d = y.view(-1, y.size(-1))
        if H.dtype != torch.float32 or not H.is_contiguous() or tuple(H.shape) != (y2d.size(0), rank):
            raise RuntimeError("add_lora_expand: H must be contiguous fp32 [T, rank]")
        if wb_t_all.dtype != y.dtype or not wb_t_all.is_contiguous():
            raise RuntimeError("add_lora_expand: wb_t_all must be contiguous, of y's dtype")
        self._check(self._lib.wp_add_lora_expand(
            self._h, y2d.data_ptr(), H.data_ptr(), wb_t_all.data_ptr(), int(wb_t_all.stride(0)),
            int(wb_t_all.size(0)), int(y2d.size(0)), int(wb_t_all.size(-2)), rank, int(y2d.stride(0)),
            int(y_offset), dt, _stream_ptr(y.device)))
        return True

    def add_lora_strided(self, y_view, x, wa_t_all, wb_t_all, scale) -> bool:
        """add_lora onto a column view of a wider row-major y (e.g. a
        tensor-parallel output shard): the view's row stride is used as is."""
        base = y_view
        if y_view.stride(-1) != 1:
            raise RuntimeError("add_lora_strided: the view's columns must be contiguous")
        rank = int(wb_t_all.size(-1))
        if not self.rank_supported(rank):
            return False
        dt = _dtype_code(x, "add_lora: x/y")
        x2d = x.reshape(-1, x.size(-1))
        self._check(self._lib.wp_add_lora(
            self._h, base.data_ptr(), x2d.data_ptr(), wa_t_all.data_ptr(), int(wa_t_all.stride(0)),
            wb_t_all.data_ptr(), int(wb_t_all.stride(0)), int(wa_t_all.size(0)), float(scale), int(x2d.size(0)),
            int(x2d.size(1)), int(wb_t_all.size(-2)), rank, int(x2d.stride(0)), int(base.stride(0)), 0, dt,
            _stream_ptr(x.device)))
        return True

    # -- staging slots (engine.py:44-54) -----------------------------------------
    def prefetch_adapter(self, adapter_id) -> int:
        """Copy adapter_id's A/B into a staging slot on the engine's private
        stream. Returns the slot index, or -1 if the id is unknown or no slot
        is free."""
        return int(self._lib.wp_prefetch_adapter_on(self._h, int(adapter_id), _stream_ptr(self.device)))

    def is_prefetch_ready(self, adapter_id) -> bool:
        return bool(self._lib.wp_is_prefetch_ready(self._h, int(adapter_id)))

    def release_prefetch(self, adapter_id):
        self._check(self._lib.wp_release_prefetch(self._h, int(adapter_id)))

    def slot_stats(self) -> Tuple[int, int]:
        n, used = ctypes.c_int32(), ctypes.c_int32()
        self._check(self._lib.wp_slot_stats(self._h, ctypes.byref(n), ctypes.byref(used)))
        return n.value, used.value

    # -- readbacks ---------------------------------------------------------------
    def read_seg_table(self, which: str = "live") -> List[Tuple[int, int, int]]:
        """(adapter_id, token_start, token_count) of every entry of the live
        (build_seg_bounds), registry (build_segments), "tiles" (prefill-mode
        128-token tiles) or "short" (prefill-mode short-run pieces) table.
        Synchronises."""
        code = {"live": _lib.WP_TABLE_LIVE, "registry": _lib.WP_TABLE_REGISTRY, "tiles": _lib.WP_TABLE_TILES,
                "short": _lib.WP_TABLE_SHORT}[which]
        n = ctypes.c_int32()
        self._check(self._lib.wp_read_seg_table(self._h, code, None, 0, ctypes.byref(n)))
        buf = (_lib.WpSegment * max(n.value, 1))()
        self._check(self._lib.wp_read_seg_table(self._h, code, buf, n.value, ctypes.byref(n)))
        return [(buf[i].adapter_id, buf[i].token_start, buf[i].token_count) for i in range(n.value)]

    def device_error(self, clear: bool = False) -> int:
        flag = ctypes.c_int32()
        self._check(self._lib.wp_device_error(self._h, 1 if clear else 0, ctypes.byref(flag)))
        return flag.value

    def apply_plan(self, dtype=torch.bfloat16, rank: int = 32) -> Tuple[int, int]:
        """(cluster size, CTAs) of the apply kernel for this dtype and rank."""
        c, g = ctypes.c_int32(), ctypes.c_int32()
        self._check(self._lib.wp_apply_plan(self._h, _DTYPES[dtype], int(rank), ctypes.byref(c), ctypes.byref(g)))
        return c.value, g.value

    def last_apply_kernel(self) -> str:
        """Name of the kernel of the latest apply launch ("split_kernel" or
        "apply_kernel"), or "" before the first one."""
        k = int(self._lib.wp_last_apply_kernel(self._h))
        return {0: "split_kernel", 1: "apply_kernel", 2: "apply_kernel", 3: "apply_kernel"}.get(k, "")

    def last_apply_cluster(self) -> int:
        """Cluster size of the latest clustered apply launch: 4 for a fused
        live call with fewer segments than clusters of 4, else 2 (0 for the
        balanced kernel or before the first launch)."""
        k = int(self._lib.wp_last_apply_kernel(self._h))
        return {1: 2, 2: 2, 3: 4}.get(k, 0)

    def kernel_launches(self) -> int:
        return int(self._lib.wp_kernel_launch_count(self._h))

    # -- scheduler bridge (engine.py:34-42, 64-69) -------------------------------
    # One scheduler tick of Whittle / GWAR / arrival-rate state, held in
    # page-locked memory mapped into the device (wp_write_bridge); the
    # scheduler-aware prefetch policy (scheduler_bridge.PrefetchPolicy) reads
    # it back each tick.
    _BRIDGE_F = ("whittle_scores", "t_remaining_ms", "gwar_pred_next3", "lambda_hat")
    _BRIDGE_U8 = ("burst_active", "promo_eligible", "is_hot", "tile_size_code")

    def write_bridge(self, whittle_scores, t_remaining_ms, gwar_pred_next3, lambda_hat, burst_active,
                     promo_eligible, is_hot, tile_size_code, num_active_adapters, num_segments, step_id,
                     global_load):
        n = int(num_active_adapters)
        if n > 64:
            raise RuntimeError("write_bridge: num_active_adapters exceeds WP_MAX_ADAPTERS")
        b = _lib.WpBridge()
        for name, t in zip(self._BRIDGE_F, (whittle_scores, t_remaining_ms, gwar_pred_next3, lambda_hat)):
            vals = torch.as_tensor(t).reshape(-1)[:n].float().tolist()
            getattr(b, name)[:len(vals)] = vals
        for name, t in zip(self._BRIDGE_U8, (burst_active, promo_eligible, is_hot, tile_size_code)):
            vals = [int(v) & 0xFF for v in torch.as_tensor(t).reshape(-1)[:n].tolist()]
            getattr(b, name)[:len(vals)] = vals
        b.num_active_adapters = n
        b.num_segments = int(num_segments)
        b.step_id = int(step_id)
        b.global_load = float(global_load)
        self._check(self._lib.wp_write_bridge(self._h, ctypes.byref(b)))

    def read_bridge_debug(self):
        b = _lib.WpBridge()
        self._check(self._lib.wp_read_bridge(self._h, ctypes.byref(b)))
        n = int(b.num_active_adapters)
        out = {name: list(getattr(b, name))[:n] for name in self._BRIDGE_F + self._BRIDGE_U8}
        out.update(num_active_adapters=n, num_segments=int(b.num_segments), step_id=int(b.step_id),
                   global_load=float(b.global_load))
        return out

    def read_bridge_via_kernel(self):
        """[whittle_scores..., n, num_segments, step_id], read on the device by a
        kernel through the bridge's device mapping (test_scheduler_bridge.py of
        the reference checks this round trip)."""
        buf = (ctypes.c_float * 67)()
        cnt = ctypes.c_int32()
        self._check(self._lib.wp_read_bridge_kernel(self._h, buf, 67, ctypes.byref(cnt)))
        return [float(v) for v in buf[:cnt.value]]
