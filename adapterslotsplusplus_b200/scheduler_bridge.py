"""Host-side adapters between the AdapterSlots scheduler and the apply path.

Restates lora_warp_pipe/scheduler_bridge.py of the reference, whose
interfaces the drop-in keeps: AdapterIdMap (:33-60, string ids -> dense int
ids in first-seen order), GwarHistory (:63-80), segments_to_warp_pipe
(:82-102, scheduler segments -> (sorted_adapter_ids, seg_offsets)) and
SchedulerBridge (:105-184, one scheduler tick into the engine's bridge).
PrefetchPolicy is new: it turns the bridge's signals into prefetch /
release calls on the staging slots or an AdapterPool (scheduler-aware
prefetch), which the reference leaves unwired.
"""

from typing import Dict, List, Optional, Sequence

import numpy as np
import torch


class AdapterIdMap:
    """Bijection between string adapter ids and small int ids, assigned in
    first-seen order and never reused."""

    def __init__(self):
        self._str_to_int: Dict[str, int] = {}
        self._int_to_str: List[str] = []

    def get_or_assign(self, adapter_id: str) -> int:
        if adapter_id not in self._str_to_int:
            self._str_to_int[adapter_id] = len(self._int_to_str)
            self._int_to_str.append(adapter_id)
        return self._str_to_int[adapter_id]

    def to_int(self, adapter_id: str) -> int:
        return self._str_to_int[adapter_id]

    def ordered_ids(self) -> List[str]:
        return list(self._int_to_str)

    def __len__(self) -> int:
        return len(self._int_to_str)


def segments_to_warp_pipe(segments, id_map: AdapterIdMap):
    """Scheduler segments (objects with ``adapter_id`` and ``segment_size``, in
    dispatch order, tokens already adapter-sorted) -> the (sorted_adapter_ids,
    seg_offsets) pair build_segments takes; offsets are the running sum of
    segment sizes."""
    ids: List[int] = []
    offsets: List[int] = [0]
    for seg in segments:
        ids.append(id_map.get_or_assign(seg.adapter_id))
        offsets.append(offsets[-1] + int(seg.segment_size))
    return ids, offsets


class GwarHistory:
    """EWMA over successive GWAR readings per adapter (the reference's
    smoother for the bridge's gwar_pred_next3 field,
    lora_warp_pipe/scheduler_bridge.py:63-80)."""

    def __init__(self, alpha: float = 0.3):
        self.alpha = alpha
        self._ewma: Dict[str, float] = {}

    def update(self, adapter_id: str, gwar_value: float) -> float:
        prev = self._ewma.get(adapter_id, gwar_value)
        new = self.alpha * gwar_value + (1.0 - self.alpha) * prev
        self._ewma[adapter_id] = new
        return new

    def get(self, adapter_id: str) -> float:
        return self._ewma.get(adapter_id, 0.0)


class SchedulerBridge:
    """One scheduler tick of AdapterSlots state into the engine's bridge
    (lora_warp_pipe/scheduler_bridge.py:105-184 of the reference): Whittle
    indices from a dispatcher (``compute_indices(fill_fracs, lambda_est)``),
    arrival rates from an estimator (``get_rate(id)``), smoothed GWAR
    readings, and merge eligibility (``is_merged(id)``), for the adapters of
    ``id_map`` in int-id order. The scheduler objects are duck-typed."""

    def __init__(self, engine, id_map: AdapterIdMap):
        self._engine = engine
        self._id_map = id_map
        self._gwar_history = GwarHistory()
        self._step_id = 0

    def write(self, num_segments: int, whittle_dispatcher=None, fill_fracs: Optional[Dict[str, float]] = None,
              lambda_est: Optional[Dict[str, float]] = None, estimator=None,
              gwar_readings: Optional[Dict[str, float]] = None, mwc=None, global_load: float = 0.0,
              queued: Optional[Sequence[str]] = None) -> None:
        ordered = self._id_map.ordered_ids()
        n = len(ordered)
        if n == 0:
            self._step_id += 1
            return
        whittle = np.zeros(n, dtype=np.float32)
        if whittle_dispatcher is not None and fill_fracs is not None and lambda_est is not None:
            idx = whittle_dispatcher.compute_indices(fill_fracs, lambda_est)
            whittle[:] = [idx.get(a, 0.0) for a in ordered]
        lam = np.zeros(n, dtype=np.float32)
        if estimator is not None:
            lam[:] = [estimator.get_rate(a) for a in ordered]
        gwar = np.zeros(n, dtype=np.float32)
        for i, a in enumerate(ordered):
            if gwar_readings is not None and a in gwar_readings:
                self._gwar_history.update(a, gwar_readings[a])
            gwar[i] = self._gwar_history.get(a)
        promo = np.zeros(n, dtype=np.uint8)
        if mwc is not None:
            promo[:] = [1 if mwc.is_merged(a) else 0 for a in ordered]
        hot = np.zeros(n, dtype=np.uint8)  # requests admitted but not yet scheduled
        if queued is not None:
            qs = set(queued)
            hot[:] = [1 if a in qs else 0 for a in ordered]
        tile = np.zeros(n, dtype=np.uint8)
        tile[gwar > 0.6] = 1
        tile[gwar > 0.85] = 2
        zeros_f = np.zeros(n, dtype=np.float32)
        zeros_u = np.zeros(n, dtype=np.uint8)
        self._engine.write_bridge(torch.from_numpy(whittle), torch.from_numpy(zeros_f), torch.from_numpy(gwar),
                                  torch.from_numpy(lam), torch.from_numpy(zeros_u), torch.from_numpy(promo),
                                  torch.from_numpy(hot), torch.from_numpy(tile), n, num_segments, self._step_id,
                                  global_load)
        self._step_id += 1


class PrefetchPolicy:
    """Scheduler-aware prefetch: turns one tick of bridge signals into
    prefetch / release calls on a staging target (WarpPipeEngine's staging
    slots or an AdapterPool: anything with prefetch(id) -> slot or -1,
    is_prefetch_ready(id) and release_prefetch(id)).

    Priority of adapter i (its int id) for the next step:
        w_hot * is_hot[i] + w_whittle * whittle_scores[i]
        + w_lambda * lambda_hat[i] * horizon_s + w_gwar * gwar_pred_next3[i]
    is_hot marks requests already admitted, so they win; the arrival rate
    over the prefetch horizon ranks the rest. Each tick keeps the `budget`
    highest-priority adapters above `min_priority` prefetched (held) and
    releases held adapters that dropped out (they stay resident, evictable);
    `protected` ids (the step in flight) are never released by the policy."""

    def __init__(self, target, budget: int, min_priority: float = 0.05, horizon_s: float = 0.01,
                 w_hot: float = 10.0, w_whittle: float = 1.0, w_lambda: float = 1.0, w_gwar: float = 0.5):
        self.target = target
        self.budget = int(budget)
        self.min_priority = float(min_priority)
        self.horizon_s = float(horizon_s)
        self.w = (w_hot, w_whittle, w_lambda, w_gwar)
        self.held: Dict[int, int] = {}  # id -> slot
        self.issued = 0
        self.refused = 0

    def priorities(self, bridge: dict) -> Dict[int, float]:
        n = int(bridge.get("num_active_adapters", 0))
        wh, ww, wl, wg = self.w
        out = {}
        for i in range(n):
            p = (wh * float(bridge["is_hot"][i]) + ww * float(bridge["whittle_scores"][i]) +
                 wl * float(bridge["lambda_hat"][i]) * self.horizon_s + wg * float(bridge["gwar_pred_next3"][i]))
            out[i] = p
        return out

    def tick(self, bridge: dict, protected: Sequence[int] = ()) -> dict:
        pr = self.priorities(bridge)
        ranked = [i for i, p in sorted(pr.items(), key=lambda kv: (-kv[1], kv[0])) if p >= self.min_priority]
        want = ranked[:self.budget]
        keep = set(want) | set(int(i) for i in protected)
        released = []
        for i in list(self.held):
            if i not in keep:
                self.target.release_prefetch(i)
                del self.held[i]
                released.append(i)
        prefetched = []
        for i in want:
            if i in self.held:
                continue
            slot = self.target.prefetch(i)
            if slot < 0:
                self.refused += 1
                break  # no slot free: the rest would be refused too
            self.held[i] = slot
            self.issued += 1
            prefetched.append(i)
        return {"prefetched": prefetched, "released": released, "held": sorted(self.held)}

    def tick_from_engine(self, engine, protected: Sequence[int] = ()) -> dict:
        """tick() on the bridge the engine holds (written by SchedulerBridge)."""
        return self.tick(engine.read_bridge_debug(), protected)
