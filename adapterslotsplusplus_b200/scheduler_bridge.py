"""Host-side adapters between the AdapterSlots scheduler and build_segments.

Mirrors the two pieces of lora_warp_pipe/scheduler_bridge.py that feed the
apply path: AdapterIdMap (:33-60, string ids -> dense int ids in first-seen
order) and segments_to_warp_pipe (:82-102, scheduler segments ->
(sorted_adapter_ids, seg_offsets)). The Whittle/GWAR bridge itself is
scheduler metadata that no compute kernel reads and is not part of this build.
"""

from typing import Dict, List


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
