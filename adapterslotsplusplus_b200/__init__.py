"""B200-native grouped multi-LoRA apply (drop-in for the WarpPipeEngine of
vac014/AdapterSlotsPlusPlus). Compute runs in libwp_b200.so (sm_100a)."""

from .config import WarpPipeConfig
from .engine import WarpPipeEngine
from .pool import AdapterPool
from .scheduler_bridge import AdapterIdMap, segments_to_warp_pipe

__all__ = ["WarpPipeConfig", "WarpPipeEngine", "AdapterPool", "AdapterIdMap", "segments_to_warp_pipe"]
