"""Drop-in module name of the reference package: ``from lora_warp_pipe import
WarpPipeEngine`` resolves to the B200 engine of adapterslotsplusplus_b200."""

from adapterslotsplusplus_b200 import AdapterIdMap, WarpPipeConfig, WarpPipeEngine, segments_to_warp_pipe

__all__ = ["WarpPipeConfig", "WarpPipeEngine", "AdapterIdMap", "segments_to_warp_pipe"]
