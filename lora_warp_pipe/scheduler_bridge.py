"""Alias of adapterslotsplusplus_b200.scheduler_bridge (reference module path)."""

from adapterslotsplusplus_b200.scheduler_bridge import *  # noqa: F401,F403
