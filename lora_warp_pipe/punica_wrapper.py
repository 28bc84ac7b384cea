"""Alias of adapterslotsplusplus_b200.punica_wrapper (reference module path)."""

from adapterslotsplusplus_b200.punica_wrapper import *  # noqa: F401,F403
