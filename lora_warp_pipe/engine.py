"""Alias of adapterslotsplusplus_b200.engine (reference module path)."""

from adapterslotsplusplus_b200.engine import *  # noqa: F401,F403
