"""Alias of adapterslotsplusplus_b200.config (reference module path)."""

from adapterslotsplusplus_b200.config import *  # noqa: F401,F403
