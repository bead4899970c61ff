"""Tile constants, mirroring app/python/config.py:1-14 of the reference.

TILE_M stays 64 because it sets the granularity of the host/device row split
(split_horizontal); the other values are what the reference's Python code
reads, kept so that callers computing shapes or shared-memory sizes from them
keep working.  BUFFER_SLOTS and TILE_N come from the compiled library, as the
reference reads them from its extension (app/python/config.py:6-8).
"""
from . import runtime

TILE_M = 64
TILE_K = 256
BUFFER_SLOTS = runtime.BUFFER_SLOTS
TILE_N = runtime.TILE_N

TILE_M_MULTICAST = 64
TILE_N_MULTICAST = 256
TILE_K_MULTICAST = 64
BUFFER_SLOTS_MULTICAST = 3
BUFFER_SLOTS_B_MULTICAST = 3
