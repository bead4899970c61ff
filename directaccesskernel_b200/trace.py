"""Optional NVTX ranges around this library's launches, for nsys timelines and
`ncu --nvtx` filters.  The reference left such ranges commented out in its
linear forward (app/python/layers/linearLayer.py:120,124).

With DAK_B200_NVTX=1 in the environment at import time, every decorated entry
point pushes an NVTX range named ``dak.<function>`` for the duration of the
call (the host-side launch; inside a CUDA graph capture the range marks the
capture).  Otherwise the decorator returns the function itself, so tracing off
costs nothing.
"""
from __future__ import annotations

import functools
import os

NVTX = os.environ.get("DAK_B200_NVTX", "") not in ("", "0")


def traced(fn):
    if not NVTX:
        return fn
    import torch

    name = f"dak.{fn.__name__}"

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        torch.cuda.nvtx.range_push(name)
        try:
            return fn(*args, **kwargs)
        finally:
            torch.cuda.nvtx.range_pop()

    return wrapper
