"""Drop-in name for the reference's `offload` package (python/offload/__init__.py):
``from offload import runtime`` gives the sm_100a runtime."""
import sys as _sys

from directaccesskernel_b200 import runtime

_sys.modules[__name__ + ".runtime"] = runtime

__all__ = ["runtime"]
