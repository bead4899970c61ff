"""Drop-in name for the reference's app/python/linear_replacement.py."""
from directaccesskernel_b200.linear_replacement import *  # noqa: F401,F403
from directaccesskernel_b200 import linear_replacement as _impl

globals().update({k: getattr(_impl, k) for k in dir(_impl) if not k.startswith("__")})
