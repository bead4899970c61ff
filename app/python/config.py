"""Drop-in name for the reference's app/python/config.py."""
from directaccesskernel_b200.config import *  # noqa: F401,F403
from directaccesskernel_b200 import config as _impl

globals().update({k: getattr(_impl, k) for k in dir(_impl) if not k.startswith("__")})
