"""Drop-in name for the reference's `split_attention` package (opt_attention/opt_attention/__init__.py):
the sm_100a split-KV decode attention hook."""
from directaccesskernel_b200.attention import decode_paged, opt_attention_forward, register

from . import _C  # noqa: F401

__all__ = ["opt_attention_forward", "register", "decode_paged"]
