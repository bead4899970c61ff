"""Drop-in name for the reference's compiled `opt_attention._C` module
(opt_attention/csrc/opt_attention_ext.cpp:322-337)."""
from directaccesskernel_b200.attention import decode, uses_tma  # noqa: F401
