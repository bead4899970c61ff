"""Drop-in name for opt_attention/opt_attention/interface.py."""
from directaccesskernel_b200.attention import _pop_host_kv_kwargs, opt_attention_forward, register  # noqa: F401
