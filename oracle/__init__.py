"""CPU oracle for the direct-access offloading hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's arithmetic (shouxulin/DirectAccessKernel),
used by tests/, by __graft_entry__.smoke() and by bench.py's CPU baseline leg as
the checker.  The product (directaccesskernel_b200) never imports it and has no
CPU path.  Each function cites the reference file:line it restates.  The oracle
is pinned against golden vectors that tests/golden/make_golden.py produced by
running the reference's own Python code (tests/test_oracle_golden.py).
"""
from .attention import (batch_split_decode, decode_attention, decode_attention_grouped, lse_merge,  # noqa: F401
                        paged_decode, paged_gather, split_partials)
from .kv_cache import paged_append, static_cache_update  # noqa: F401
from .linear import gemv_horizontal, horizontal_split, linear, split_horizontal  # noqa: F401
