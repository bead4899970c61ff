"""B200-native (sm_100a) direct-access offloading: split-tier linear layers
and split-KV decode attention whose weights / KV pages partly live in pinned
host memory and are streamed by the kernels straight into shared memory.

Every compute module (runtime, layers, attention, ...) loads libdak_b200.so
through ``_lib`` on import and raises ImportError when it is missing: the CUDA
kernels are the only compute path.  This file imports nothing so that the
build step (``python -m directaccesskernel_b200.build``) can run first.
"""

__all__ = ["runtime", "layers", "attention", "placement", "linear_replacement", "utils", "config"]
