"""hsd_b200: the sparse MoE down-projection hot path of mlx-heimr-sparse-down on B200.

The operators keep the reference's names, argument order and keyword defaults
(hsd/layout.py, hsd/decode.py, hsd/prefill.py, hsd/mamba.py) and run hand-written sm_100a
CUDA kernels from libhsd.so through its C ABI (include/hsd.h). There is no CPU path:
calling an operator without the library or on CPU tensors raises.
"""
from ._lib import HsdError, device_status  # noqa: F401
from .decode import live_rows, sparse_down  # noqa: F401
from .layout import nibble_transpose, swap_last2, to_neuron_major  # noqa: F401
from .mamba import mamba_rollback, mamba_verify  # noqa: F401
from .prefill import build_tiles, build_union, sparse_down_prefill  # noqa: F401

__version__ = "0.1.0"
