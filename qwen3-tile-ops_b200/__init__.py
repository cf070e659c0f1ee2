"""q3b200 — B200-native Qwen3 w8a8 forward path behind the reference's
operator API (kernels/*.h of mland2333/qwen3-tile-ops).

``ops``   : one function per reference operator, over CUDA ``MatrixView`` s.
``model`` : the pqwf blob on the device, ``forward_chunk`` and greedy generate.
``_lib``  : the ctypes binding of ``include/q3_ops.h`` (``libq3b200.so``).
``engine``, ``tp``, ``tokenizer``, ``chat``: the serving loop, tensor-parallel
decode, the BPE tokenizer and text in / text out (imported on demand).
"""

from . import _lib, model, ops  # noqa: F401
from ._lib import Q3Error  # noqa: F401
