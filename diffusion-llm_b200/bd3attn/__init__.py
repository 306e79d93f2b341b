"""B200 (sm_100a) BD3-LM attention: the C-ABI library and its PyTorch wrappers.

``bd3attn.ops`` holds one tensor-level wrapper per C entry point; the drop-in modules with
the reference's file names and call signatures live beside this package in ``kernels/``.
"""

from bd3attn import ops  # noqa: F401
from bd3attn._lib import LIB, LIB_PATH, BD3Error  # noqa: F401
