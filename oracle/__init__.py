"""CPU oracle for the BD3-LM attention hot path.

TEST INFRASTRUCTURE ONLY. Nothing on the product path imports this package: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and
``--impl reference`` arm) use it, and only as the checker or as the timed CPU baseline.
The CUDA library and its Python wrappers fail loudly instead of falling back to it.

The restatement follows the reference (tusharsonthalia/diffusion-llm) function by
function; every function cites the file:line it restates. It is pinned against the
reference itself by ``tests/golden/*.npz``, which ``tests/golden/make_golden.py``
produced by importing the reference's ``model/modules.py`` and ``model/bd3lm.py``.
"""

from oracle.attention import (  # noqa: F401
    attention,
    attention_grads,
    block_causal_mask,
    block_diff_mask,
    live_block_mask,
    lse_merge,
)
from oracle import tile_ranges  # noqa: F401
