"""The attention backend registry of the reference (bench/attention.py), with its block-sparse
backends on the sm_100a library.

Same names and signatures as the reference: the adapters ``bsfa``, ``bsdfa`` and ``split_kv``
(q, k, v, mask=None, block_size=None; the mask is ignored and rebuilt from block_size,
bench/attention.py:51-66), ``torch_sdpa`` and ``flex`` (PyTorch's, for comparison),
``BACKENDS``, ``BLOCK_SIZE_BACKENDS``, ``with_nvtx`` and ``install_attention(name, nvtx,
block_size)``, which points ``model.modules.scaled_dot_product_attention`` at the chosen
backend (bench/attention.py:117-127), so the reference's train/train.py and
inference/generate.py run their attention here unchanged.

``install_attention`` also takes ``modules=``: any object whose ``scaled_dot_product_attention``
attribute the model layers call (the reference's ``model.modules`` by default, imported on
first use). ``"custom"`` (the reference's own masked attention) is in ``BACKENDS`` when
``model.modules`` is importable.
"""

from __future__ import annotations

from collections.abc import Callable
from functools import partial

import torch
import torch.nn.functional as F
from torch import Tensor

from kernels.BlockSparseDecodeAttention import block_sparse_decode_attention
from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
from kernels.SplitKVDecodeAttention import split_kv_decode_attention

AttentionFn = Callable[..., Tensor]

FORWARD_RANGE = "attention"
BACKWARD_RANGE = "attention backward"


def torch_sdpa(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None = None) -> Tensor:
    """PyTorch SDPA with the boolean mask as attn_mask (the reference's "sdpa" backend)."""
    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask)


_flex_fn = None
_block_masks: dict = {}


def flex(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None = None) -> Tensor:
    """PyTorch flex_attention with a block mask built once per mask tensor (the reference's
    "flex" backend; compiled on first use)."""
    global _flex_fn
    from torch.nn.attention.flex_attention import create_block_mask, flex_attention
    if _flex_fn is None:
        _flex_fn = torch.compile(flex_attention)
    if mask is None:
        return _flex_fn(q, k, v)
    key = (mask.data_ptr(), tuple(mask.shape))
    if key not in _block_masks:
        def mask_mod(batch, head, q_idx, kv_idx):
            return mask[q_idx, kv_idx]
        _block_masks[key] = create_block_mask(mask_mod, None, None, *mask.shape,
                                              device=mask.device)
    return _flex_fn(q, k, v, block_mask=_block_masks[key])


def bsfa(q, k, v, mask=None, block_size=None):
    """Block-sparse attention forward + backward on the 2n training layout (tcgen05); the
    mask argument is ignored, the BD3-LM mask follows from block_size."""
    return BlockSparseFlashAttention.apply(q, k, v, block_size)


def bsdfa(q, k, v, mask=None, block_size=None):
    """Block-causal decode / prefill attention of the last q_len positions (forward only)."""
    return block_sparse_decode_attention(q, k, v, block_size)


def split_kv(q, k, v, mask=None, block_size=None):
    """Split-KV decode attention (forward only) for decode steps with few queries."""
    return split_kv_decode_attention(q, k, v, block_size)


BACKENDS: dict[str, AttentionFn] = {
    "sdpa": torch_sdpa,
    "flex": flex,
    "bsfa": bsfa,
    "bsdfa": bsdfa,
    "split_kv": split_kv,
}
# backends that ignore the mask and need the block size instead
BLOCK_SIZE_BACKENDS = ("bsfa", "bsdfa", "split_kv")

try:  # the reference's own attention, when its model package is importable
    from model import modules as _ref_modules
    BACKENDS["custom"] = _ref_modules.scaled_dot_product_attention
except ImportError:
    _ref_modules = None


class _OpenRange(torch.autograd.Function):
    """Identity on (q, k, v) that opens the forward NVTX range (and closes the backward's)."""

    @staticmethod
    def forward(ctx, q, k, v):
        torch.cuda.nvtx.range_push(FORWARD_RANGE)
        return q.view_as(q), k.view_as(k), v.view_as(v)

    @staticmethod
    def backward(ctx, *grad_outputs):
        torch.cuda.nvtx.range_pop()
        return grad_outputs


class _CloseRange(torch.autograd.Function):
    """Identity on the output that closes the forward range (and opens the backward's)."""

    @staticmethod
    def forward(ctx, o):
        torch.cuda.nvtx.range_pop()
        return o.view_as(o)

    @staticmethod
    def backward(ctx, *grad_outputs):
        torch.cuda.nvtx.range_push(BACKWARD_RANGE)
        return grad_outputs


def with_nvtx(attention: AttentionFn) -> AttentionFn:
    """Wrap a backend in NVTX ranges for both forward and backward."""

    def annotated(q, k, v, mask=None):
        q, k, v = _OpenRange.apply(q, k, v)
        return _CloseRange.apply(attention(q, k, v, mask))

    return annotated


def install_attention(name: str, nvtx: bool = False, block_size: int | None = None,
                      modules=None) -> None:
    """Route every attention layer through the named backend (KeyError for an unknown name,
    AssertionError when a block-size backend gets no block_size, as the reference)."""
    attention = BACKENDS[name]
    if name in BLOCK_SIZE_BACKENDS:
        assert block_size is not None, f"{name} needs block_size"
        attention = partial(attention, block_size=block_size)
    if modules is None:
        if _ref_modules is None:
            raise ImportError("install_attention needs the reference's model.modules on "
                              "sys.path, or modules= naming the module to patch")
        modules = _ref_modules
    modules.scaled_dot_product_attention = with_nvtx(attention) if nvtx else attention
