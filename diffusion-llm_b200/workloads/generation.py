"""BD3-LM generation with the stand-in backbone: the reference's sampling loop
(sample/sampler.py:69-122: per block, ``steps`` ancestral steps of the cached forward and the
SUBS sampler, then a commit of the finished block's K/V) in two implementations.

``CachedGeneration`` runs it on this library: per layer the fused QKV/RoPE cache write into
preallocated caches (rows from device positions) and the split-KV decode over the cache
(key count on the device); the fused sampler step with (t, s) and (seed, offset) on the
device; the commit is the same forward without the LM head. One whole block (``steps``
sampler steps, the commit, copying the block out and advancing the device counters) is
captured once as a CUDA graph, so a run is one graph replay per block.

``ReferenceGeneration`` is the reference's flow in PyTorch ops, eager: RoPE as elementwise
ops, a cache that concatenates (model/kv_cache.py:42-55, model/modules.py:410-417),
``F.scaled_dot_product_attention`` without a mask over cache + block, SUBS
(model/subs.py:11-43) with the reference's log_softmax (model/modules.py:791-799), float64
weights and Gumbel-max (sample/sampler.py:11-34, 114-122), and a commit that runs the whole
backbone with store=True (model/bd3lm.py:210-233).

Both take a ``Backbone`` (workloads/backbone.py) in bf16; tokens/s = batch * length / time.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from bd3attn import ops
from bd3attn.sampler import subs_sample_step_dev
from workloads.backbone import Backbone, rope, rope_tables, use_attention

EPS = 1e-10
NEG_INF = -1e6


class CachedGeneration:
    """Generation through the in-place KV cache, split-KV decode and fused sampler, one CUDA
    graph replay per block."""

    def __init__(self, model: Backbone, batch: int, n_blocks: int, steps: int = 16,
                 seed: int = 0, use_graph: bool = True):
        self.m, self.B, self.n_blocks, self.steps = model, batch, n_blocks, steps
        self.bs, self.H = model.block_size, model.n_heads
        d = model.embed.embedding_dim
        self.Dh = d // self.H
        self.L = n_blocks * self.bs
        dev = model.head.weight.device
        dt = model.head.weight.dtype
        cos, sin = rope_tables(self.Dh, self.L, dev)
        self.cos, self.sin = cos.contiguous(), sin.contiguous()
        self.kc = [torch.zeros(batch, self.H, self.L, self.Dh, dtype=dt, device=dev)
                   for _ in model.layers]
        self.vc = [torch.zeros_like(k) for k in self.kc]
        self.q_buf = [torch.empty(batch, self.H, self.bs, self.Dh, dtype=dt, device=dev)
                      for _ in model.layers]
        self.block = torch.empty(batch, self.bs, dtype=torch.int64, device=dev)
        self.out = torch.empty(batch, self.L, dtype=torch.int64, device=dev)
        self.pos = torch.empty(self.bs, dtype=torch.int64, device=dev)
        self.kv_len = torch.empty(1, dtype=torch.int32, device=dev)
        self.ts = torch.tensor([[1 - i / steps, 1 - (i + 1) / steps] for i in range(steps)],
                               dtype=torch.float64, device=dev)
        self.rng = torch.empty(steps, 2, dtype=torch.int64, device=dev)
        self.seed, self.use_graph, self.graph = seed, use_graph, None

    def _reset(self):
        self.pos.copy_(torch.arange(self.bs))
        self.kv_len.fill_(self.bs)
        self.rng[:, 0] = self.seed
        self.rng[:, 1].copy_(torch.arange(self.steps))

    def forward_block(self, with_logits: bool = True):
        """The current block through every layer: its K/V written at the cache rows of its
        positions, its queries attending the committed cache and the block itself."""
        m, B, bs = self.m, self.B, self.bs
        x = m.embed(self.block)
        for i, layer in enumerate(m.layers):
            qkv = layer.qkv(layer.norm1(x))
            q = ops.qkv_rope_cache_raw(qkv, self.H, self.cos, self.sin, self.kc[i], self.vc[i],
                                       -1, positions=self.pos, q_out=self.q_buf[i])
            o = ops.decode_raw(q, self.kc[i], self.vc[i], bs, kv_len_dev=self.kv_len)
            x = x + layer.out(o.transpose(1, 2).reshape(B, bs, -1))
            x = x + layer.down(F.gelu(layer.up(layer.norm2(x)), approximate="tanh"))
        return m.head(m.norm(x)) if with_logits else None

    def _one_block(self):
        self.block.fill_(self.m.mask_index)
        for i in range(self.steps):
            logits = self.forward_block()
            subs_sample_step_dev(logits, self.block, self.m.mask_index, self.ts[i], self.rng[i],
                                 out=self.block)
        self.forward_block(with_logits=False)  # commit: the finished block's K/V
        self.out.index_copy_(1, self.pos, self.block)
        self.pos += self.bs
        self.kv_len += self.bs
        self.rng[:, 1] += self.steps

    @torch.no_grad()
    def run(self) -> torch.Tensor:
        """Generate (batch, n_blocks * block_size) tokens; returns the output buffer."""
        if self.use_graph and self.graph is None:
            self._reset()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._one_block()  # first calls (library set-up) outside the capture
            torch.cuda.current_stream().wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._one_block()
        self._reset()
        for _ in range(self.n_blocks):
            if self.use_graph:
                self.graph.replay()
            else:
                self._one_block()
        return self.out


def _log_softmax(x: torch.Tensor) -> torch.Tensor:
    """The reference's log_softmax (model/modules.py:791-799): five elementwise ops."""
    shifted = x - x.amax(dim=-1, keepdim=True)
    return shifted - torch.log(torch.exp(shifted).sum(dim=-1, keepdim=True))


def subs_log_probs(logits: torch.Tensor, block: torch.Tensor, mask_index: int) -> torch.Tensor:
    """SUBS (model/subs.py:11-43): -1e6 on the [MASK] logit, log_softmax, and one-hot rows
    for the tokens that are already unmasked."""
    bias = torch.zeros(logits.shape[-1], device=logits.device, dtype=logits.dtype)
    bias[mask_index] = NEG_INF
    log_probs = _log_softmax(logits + bias)
    carry = torch.full_like(log_probs, NEG_INF).scatter(-1, block.unsqueeze(-1), 0.0)
    return torch.where((block != mask_index).unsqueeze(-1), carry, log_probs)


def reference_step(logits: torch.Tensor, block: torch.Tensor, mask_index: int, t: float,
                   s: float, generator: torch.Generator | None) -> torch.Tensor:
    """The reference's ancestral update (sample/sampler.py:100-122, 11-34): float64 weights,
    Gumbel-max over float64 uniforms, and the where() that keeps unmasked tokens."""
    q = torch.exp(subs_log_probs(logits, block, mask_index)).double() * (1 - s / t)
    q[..., mask_index] = s / t
    u = torch.rand(q.shape, dtype=torch.float64, device=q.device, generator=generator)
    new = torch.argmax(q / (EPS - torch.log(u + EPS)), dim=-1)
    return torch.where(block != mask_index, block, new)


class ReferenceGeneration:
    """The reference's cached sampling flow in eager PyTorch ops (see the module docstring)."""

    def __init__(self, model: Backbone, batch: int, n_blocks: int, steps: int = 16,
                 generator: torch.Generator | None = None):
        self.m, self.B, self.n_blocks, self.steps = model, batch, n_blocks, steps
        self.bs, self.H = model.block_size, model.n_heads
        self.L = n_blocks * self.bs
        dev = model.head.weight.device
        cos, sin = rope_tables(model.embed.embedding_dim // self.H, self.L, dev)
        self.cos, self.sin = cos, sin
        self.gen = generator

    def _forward(self, block, positions, cache, store):
        m, B, bs = self.m, self.B, self.bs
        cos, sin = self.cos[positions], self.sin[positions]
        x = m.embed(block)
        for i, layer in enumerate(m.layers):
            q, k, v = layer.qkv(layer.norm1(x)).view(B, bs, 3, self.H, -1).permute(2, 0, 3, 1, 4)
            q, k = rope(q, cos, sin), rope(k, cos, sin)
            k_all, v_all = k, v
            if cache[i] is not None:
                k_all = torch.cat([cache[i][0], k], dim=-2)
                v_all = torch.cat([cache[i][1], v], dim=-2)
            if store:
                cache[i] = (k_all, v_all)
            o = F.scaled_dot_product_attention(q, k_all, v_all)
            x = x + layer.out(o.transpose(1, 2).reshape(B, bs, -1))
            x = x + layer.down(F.gelu(layer.up(layer.norm2(x)), approximate="tanh"))
        return m.head(m.norm(x))

    @torch.no_grad()
    def run(self) -> torch.Tensor:
        mask_index = self.m.mask_index
        cache = [None] * len(self.m.layers)
        blocks = []
        for b in range(self.n_blocks):
            positions = torch.arange(b * self.bs, (b + 1) * self.bs, device=self.cos.device)
            block = torch.full((self.B, self.bs), mask_index, dtype=torch.int64,
                               device=self.cos.device)
            for i in range(self.steps):
                t, s = 1 - i / self.steps, 1 - (i + 1) / self.steps
                logits = self._forward(block, positions, cache, False)
                block = reference_step(logits, block, mask_index, t, s, self.gen)
            self._forward(block, positions, cache, True)  # commit (the backbone with store)
            blocks.append(block)
        return torch.cat(blocks, dim=-1)


class MDLMGeneration:
    """The MDLM variant of the sampling loop (block size = the whole sequence, no cache):
    every step re-encodes all ``length`` tokens with bidirectional attention and updates
    the masked ones. With ``use_library`` the layers' attention is the block-causal prefill
    kernel (``bsdfa`` with block_size = length, so every key is visible) and the step is
    the fused sampler; otherwise PyTorch's ``F.scaled_dot_product_attention`` and the
    reference's sampler ops (SUBS, float64 weights, Gumbel-max, where). Eager: at 1024
    tokens per sequence each step is long enough that launches do not matter."""

    def __init__(self, model: Backbone, batch: int, length: int, steps: int = 64,
                 use_library: bool = True, seed: int = 0):
        self.m, self.B, self.L, self.steps = model, batch, length, steps
        self.use_library, self.seed = use_library, seed
        dev = model.head.weight.device
        cos, sin = rope_tables(model.embed.embedding_dim // model.n_heads, length, dev)
        self.cos, self.sin = cos, sin

    @torch.no_grad()
    def run(self) -> torch.Tensor:
        from bd3attn.sampler import subs_sample_step
        use_attention("bsdfa" if self.use_library else "sdpa", block_size=self.L)
        mask_index = self.m.mask_index
        dev = self.cos.device
        x = torch.full((self.B, self.L), mask_index, dtype=torch.int64, device=dev)
        gen_cpu = torch.Generator().manual_seed(self.seed)
        gen_dev = torch.Generator(device=dev).manual_seed(self.seed)
        for i in range(self.steps):
            t, s = 1 - i / self.steps, 1 - (i + 1) / self.steps
            logits = self.m.encode(x, None, self.cos, self.sin)
            if self.use_library:
                subs_sample_step(logits, x, mask_index, t, s, generator=gen_cpu, out=x)
            else:
                x = reference_step(logits, x, mask_index, t, s, gen_dev)
        return x
