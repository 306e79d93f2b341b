"""Generate the golden fixtures that pin the CPU oracle to the reference itself.

Run once, in a checkout where the reference (tusharsonthalia/diffusion-llm) is importable:

    python tests/golden/make_golden.py /path/to/diffusion-llm

It imports the reference's own ``model/bd3lm.py:block_diff_mask`` (:10-52) and
``model/modules.py:scaled_dot_product_attention`` (:738-771), runs them on seeded
inputs on the CPU, and writes ``tests/golden/golden.npz``; ``kv_cases`` does the same for
``model/modules.py:RoPE`` (:164-240) and ``model/kv_cache.py:KVCache`` (:9-55) into
``tests/golden/golden_kv.npz``; ``sampler_cases`` runs the sampler's denoising step
(``model/subs.py``, ``sample/sampler.py``) into ``tests/golden/golden_sampler.npz``. Inputs are bf16-valued (the
dtype of the CUDA path) and stored as raw bf16 bits; reference outputs are stored in fp32,
exactly as the reference returns them for fp32 inputs. The tests read only the .npz; the
reference is not needed to run them.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

MASK_CASES = [(128, 4), (128, 16), (128, 128), (256, 16), (256, 32), (256, 64),
              (384, 48), (512, 512)]
# (n, block_size): training attention over cat(x_t, x_0), B=1, H=1, D=64
TRAIN_CASES = [(128, 4), (128, 16), (128, 128)]
# (q_len, kv_len, block_size, cached): decode / prefill, B=1, H=2, D=64
DECODE_CASES = [(16, 16, 16, True), (16, 144, 16, True), (16, 528, 16, False),
                (40, 200, 16, False), (96, 96, 16, False)]
D = 64


def bf16_inputs(gen: torch.Generator, shape) -> torch.Tensor:
    return torch.randn(shape, generator=gen).to(torch.bfloat16).float()


def bits(x: torch.Tensor) -> np.ndarray:
    return x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from model.bd3lm import block_diff_mask  # noqa: E402
    from model import modules  # noqa: E402

    sdpa = modules.scaled_dot_product_attention
    out = {}
    for n, bs in MASK_CASES:
        m = block_diff_mask(n, bs).numpy()
        out[f"mask_n{n}_bs{bs}"] = np.packbits(m, axis=-1)

    gen = torch.Generator().manual_seed(1234)
    for n, bs in TRAIN_CASES:
        tag = f"train_n{n}_bs{bs}"
        q, k, v, do = (bf16_inputs(gen, (1, 1, 2 * n, D)) for _ in range(4))
        mask = block_diff_mask(n, bs)
        qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
        o = sdpa(qg, kg, vg, mask)
        dq, dk, dv = torch.autograd.grad(o, (qg, kg, vg), do)
        for name, t in (("q", q), ("k", k), ("v", v), ("do", do)):
            out[f"{tag}_{name}"] = bits(t)
        for name, t in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv)):
            out[f"{tag}_{name}"] = t.detach().numpy().astype(np.float32)

    for q_len, kv_len, bs, cached in DECODE_CASES:
        tag = f"decode_q{q_len}_kv{kv_len}_bs{bs}"
        q = bf16_inputs(gen, (1, 2, q_len, D))
        k = bf16_inputs(gen, (1, 2, kv_len, D))
        v = bf16_inputs(gen, (1, 2, kv_len, D))
        if cached:
            mask = None  # a cached step attends everything (model/bd3lm.py:205)
        else:
            n_big = ((kv_len + bs - 1) // bs) * bs
            full = block_diff_mask(n_big, bs)[n_big:n_big + kv_len, n_big:n_big + kv_len]
            mask = full[kv_len - q_len:]
        o = sdpa(q, k, v, mask)
        for name, t in (("q", q), ("k", k), ("v", v)):
            out[f"{tag}_{name}"] = bits(t)
        out[f"{tag}_o"] = o.numpy().astype(np.float32)

    # block-sparse decode with a per-(batch, head) live-block list (64-token blocks)
    B, H, q_len, kv_len, kvb, bs = 2, 2, 16, 512, 64, 16
    rng = np.random.default_rng(7)
    n_blk = kv_len // kvb
    live = np.zeros((B, H, 3), dtype=np.int32)
    for b in range(B):
        for h in range(H):
            pick = rng.choice(n_blk - 1, size=2, replace=False)
            live[b, h] = sorted(list(pick) + [n_blk - 1])
    q = bf16_inputs(gen, (B, H, q_len, D))
    k = bf16_inputs(gen, (B, H, kv_len, D))
    v = bf16_inputs(gen, (B, H, kv_len, D))
    mask = torch.zeros(B, H, q_len, kv_len, dtype=torch.bool)
    for b in range(B):
        for h in range(H):
            for blk in live[b, h]:
                mask[b, h, :, blk * kvb:(blk + 1) * kvb] = True
    o = sdpa(q, k, v, mask)
    tag = "live"
    for name, t in (("q", q), ("k", k), ("v", v)):
        out[f"{tag}_{name}"] = bits(t)
    out[f"{tag}_blocks"] = live
    out[f"{tag}_o"] = o.numpy().astype(np.float32)

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")
    kv_cases(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_kv.npz"))
    sampler_cases(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_sampler.npz"))


# (dtype, seq, positions) for the reference's RoPE on (1, 2, seq, 64) activations
ROPE_CASES = [("bf16", 5, [0, 3, 7, 20, 63]), ("f16", 4, [1, 2, 3, 4]),
              ("f32", 6, [63, 0, 31, 32, 5, 6])]
_TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def kv_cases(path: str) -> None:
    """RoPE (model/modules.py:164-240) and KVCache (model/kv_cache.py:9-55) fixtures: the
    reference's own tables, rotated activations and concatenated cache contents."""
    from model import modules  # noqa: E402
    from model.kv_cache import KVCache  # noqa: E402

    out = {}
    rope = modules.RoPE(64, 64)
    out["rope_sin"] = rope.sin_table.numpy()
    out["rope_cos"] = rope.cos_table.numpy()
    gen = torch.Generator().manual_seed(99)
    for dt, seq, pos in ROPE_CASES:
        x = (3 * torch.randn((1, 2, seq, 64), generator=gen)).to(_TORCH_DT[dt])
        y = rope(x, torch.tensor(pos))
        out[f"rope_{dt}_x"] = x.float().numpy()
        out[f"rope_{dt}_pos"] = np.array(pos, dtype=np.int64)
        out[f"rope_{dt}_y"] = y.float().numpy()
    # two layers, three appends of 2, 3 and 1 tokens
    cache = KVCache.empty(2)
    for i, s in enumerate((2, 3, 1)):
        for layer in range(2):
            k = torch.randn((1, 2, s, 64), generator=gen)
            v = torch.randn((1, 2, s, 64), generator=gen)
            out[f"kv_append{i}_l{layer}_k"] = k.numpy()
            out[f"kv_append{i}_l{layer}_v"] = v.numpy()
            cache.append(layer, k, v)
    for layer in range(2):
        k, v = cache.get(layer)
        out[f"kv_final_l{layer}_k"] = k.numpy()
        out[f"kv_final_l{layer}_v"] = v.numpy()
    out["kv_length"] = np.array(cache.length, dtype=np.int64)
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")



def sampler_cases(path: str) -> None:
    """One ancestral step of sample/sampler.py:100-122 through the reference's own
    subs_parameterization (model/subs.py:11-43) and sample_categorical (sample/sampler.py:11-34)
    on seeded logits; the step's uniforms are replayed by reseeding torch's generator before
    torch.rand, which sample_categorical's torch.rand_like draws from identically."""
    from model.subs import subs_parameterization  # noqa: E402
    from sample.sampler import sample_categorical  # noqa: E402

    out = {}
    gen = torch.Generator().manual_seed(2024)
    B, S, V, mask = 2, 8, 1000, 999
    # (fp16 logits make the reference's SUBS raise: -1e6 does not fit in fp16)
    for dt, (t, s) in (("f32", (0.75, 0.5)), ("bf16", (1.0, 0.9375)), ("f32", (0.5, 0.0))):
        tag = dt if dt == "bf16" or s else "f32_last"
        logits = (3 * torch.randn((B, S, V), generator=gen)).to(_TORCH_DT[dt])
        xt = torch.randint(0, V - 1, (B, S), generator=gen)
        xt[torch.rand((B, S), generator=gen) < 0.6] = mask
        log_probs = subs_parameterization(logits, xt, mask)
        q = torch.exp(log_probs).double() * (1 - s / t)
        q[..., mask] = s / t
        torch.manual_seed(77)
        new = sample_categorical(q)
        torch.manual_seed(77)
        u = torch.rand(q.shape, dtype=torch.float64)
        nxt = torch.where(xt != mask, xt, new)
        out[f"{tag}_logits"] = logits.float().numpy()
        out[f"{tag}_xt"] = xt.numpy()
        out[f"{tag}_ts"] = np.array([t, s], dtype=np.float64)
        out[f"{tag}_u"] = u.numpy()
        out[f"{tag}_q"] = q.numpy()
        out[f"{tag}_next"] = nxt.numpy()
    out["mask_index"] = np.array(mask, dtype=np.int64)
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../diffusion-llm")
