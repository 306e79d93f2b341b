"""The reference's own callers, unchanged, run against this repository's ``kernels`` package.

Run as a subprocess by tests/test_reference_callers.py and by bench.py (the reference's
training loop on both attention backends), one case per call:

    python baseline/ref_callers.py <case> [json arguments]

The import path is this repository's package root (``kernels``, ``bd3attn``) followed by the
installed reference (baseline/_ref: ``model``, ``bench``, ``sample``, ``inference``,
``train``). Its ``kernels`` directory is a namespace package, so the regular package here
wins: the reference's bench/attention.py, model/bd3lm.py, sample/sampler.py,
inference/generate.py and train/train.py import the sm_100a kernels by their reference
names. Each case prints one JSON line with what it measured; the test asserts on it.

Cases:
  registry        (CPU) the reference's registry binds to this package's kernels
  train           BD3LM forward + backward, "bsfa" against the reference's "custom"
  sample          sample_bd3lm with the KV cache, "split_kv" against "custom"
  compile         the compile rungs of inference/generate.py (backbone.compile(dynamic=True))
  attention_bench bench/attention_bench.py's backends() and time_fwd_bwd() with "bsfa"
  train_loop      train/train.py's main() with --attn bsfa and --attn custom
"""

from __future__ import annotations

import copy
import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
PKG = os.path.join(REPO, "diffusion-llm_b200")
REF = os.path.join(HERE, "_ref")

# this package first, then the installed reference; nothing else from the repository root
# (its bench.py would shadow the reference's bench package)
sys.path[:] = [PKG, REF] + [p for p in sys.path if p not in (HERE, REPO, "")]

import torch  # noqa: E402


def _under(path: str, root: str) -> bool:
    return os.path.realpath(path).startswith(os.path.realpath(root) + os.sep)


def _small_bd3lm(n: int = 256, block_size: int = 16, vocab: int = 101, seed: int = 0):
    """A small BD3LM on the GPU, head_dim 64. The reference zero-initialises the adaLN
    modulations and the LM head (constant logits); those are drawn from the seed instead,
    so attention changes the outputs."""
    from model.bd3lm import BD3LM
    torch.manual_seed(seed)
    model = BD3LM(vocab, n, 128, 2, 2, 256, 32, block_size, device=torch.device("cuda"))
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    with torch.no_grad():
        for p in model.parameters():
            if not p.any():
                p.normal_(0.0, 0.05, generator=g)
    return model


def case_registry(_args) -> dict:
    import bench.attention as ba
    import bench.attention_bench as bab
    import bench.decode_ncu  # noqa: F401
    import inference.generate as gen
    import train.train  # noqa: F401
    from model import modules
    out = {"registry_file": os.path.relpath(ba.__file__, REPO),
           "backends": sorted(ba.BACKENDS)}
    assert _under(ba.__file__, REF), ba.__file__
    for name, fn in (("BlockSparseFlashAttention", ba.BlockSparseFlashAttention.forward),
                     ("block_sparse_decode_attention", ba.block_sparse_decode_attention),
                     ("split_kv_decode_attention", ba.split_kv_decode_attention),
                     ("attention_bench.BlockSparseFlashAttention",
                      bab.BlockSparseFlashAttention.forward)):
        assert _under(fn.__code__.co_filename, PKG), (name, fn.__code__.co_filename)
    for rung in ("split_kv", "bsdfa", "bsfa"):
        ba.install_attention(rung, block_size=16)
        installed = modules.scaled_dot_product_attention
        assert installed.func is ba.BACKENDS[rung] and installed.keywords == {"block_size": 16}
    ba.install_attention("custom")
    assert gen.METHODS.keys() == {"baseline", "bf16", "compile", "kv_cache", "split_kv"}
    out["kernels_from"] = os.path.relpath(
        os.path.dirname(ba.BlockSparseFlashAttention.forward.__code__.co_filename), REPO)
    return out


def case_train(_args) -> dict:
    """Logits and parameter gradients of BD3LM.forward + bd3lm_loss under bf16 autocast."""
    import bench.attention as ba
    from train.bd3lm_loss import bd3lm_loss
    base = _small_bd3lm()
    g = torch.Generator().manual_seed(2)
    x0 = torch.randint(0, 100, (2, base.max_seq_len), generator=g).cuda()
    res = {}
    for name in ("custom", "bsfa"):
        model = copy.deepcopy(base).train()
        ba.install_attention(name, block_size=base.block_size)
        torch.manual_seed(3)  # the loss draws the per-block times and the masking
        with torch.autocast("cuda", torch.bfloat16):
            loss = bd3lm_loss(model, x0)
        loss.backward()
        torch.manual_seed(3)
        with torch.no_grad(), torch.autocast("cuda", torch.bfloat16):
            xt = torch.where(torch.rand(x0.shape, device="cuda") < 0.5, model.mask_index, x0)
            lp = model(xt, x0).float()
        grads = torch.cat([p.grad.float().flatten() for p in model.parameters()])
        res[name] = (loss.item(), lp, grads)
    (lc, lpc, gc), (lb, lpb, gb) = res["custom"], res["bsfa"]
    finite = lpc > -1e5
    probs_c, probs_b = lpc.exp(), lpb.exp()
    return {"loss_custom": lc, "loss_bsfa": lb,
            "loss_rel": abs(lb - lc) / abs(lc),
            "logprob_max_abs": (lpb - lpc)[finite].abs().max().item(),
            "prob_max_abs": (probs_b - probs_c).abs().max().item(),
            "grad_rel_norm": ((gb - gc).norm() / gc.norm()).item(),
            "masked_equal": bool(torch.equal(lpc <= -1e5, lpb <= -1e5))}


def _teacher_forced(model, tokens, backend: str, cached: bool) -> torch.Tensor:
    """SUBS log-probs of every block of ``tokens`` with half of the block masked, given the
    finished blocks before it: through the KV cache (cached_block_logprobs, commit_block)
    or by re-encoding (block_logprobs)."""
    import bench.attention as ba
    from model.kv_cache import KVCache
    ba.install_attention(backend, block_size=model.block_size)
    bs = model.block_size
    hide = torch.arange(bs, device=tokens.device) % 2 == 0
    cache = KVCache.empty(model.n_layers)
    out = []
    with torch.no_grad(), torch.autocast("cuda", torch.bfloat16):
        for j in range(tokens.shape[1] // bs):
            blk = tokens[:, j * bs:(j + 1) * bs]
            noisy = torch.where(hide, model.mask_index, blk)
            if cached:
                out.append(model.cached_block_logprobs(noisy, cache).float())
                model.commit_block(blk, cache)
            else:
                x_accum = torch.cat([tokens[:, :j * bs], noisy], dim=-1)
                out.append(model.block_logprobs(x_accum).float())
    return torch.cat(out, dim=1)


def case_sample(_args) -> dict:
    """sample_bd3lm(kv_cache=True) with "split_kv" and with "custom" from the same seed, and
    both backends teacher-forced over the "custom" run's tokens (cached, and uncached with
    "bsdfa" against "custom")."""
    import bench.attention as ba
    from sample.sampler import sample_bd3lm
    model = _small_bd3lm().eval()
    runs = {}
    for name in ("custom", "split_kv"):
        ba.install_attention(name, block_size=model.block_size)
        torch.manual_seed(4)
        with torch.autocast("cuda", torch.bfloat16):
            runs[name] = sample_bd3lm(model, 2, 4, 4, kv_cache=True)
    tc, ts = runs["custom"], runs["split_kv"]
    lp_c = _teacher_forced(model, tc, "custom", cached=True)
    lp_s = _teacher_forced(model, tc, "split_kv", cached=True)
    lp_cu = _teacher_forced(model, tc, "custom", cached=False)
    lp_bu = _teacher_forced(model, tc, "bsdfa", cached=False)
    fin = lp_c > -1e5
    return {"tokens_shape": list(ts.shape),
            "no_mask_left": bool((ts != model.mask_index).all()),
            "token_agreement": (tc == ts).float().mean().item(),
            "cached_logprob_max_abs": (lp_s - lp_c)[fin].abs().max().item(),
            "uncached_logprob_max_abs": (lp_bu - lp_cu)[fin].abs().max().item(),
            "cached_vs_uncached_max_abs": (lp_s - lp_bu)[fin].abs().max().item()}


def case_compile(_args) -> dict:
    """The generate.py rungs compile / kv_cache / split_kv on a small BD3LM: the backbone
    compiled with dynamic=True runs the library's ops (counted at the C-ABI wrappers) with
    no graph break, and its log-probs equal the eager backbone's."""
    import bench.attention as ba
    import torch._dynamo
    from torch._dynamo.utils import counters

    from bd3attn import ops
    from sample.sampler import sample_bd3lm
    calls = {"decode": 0}
    raw = ops.decode_raw

    def counted(*a, **k):
        calls["decode"] += 1
        return raw(*a, **k)

    ops.decode_raw = counted
    model = _small_bd3lm().eval()
    eager = copy.deepcopy(model)
    prompt = torch.randint(0, 100, (1, 96), generator=torch.Generator().manual_seed(5)).cuda()
    # inference/generate.py: compiled() then split_kv()
    ba.install_attention("bsdfa", block_size=model.block_size)
    torch._dynamo.config.recompile_limit = 64
    model.backbone.compile(dynamic=True)
    ba.install_attention("split_kv", block_size=model.block_size)
    counters.clear()
    torch.manual_seed(6)
    with torch.autocast("cuda", torch.bfloat16):
        tokens = sample_bd3lm(model, 1, 3, 2, True, prompt)
    breaks = {str(k): v for k, v in counters["graph_break"].items()}
    lp_compiled = _teacher_forced(model, tokens, "split_kv", cached=True)
    lp_eager = _teacher_forced(eager, tokens, "split_kv", cached=True)
    fin = lp_eager > -1e5
    return {"graph_breaks": breaks, "library_decode_calls": calls["decode"],
            "tokens_shape": list(tokens.shape),
            "no_mask_left": bool((tokens != model.mask_index).all()),
            "compiled_vs_eager_logprob_max_abs": (lp_compiled - lp_eager)[fin].abs().max().item(),
            "frames_compiled": int(counters["stats"].get("unique_graphs", 0))}


def case_attention_bench(_args) -> dict:
    """bench/attention_bench.py's own backends() and time_fwd_bwd() at one of its configs
    (n = 1024, block 16), with harness.check comparing "bsfa" against "custom"."""
    import bench.attention_bench as ab
    from bench.harness import check
    n, bs = 1024, 16
    mask, fns = ab.backends(n, bs)
    q, k, v = ab.randn_qkv(2, 2 * n, torch.bfloat16)
    with torch.autocast("cuda", torch.bfloat16):
        o_ref = fns["custom"](q, k, v)
        o = fns["bsfa"](q, k, v)
        fwd_ms, bwd_ms, peak_gb = ab.time_fwd_bwd(fns["bsfa"], q, k, v, warmup=3, rep=5)
    c = check(o, o_ref, atol=2e-2, rtol=0.0)
    return {"check_passed": c.passed, "max_abs": c.max_abs, "cosine": c.cosine,
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "peak_gb": peak_gb,
            "density": mask.float().mean().item()}


def case_train_loop(args) -> dict:
    """train/train.py's main() (bd3lm, bf16 autocast, AdamW, clipping) for both attention
    backends on a synthetic memory-mapped token file. Arguments: a JSON object of
    TrainConfig fields (model size, batch, steps); the defaults are a small model."""
    import numpy as np

    from train import train as tr
    cfg = {"seq_len": 256, "batch_size": 4, "d_model": 128, "n_heads": 2, "n_layers": 2,
           "d_ff": 256, "d_cond": 32, "steps": 24, "warmup_steps": 4}
    cfg.update(args)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        # a learnable stream: a random 64-token motif repeated, so attention to the clean
        # blocks predicts the masked tokens
        motif = np.random.default_rng(0).integers(0, 1000, 64, dtype=np.uint16)
        np.tile(motif, 1 << 14).tofile(os.path.join(tmp, "train.bin"))
        os.environ["RESULTS_DIR"] = os.path.join(tmp, "results")
        for attn in ("bsfa", "custom"):
            run = os.path.join(tmp, attn)
            tr.main(tr.TrainConfig(model="bd3lm", attn=attn, data_dir=tmp, out_dir=run, **cfg))
            with open(os.path.join(run, "metrics.json")) as f:
                m = json.load(f)
            out[attn] = {"tokens_per_s": m["tokens_per_s"], "median_step_ms": m["median_step_ms"],
                         "losses": m["losses"]}
    lb, lc = out["bsfa"]["losses"], out["custom"]["losses"]
    out["loss_max_rel_diff"] = max(abs(a - b) / abs(b) for a, b in zip(lb, lc))
    out["config"] = cfg
    return out


CASES = {"registry": case_registry, "train": case_train, "sample": case_sample,
         "compile": case_compile, "attention_bench": case_attention_bench,
         "train_loop": case_train_loop}

if __name__ == "__main__":
    if not os.path.isdir(REF):
        raise SystemExit("baseline/_ref is missing: python baseline/install_reference.py --src …")
    arg = json.loads(sys.argv[2]) if len(sys.argv) > 2 else {}
    print(json.dumps({"case": sys.argv[1], **CASES[sys.argv[1]](arg)}), flush=True)
