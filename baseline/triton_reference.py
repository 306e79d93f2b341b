"""Time the reference's own Triton kernels, unchanged, on this GPU (the secondary comparator).

    python baseline/triton_reference.py

Imports the reference installed in baseline/_ref (baseline/install_reference.py) with nothing
of this repository on the import path, so ``kernels`` is the reference's package, and times
at the benchmark configs:
  C2   BlockSparseFlashAttention.apply forward, and forward + backward (autograd), B=8, H=12,
       n=1024, block 16, bf16 (useful FLOPs as bench.py: 4*D*nnz*B*H forward, bwd 2.5x);
  C3   split_kv_decode_attention, a 16-token block over 64K + 16 keys at B=32 and 16K + 16 at
       B=8 (bytes B*H*(256*kv_len + 4096));
  pre  block_sparse_decode_attention over 3088 queries and keys at B=1 (the reference's
       bench/decode_ncu.py "uncached" shape).
Each is timed as the reference's bench/harness.py does (CUDA events, a 256 MiB buffer written
before every repetition, median). Config 4's per-head live-block mask has no reference kernel.

The reference's kernels build TMA descriptors on the device (tl.make_tensor_descriptor), for
which Triton asks the caller for a scratch allocator (triton.set_allocator) that the reference
never installs. A first attempt runs exactly as the reference would; if Triton refuses for want
of an allocator, the error is recorded and the run is repeated with a torch-backed allocator
installed by this harness (the kernels themselves stay unchanged). Prints one JSON line.
"""

from __future__ import annotations

import json
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")
sys.path[:] = [REF] + [p for p in sys.path if p not in (HERE, REPO, "")]

import torch  # noqa: E402

H, D = 12, 64


def timed(fn, warmup: int = 3, rep: int = 10) -> float:
    """Median milliseconds of fn() over rep calls, each after a 256 MiB write (L2 flush)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    l2 = torch.empty(256 * 2**20, dtype=torch.uint8, device="cuda")
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(rep)]
    for a, b in evs:
        l2.zero_()
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in evs)


def run_cases(alloc=None) -> dict:
    """Time each config; a config that fails records its error instead of a time."""
    import triton
    from kernels.BlockSparseDecodeAttention import block_sparse_decode_attention
    from kernels.BlockSparseFlashAttention import BlockSparseFlashAttention
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    out = {"kernels_from": os.path.relpath(
        os.path.dirname(sys.modules["kernels.BlockSparseFlashAttention"].__file__), REPO)}
    g = torch.Generator(device="cuda").manual_seed(0)

    def randn(*shape):
        return torch.empty(*shape, dtype=torch.bfloat16, device="cuda").normal_(generator=g)

    def case(name, fn):
        try:
            out[name] = fn()
        except Exception as e:
            out[name] = {"error": f"{type(e).__name__}: {str(e).splitlines()[0][:300]}"}
        torch.cuda.empty_cache()

    B, n, bs = 8, 1024, 16
    fwd_flops = 4.0 * D * (n * n + n * bs) * B * H

    def c2():
        q, k, v = (randn(B, H, 2 * n, D).requires_grad_(True) for _ in range(3))
        do = randn(B, H, 2 * n, D)
        ms_f = timed(lambda: BlockSparseFlashAttention.apply(q, k, v, bs))
        res = {"fwd_ms": round(ms_f, 4), "fwd_tflops": round(fwd_flops / ms_f / 1e9, 2)}

        def fwd_bwd():
            o = BlockSparseFlashAttention.apply(q, k, v, bs)
            if alloc is not None:
                # the backward runs in autograd's device thread, which does not see the
                # allocator set in this thread: set it there too (a hook on O runs first)
                o.register_hook(lambda grad: (triton.set_allocator(alloc), grad)[1])
            torch.autograd.grad(o, (q, k, v), do)
        try:
            ms_fb = timed(fwd_bwd)
            res.update({"fwd_bwd_ms": round(ms_fb, 4),
                        "fwd_bwd_tflops": round(3.5 * fwd_flops / ms_fb / 1e9, 2)})
        except Exception as e:
            res["bwd_error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:300]}"
        return res
    case("c2_b8_n1024_bs16", c2)

    def c3(b3, kv):
        qd, kd, vd = randn(b3, H, 16, D), randn(b3, H, kv, D), randn(b3, H, kv, D)
        ms = timed(lambda: split_kv_decode_attention(qd, kd, vd, bs))
        by = b3 * H * (256 * kv + 4096)
        return {"us": round(ms * 1e3, 2), "GBps": round(by / ms / 1e6, 1)}
    for b3, kv in ((32, 65536 + 16), (8, 16384 + 16)):
        case(f"c3_splitkv_b{b3}_kv{(kv - 16) // 1024}k", lambda b3=b3, kv=kv: c3(b3, kv))

    def prefill():
        qp, kp, vp = randn(1, H, 3088, D), randn(1, H, 3088, D), randn(1, H, 3088, D)
        return {"us": round(timed(lambda: block_sparse_decode_attention(qp, kp, vp, bs)) * 1e3, 2)}
    case("prefill_b1_3088", prefill)
    return out


def main() -> None:
    import triton
    res = {"triton": triton.__version__, "gpu": torch.cuda.get_device_name()}
    # as the reference runs: no allocator installed
    from kernels.SplitKVDecodeAttention import split_kv_decode_attention
    q = torch.randn(1, H, 16, D, dtype=torch.bfloat16, device="cuda")
    k = torch.randn(1, H, 1040, D, dtype=torch.bfloat16, device="cuda")
    try:
        split_kv_decode_attention(q, k, k, 16)
        torch.cuda.synchronize()
        res["as_is"] = "ran"
        res.update(run_cases())
        res["allocator"] = "none (as the reference runs)"
    except Exception as e:
        res["as_is_error"] = f"{type(e).__name__}: {str(e).splitlines()[0][:300]}"

        def alloc(size, align, stream):
            return torch.empty(size, dtype=torch.int8, device="cuda")
        triton.set_allocator(alloc)
        res.update(run_cases(alloc))
        res["allocator"] = "torch-backed, installed by this harness"
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    if not os.path.isdir(os.path.join(REF, "kernels")):
        print(json.dumps({"unavailable": "baseline/_ref is missing (baseline/install_reference.py)"}))
        sys.exit(0)
    main()
