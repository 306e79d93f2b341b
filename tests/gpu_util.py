"""Shared helpers of the GPU parity tests: seeded inputs drawn on the CPU (so the oracle and
the GPU see identical values) and the tolerances stated by the task:
bf16 O and dQ/dK/dV within 2e-2 max-abs of an fp32-or-better reference, LSE within 1e-3."""

import torch

O_TOL = 2e-2
GRAD_TOL = 2e-2
LSE_TOL = 1e-3


def randn(gen, shape, dtype=torch.bfloat16):
    return torch.randn(shape, generator=gen).to(dtype)


def qkv(seed, B, H, Sq, Sk, dtype=torch.bfloat16, D=64):
    g = torch.Generator().manual_seed(seed)
    return randn(g, (B, H, Sq, D), dtype), randn(g, (B, H, Sk, D), dtype), \
        randn(g, (B, H, Sk, D), dtype)


def max_abs(a, b):
    return (a.detach().double().cpu() - b.detach().double().cpu()).abs().max().item()


def assert_close(name, got, ref, tol):
    err = max_abs(got, ref)
    assert err <= tol, f"{name}: max-abs {err:.3e} > {tol:.1e}"
    return err


def assert_device_ok():
    from bd3attn import ops
    torch.cuda.synchronize()
    st = ops.device_status(clear=True)
    site = ops.debug_wait_site()
    assert st == 0, f"device status bits {st} (a bounded wait ran out: {site})"
