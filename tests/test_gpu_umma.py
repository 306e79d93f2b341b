"""Device building blocks checked in isolation (libbd3diag.so): each tcgen05 operand layout the
kernels use, and the FMA-pipe exponential of the forward softmax."""

import ctypes
import os

import pytest
import torch

from conftest import REPO
from gpu_util import assert_device_ok

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def diag():
    lib = ctypes.CDLL(os.path.join(REPO, "tests", "diag", "libbd3diag.so"))
    fn = lib.bd3diag_umma_selftest
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 9
    return fn


def test_umma_layouts(diag):
    g = torch.Generator().manual_seed(11)
    A, Bk, V, Y = (torch.randn(128, 64, generator=g).bfloat16() for _ in range(4))
    X = torch.randn(128, 128, generator=g).bfloat16()
    dev = [t.cuda() for t in (A, Bk, V, X, Y)]
    S = torch.empty(128, 128, device="cuda")
    O = torch.empty(128, 64, device="cuda")
    C = torch.empty(128, 64, device="cuda")
    rc = diag(*[ctypes.c_void_p(t.data_ptr()) for t in dev + [S, O, C]],
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert_device_ok()
    S_ref = A.float() @ Bk.float().T
    torch.testing.assert_close(S.cpu(), S_ref, atol=1e-3, rtol=1e-3)
    P = (S.cpu() * 0.0625).bfloat16().float()
    torch.testing.assert_close(O.cpu(), P @ V.float(), atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(C.cpu(), X.float().T @ Y.float(), atol=1e-3, rtol=1e-3)


def test_exp2_fma2_error_bound():
    """The forward's FMA-pipe exponential: relative error at most 1e-4 against exp2 over the
    softmax's argument range, exact +0 at and below -127 (and for -inf, the masked entries),
    within the same bound of the MUFU ex2.approx it stands in for."""
    lib = ctypes.CDLL(os.path.join(REPO, "tests", "diag", "libbd3diag.so"))
    fn = lib.bd3diag_exp2
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p]
    g = torch.Generator().manual_seed(3)
    t = torch.cat([torch.linspace(-126.0, 8.0, 400_000), -126 + 134 * torch.rand(200_000, generator=g),
                   torch.tensor([-127.0, -128.0, -1000.0, float("-inf"), 0.0, -1.0, 1.0, 8.0])])
    t = t[: t.numel() // 2 * 2].float()
    td = t.cuda()
    poly, mufu = torch.empty_like(td), torch.empty_like(td)
    assert fn(td.data_ptr(), poly.data_ptr(), mufu.data_ptr(), td.numel(),
              torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    poly, mufu = poly.cpu().double(), mufu.cpu().double()
    ref = torch.exp2(t.double())
    normal = t >= -126
    rel = ((poly - ref).abs() / ref)[normal]
    assert rel.max().item() < 1e-4, rel.max().item()
    assert ((poly - mufu).abs() / ref)[normal].max().item() < 1.2e-4
    assert (poly[t <= -127] == 0).all() and (poly[t <= -127].sign() >= 0).all()
    assert poly[t == 0].eq(1.0).all() and poly[t == 1].eq(2.0).all() and poly[t == 8].eq(256.0).all()
