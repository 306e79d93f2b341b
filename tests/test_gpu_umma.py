"""Each tcgen05 operand layout the kernels use, checked in isolation (libbd3diag.so)."""

import ctypes
import os

import pytest
import torch

from conftest import PKG_ROOT
from gpu_util import assert_device_ok

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def diag():
    lib = ctypes.CDLL(os.path.join(PKG_ROOT, "lib", "libbd3diag.so"))
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
