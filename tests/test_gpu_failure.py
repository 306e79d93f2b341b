"""Failure handling on the GPU without a fault: the bounded wait every kernel uses gives up
on a barrier nothing arrives at, records it in the sticky device status, and returns, so
the kernel exits and the context stays usable (bd3_debug_wait_timeout, a 1 ms limit)."""

import pytest
import torch

import oracle
from gpu_util import O_TOL, assert_close, assert_device_ok, qkv

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_stays_usable():
    from bd3attn import ops
    ops.device_status(clear=True)
    gave_up, ns = ops.debug_wait_timeout(1_000_000)  # no arrival: must give up after 1 ms
    assert gave_up == 1
    assert 1_000_000 <= ns < 100_000_000, ns
    assert ops.device_status(clear=True) == 1  # bit 1: a bounded wait ran out
    assert ops.device_status(clear=True) == 0  # and reading it cleared it
    site = ops.debug_wait_site()  # the probe's one waiting thread, parity 0
    assert site is not None and site["block"] == 0 and site["thread"] == 0 and site["parity"] == 0
    assert ops.debug_wait_site() is None  # reading it cleared it
    # control: with the arrival the same wait completes at once and records nothing
    gave_up, ns = ops.debug_wait_timeout(1_000_000, arrive=True)
    assert gave_up == 0 and ns < 1_000_000
    assert ops.device_status(clear=True) == 0
    # the next regular launch on the same context is clean and correct
    q, k, v = qkv(5, 2, 12, 16, 1040)
    o = ops.decode_raw(q.cuda(), k.cuda(), v.cuda(), 16)
    assert_device_ok()
    ref, _ = oracle.attention(q, k, v, oracle.block_causal_mask(16, 1040, 16))
    assert_close("O after the timeout", o, ref, O_TOL)


def test_repeated_timeouts_stay_sticky_until_read():
    from bd3attn import ops
    ops.device_status(clear=True)
    for _ in range(3):
        assert ops.debug_wait_timeout(20_000)[0] == 1
    torch.cuda.synchronize()
    assert ops.debug_wait_site() is not None
    assert ops.device_status(clear=False) == 1  # read without clearing: still set
    assert ops.device_status(clear=True) == 1
    assert ops.device_status(clear=True) == 0
