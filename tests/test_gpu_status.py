"""Failure detection on a real GPU, without a fault.

Every pipeline wait in the kernels (on an mbarrier a TMA copy or a producer completes) is bounded at
about one second; when one runs out the kernel sets bit 0 of a device status word, stops and
returns, so the context stays usable and the host learns of it through cc1d_status().
cc1d_selftest_wait_timeout launches a block that waits on an mbarrier nothing ever completes. The
test checks that the wait gives up in bounded time, that the bit is reported and cleared on read,
and that the library still works afterwards: a forward gives the same bits as before and leaves the
status clear.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_timeout_sets_status_and_context_survives():
    from causal_conv1d_b200 import _native, causal_conv1d_fn
    from causal_conv1d_b200.causal_conv1d import _stream

    dev = torch.device("cuda", 0)
    assert _native.status(clear=True) == 0
    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 300, 256, generator=g).to(torch.bfloat16).to(dev)
    w = torch.randn(256, 4, generator=g).to(dev)
    before = causal_conv1d_fn(x, w, activation="silu")
    torch.cuda.synchronize()

    t0 = time.perf_counter()
    _native.check(_native.lib.cc1d_selftest_wait_timeout(_stream(dev)), "cc1d_selftest_wait_timeout")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert 0.5 < elapsed < 30, f"the bounded wait took {elapsed:.2f} s"
    assert _native.status(clear=True) & 1, "the timed-out wait did not set the status bit"
    assert _native.status() == 0, "reading with clear=True must reset the status word"

    after = causal_conv1d_fn(x, w, activation="silu")
    torch.cuda.synchronize()
    assert torch.equal(before, after)
    assert _native.status(clear=True) == 0
