"""Failure detection on the GPU, without faulting it.

Every pipeline wait in the library's kernels is bounded: when a barrier phase
does not complete in time, the waiting thread records ACTUNE_DEV_TIMEOUT and the
wait site in the device error word and the kernel finishes.  Here the limit is
shortened to 50 ms and the self-test kernel waits on a barrier that nothing
arrives on (nothing in flight, no tensor memory held).  The test checks that the
call returns, that the error word names the timeout and the site, that resetting
it clears it, and that the context still runs a packed linear correctly
afterwards.
"""
import time

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports_without_hanging():
    from actune_b200 import _lib, ops
    L = _lib.lib()
    _lib.device_error(reset=True)
    default = _lib.wait_limit_ns()
    assert default == 2_000_000_000
    _lib.set_wait_limit_ns(50_000_000)
    try:
        stream = torch.cuda.current_stream()
        t0 = time.perf_counter()
        _lib.check(L.actune_selftest_wait_timeout(42, torch.cuda.current_stream().cuda_stream), "selftest")
        stream.synchronize()
        elapsed = time.perf_counter() - t0
        assert 0.04 <= elapsed < 1.5, elapsed          # gave up after about the limit, not the default 2 s
        assert _lib.device_error(reset=True) == (1, 42)  # ACTUNE_DEV_TIMEOUT at the probe's site
        assert _lib.device_error() == (0, 0)
    finally:
        _lib.set_wait_limit_ns(default)
    assert _lib.wait_limit_ns() == default
    # The context is still usable: a packed linear afterwards is bit-exact.
    g = torch.Generator().manual_seed(3)
    x = torch.randn(40, 256, generator=g).bfloat16().cuda()
    wt = (torch.randn(96, 256, generator=g) * 0.02).bfloat16().cuda()
    codes, ws = ops.weight_codes(wt, 4, 8)
    pw = ops.pack_rows(codes, 4)
    pa, as_ = ops.quantize_group64(x, 8)
    y = ops.packed_linear(pa, as_, pw, ws, None, 256, 4, 8, out_dtype=torch.float32)
    exact = O.packed_linear(pa.cpu().numpy(), as_.cpu().numpy(), pw.cpu().numpy(), ws.cpu().numpy(), None, 256, 4, 8)
    assert np.array_equal(y.cpu().numpy(), exact)
    assert _lib.device_error() == (0, 0)


def test_wait_limit_rejects_out_of_range_values():
    from actune_b200 import _lib
    L = _lib.lib()
    assert L.actune_set_wait_limit_ns(10) == _lib.ERR_INVALID_VALUE
    assert L.actune_set_wait_limit_ns(120_000_000_000) == _lib.ERR_INVALID_VALUE
    assert L.actune_selftest_wait_timeout(0, None) == _lib.ERR_INVALID_VALUE
