"""actune_grouped_linear_noalloc: the allocation-free entry point.

For callers that cannot allocate device memory when they run the linear (a host
whose memory belongs to another allocator, a control loop that must not
allocate once running), this entry point keeps its activation scratch in a
fixed device array inside the library.  The test calls it through the C ABI
and compares its output with the workspace entry point (actune_grouped_linear)
on the same inputs -- bit for bit, the tolerance the other GPU tests use for
this arithmetic -- for two calls in a row with different inputs, so a stale
scratch from the first call would show in the second.  It sits in its own file
named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_BYTES = 8 << 20  # ACTUNE_NOALLOC_SCRATCH_BYTES in include/actune_b200.h


def _noalloc():
    from actune_b200 import _lib
    L = _lib.lib()
    fn = L.actune_grouped_linear_noalloc
    p, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    fn.argtypes = [p, i32, i64, i64, p, p, p, i32, i64, i32, i32, p, i32, i32, p]
    fn.restype = i32
    return fn


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _inputs(seed, m, k, n, w, a):
    from actune_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    weight = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    codes, ws = ops.weight_codes(weight, w, a)
    pw = ops.pack_rows(codes, w)
    bias = torch.randn(n, device="cuda", generator=g).bfloat16()
    return x, pw, ws, bias


def test_noalloc_matches_workspace_entry_on_two_calls():
    from actune_b200 import _lib, ops
    fn = _noalloc()
    for call, (m, k, n, w, a) in enumerate([(37, 4096, 512, 4, 8), (300, 1024, 256, 2, 4)]):
        x, pw, ws, bias = _inputs(100 + call, m, k, n, w, a)
        expected = ops.grouped_linear(x, pw, ws, bias, w, a)  # existing entry point, own workspace
        out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        rc = fn(_ptr(x), _lib.DTYPE_BF16, m, k, _ptr(pw), _ptr(ws), _ptr(bias), _lib.DTYPE_BF16, n, w, a,
                _ptr(out), _lib.DTYPE_BF16, _lib.VARIANT_AUTO,
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert rc == _lib.OK, _lib.status_string(rc)
        assert torch.equal(out, expected), f"call {call}"
    assert _lib.device_error()[0] == 0


def test_noalloc_refuses_requests_beyond_its_scratch():
    from actune_b200 import _lib
    fn = _noalloc()
    m, k = 4096, 4096  # A8: 16 MiB of packed activations > 8 MiB
    assert _lib.lib().actune_grouped_linear_workspace_size(m, k, 8) > NOALLOC_SCRATCH_BYTES
    null = ctypes.c_void_p(0)
    rc = fn(null, _lib.DTYPE_BF16, m, k, null, null, null, 0, 64, 4, 8, null, _lib.DTYPE_BF16, 0, null)
    assert rc == _lib.ERR_WORKSPACE


def test_noalloc_boundary_exactly_at_the_scratch_size():
    """A request whose scratch is exactly the array's size runs and matches the
    workspace entry point; one more token row is refused."""
    from actune_b200 import _lib, ops
    fn = _noalloc()
    m, k, n, w, a = 7710, 1024, 256, 4, 8
    size = _lib.lib().actune_grouped_linear_workspace_size
    assert size(m, k, a) == NOALLOC_SCRATCH_BYTES and size(m + 1, k, a) > NOALLOC_SCRATCH_BYTES
    x, pw, ws, bias = _inputs(300, m, k, n, w, a)
    expected = ops.grouped_linear(x, pw, ws, bias, w, a)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = fn(_ptr(x), _lib.DTYPE_BF16, m, k, _ptr(pw), _ptr(ws), _ptr(bias), _lib.DTYPE_BF16, n, w, a,
            _ptr(out), _lib.DTYPE_BF16, _lib.VARIANT_AUTO, stream)
    torch.cuda.synchronize()
    assert rc == _lib.OK, _lib.status_string(rc)
    assert torch.equal(out, expected)
    null = ctypes.c_void_p(0)
    rc = fn(null, _lib.DTYPE_BF16, m + 1, k, null, null, null, 0, n, w, a, null, _lib.DTYPE_BF16, 0, null)
    assert rc == _lib.ERR_WORKSPACE
