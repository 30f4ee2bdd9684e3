"""The kernels' shared failure path, exercised without a fault: a bounded
mbarrier wait that nothing completes expires, the kernel records
H3B_ERR_TIMEOUT in the device error word and returns, the host reads the
status, and the context keeps working."""
import numpy as np
import pytest
import torch

from oracle import nvfp4_ref as R

H3B_ERR_INVALID_ARG = 1
H3B_ERR_TIMEOUT = 5


def test_selftest_rejects_bounds_outside_range():
    from h3_engine_b200 import _lib
    lib = _lib.lib()
    assert lib.h3b_selftest_bounded_wait(0, None) == H3B_ERR_INVALID_ARG
    assert lib.h3b_selftest_bounded_wait(1000001, None) == H3B_ERR_INVALID_ARG
    assert "wait" in _lib.status_string(H3B_ERR_TIMEOUT)


@pytest.mark.gpu
def test_bounded_wait_expires_reports_and_context_survives(cuda):
    from h3_engine_b200 import _lib, ops
    lib = _lib.lib()
    assert _lib.device_error(clear=True) == 0
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    _lib.check(lib.h3b_selftest_bounded_wait(20000, stream.cuda_stream), "selftest")
    e1.record(stream)
    assert _lib.device_error(clear=True) == H3B_ERR_TIMEOUT
    assert e0.elapsed_time(e1) >= 19.0             # the wait ran to its 20 ms bound
    # the context is intact: a quantization right after is bit-exact
    g = torch.Generator().manual_seed(9)
    x = torch.randn(256, 512, generator=g).to(torch.bfloat16)
    q, sf, gs = ops.quantize(x.to(cuda))
    rq, rs, rgs = R.quantize(x.float().numpy(), mpad=q.shape[0])
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(sf.cpu().numpy(), R.swizzle(rs))
    assert _lib.device_error() == 0
