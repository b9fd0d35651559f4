"""Failure detection on the GPU without a fault: a bounded wait that runs out.

Every pipeline wait in the library's kernels is bounded; a wait that outlasts
its limit sets the device error flag and the kernel returns instead of
hanging. r4c_watchdog_selftest() runs that same wait routine on a barrier
nothing arrives at (a flag that nothing sets), so the wait runs out on
purpose: the kernel must return within about its limit, the host must read
the error code, and the context must stay usable for a normal call after it.
"""
import time

import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports(cuda_ready):
    from rdna4_conv3d import _native
    assert _native.device_error() == 0
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _native.watchdog_selftest(20_000_000)            # 20 ms limit
    code = _native.device_error(clear=False)          # synchronizes the stream
    elapsed = time.perf_counter() - t0
    assert code == 3, code
    assert 0.015 <= elapsed < 2.0, elapsed            # waited about its limit, then returned
    assert _native.device_error(clear=True) == 3      # read and clear
    assert _native.device_error() == 0


def test_context_usable_after_timeout(cuda_ready):
    import sys
    from rdna4_conv3d import _native
    _native.watchdog_selftest(5_000_000)
    assert _native.device_error() == 3
    cw = sys.modules["rdna4_conv3d.conv3d_wmma"]
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1, 24, 6, 10, 12, generator=g).to(torch.bfloat16)
    w = (torch.randn(24, 24, 3, 3, 3, generator=g) / 25.0).to(torch.bfloat16)
    y = cw._launch_fwd(x.cuda(), w.cuda(), None, (1, 1, 1)).cpu()
    assert O.max_rel(y, O.torch_conv_fwd(x, w, None, 1)) <= 2e-2
    assert _native.device_error() == 0


def test_selftest_rejects_bad_limits(cuda_ready):
    from rdna4_conv3d import _native
    with pytest.raises(_native.NativeError):
        _native.watchdog_selftest(0)
    with pytest.raises(_native.NativeError):
        _native.watchdog_selftest(5_000_000_000)
