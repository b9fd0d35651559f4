"""The allocation-free weight-gradient entry point, through the C ABI.

r4c_conv3d_dw_noalloc() serves callers that cannot allocate device memory
(a guest op inside another framework's memory pool, or a path that must not
call cudaMalloc): its split-K scratch is a fixed array inside the library.
It must return what r4c_conv3d_dw() returns with a caller workspace, call
after call (the scratch keeps the previous call's contents), and refuse
problems whose scratch would not fit.

Collected last on purpose (file name): a failure here leaves every other test
already run.
"""
import ctypes

import pytest
import torch

import oracle as O
from rdna4_conv3d import _native

pytestmark = pytest.mark.gpu

DW_TOL = 3e-2   # norm-relative, the dW tolerance of the parity tests


def _bind():
    lib = _native.lib()
    fn = lib.r4c_conv3d_dw_noalloc
    fn.argtypes = [ctypes.POINTER(_native.ConvDesc), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _cl(t):
    return t.contiguous(memory_format=torch.channels_last_3d)


# (n, cin, cout, d, h, w, k, pad), dtype, kernel family forced (0 = automatic,
# 1 = the SIMT weight-gradient kernel): every dW path that uses the scratch
NOALLOC_CASES = [
    ((2, 24, 24, 16, 32, 32, 3, 1), torch.bfloat16, 0),   # tcgen05 dW
    ((2, 24, 24, 16, 32, 32, 3, 1), torch.float16, 0),
    ((1, 12, 24, 4, 6, 8, 3, 1), torch.bfloat16, 0),      # tcgen05 dW after channel padding into the scratch
    ((1, 48, 24, 8, 16, 16, 1, 0), torch.bfloat16, 0),    # k1
    ((1, 1, 24, 8, 16, 16, 3, 1), torch.bfloat16, 0),     # stem dW (one input channel)
    ((1, 3, 16, 6, 8, 16, 3, 1), torch.float16, 0),       # stem dW, three input channels
    ((1, 5, 7, 4, 5, 6, 3, 1), torch.bfloat16, 1),        # SIMT dW (split-K partials in the scratch)
    ((1, 16, 8, 4, 6, 8, 3, 1), torch.float16, 1),
]


@pytest.mark.parametrize("case,dtype,force", NOALLOC_CASES,
                         ids=["cfg1", "cfg1-fp16", "cpad", "k1", "stem", "stem3-fp16", "simt", "simt-fp16"])
def test_noalloc_matches_workspace_entry(cuda_ready, case, dtype, force):
    fn = _bind()
    n, cin, cout, d, h, w, k, pad = case
    g = torch.Generator().manual_seed(7)
    x = _cl(torch.randn(n, cin, d, h, w, generator=g).to(dtype).cuda())
    od, oh, ow = (s + 2 * pad - (k - 1) for s in (d, h, w))
    go = _cl(torch.randn(n, cout, od, oh, ow, generator=g).to(dtype).cuda())
    desc = _native.make_desc(n, d, h, w, cin, cout, k, (pad, pad, pad), dtype, force)
    assert 0 < _native.workspace_bytes(desc, _native.LEG_DW) <= 32 << 20

    ref_dw, ref_db = _native.conv_dw(desc, x, go, True)     # existing entry point, torch workspace
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):                                        # two calls in a row share the scratch
        dw = torch.full((cout, cin, k, k, k), float("nan"), device="cuda")
        db = torch.full((cout,), float("nan"), device="cuda")
        st = fn(ctypes.byref(desc), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(go.data_ptr()),
                ctypes.c_void_p(dw.data_ptr()), ctypes.c_void_p(db.data_ptr()), stream)
        assert st == 0, _native.strerror(st)
        torch.cuda.synchronize()
        assert torch.isfinite(dw).all() and torch.isfinite(db).all()
        assert O.norm_rel(dw.cpu(), ref_dw.cpu()) <= DW_TOL
        assert O.norm_rel(db.cpu(), ref_db.cpu()) <= DW_TOL
    assert _native.device_error() == 0


def test_noalloc_rejects_oversized_problem(cuda_ready):
    fn = _bind()
    desc = _native.make_desc(1, 4, 4, 4, 1024, 1024, 3, (1, 1, 1), torch.bfloat16)
    assert _native.workspace_bytes(desc, _native.LEG_DW) > 32 << 20
    st = fn(ctypes.byref(desc), None, None, None, None, None)
    assert st == -7  # R4C_ERR_TOO_LARGE, nothing launched
