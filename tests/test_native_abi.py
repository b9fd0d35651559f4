"""The C-ABI library loads and exports every symbol include/*.h declares.

CPU only: host-side entry points (plan, sizes, strerror, descriptor checks)
are called; nothing launches a kernel.
"""
import ctypes
import glob
import os
import re

import torch

from conftest import ROOT
from rdna4_conv3d import _native

HEADERS = glob.glob(os.path.join(ROOT, "include", "*.h"))


def _declared():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(r4c_[a-z0-9_]+)\s*\(", src))
    return names


def test_header_declares_entry_points():
    names = _declared()
    for n in ("r4c_conv3d_fwd", "r4c_conv3d_dx", "r4c_conv3d_dw", "r4c_tconv_fwd", "r4c_tconv_dx",
              "r4c_tconv_dw", "r4c_pack_weight", "r4c_workspace_size", "r4c_strerror"):
        assert n in names


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(_native.library_path())
    missing = [n for n in sorted(_declared()) if not hasattr(lib, n)]
    assert not missing, missing


def test_strerror_and_version():
    assert _native.strerror(0) == "ok"
    assert "workspace" in _native.strerror(-3)
    assert _native.lib().r4c_version() >= 1


def _d(n=2, cin=24, cout=24, d=16, h=32, w=32, k=3, p=1, dt=torch.bfloat16, force=0):
    return _native.make_desc(n, d, h, w, cin, cout, k, (p, p, p), dt, force)


def test_plan_families():
    assert _native.plan_kernel(_d(), _native.LEG_FWD) == _native.KERNEL_TC
    assert _native.plan_kernel(_d(), _native.LEG_DX) == _native.KERNEL_TC
    # odd input channels: the forward pads them to 8 in workspace and stays on
    # tcgen05; dX and dW of that layer pad dY's 7 channels to 8 the same way
    assert _native.plan_kernel(_d(cin=5, cout=7), _native.LEG_FWD) == _native.KERNEL_TC
    assert _native.workspace_bytes(_d(cin=5, cout=7), _native.LEG_FWD) >= 2 * 16 * 32 * 32 * 8 * 2
    assert _native.plan_kernel(_d(cin=5, cout=7), _native.LEG_DX) == _native.KERNEL_TC
    assert _native.workspace_bytes(_d(cin=5, cout=7), _native.LEG_DX) >= 2 * 16 * 32 * 32 * 8 * 2
    assert _native.plan_kernel(_d(cin=24, cout=4, k=1, p=0), _native.LEG_DW) == _native.KERNEL_TC
    # the generic family can be forced
    assert _native.plan_kernel(_d(force=1), _native.LEG_FWD) == _native.KERNEL_GENERIC
    assert "tcgen05" in _native.describe_plan(_d(), _native.LEG_FWD)


def test_stem_family():
    # k=3 forward with 1..4 input channels (and W*Cin a multiple of 8): the stem
    # kernel, no channel-padding workspace, weight image [16-padded Cout][K]
    # with K = 9 groups of 4*Cin (3*Cin taps + Cin zeros) rounded up to 16
    for cin, cout, w, kpad in ((1, 24, 32, 48), (2, 16, 12, 80), (3, 8, 8, 112), (4, 200, 10, 144)):
        dsc = _d(cin=cin, cout=cout, w=w)
        assert _native.plan_kernel(dsc, _native.LEG_FWD) == _native.KERNEL_TC
        assert "stem" in _native.describe_plan(dsc, _native.LEG_FWD)
        assert _native.workspace_bytes(dsc, _native.LEG_FWD) == 0
        assert _native.packed_weight_bytes(dsc, _native.LEG_FWD) == (cout + 15) // 16 * 16 * kpad * 2
        # dX: the stem dX kernel for one input channel (Cout a multiple of 4
        # up to 32, pad 1, even W <= 256), else the general kernel; dW takes
        # the stem dW kernel when Cout is a multiple of 8 and its buffers fit
        if cin == 1 and cout <= 32:
            assert "stem dX" in _native.describe_plan(dsc, _native.LEG_DX)
            assert _native.packed_weight_bytes(dsc, _native.LEG_DX) == 96 * 128
            assert _native.workspace_bytes(dsc, _native.LEG_DX) == 0
        else:
            assert "stem" not in _native.describe_plan(dsc, _native.LEG_DX)
        if cout % 8 == 0 and cout <= 32:
            assert "stem dW" in _native.describe_plan(dsc, _native.LEG_DW)
            assert _native.workspace_bytes(dsc, _native.LEG_DW) > 0
    # Cout not a multiple of 8: the dW leaves the stem kernel
    assert "stem" not in _native.describe_plan(_d(cin=1, cout=7, w=32), _native.LEG_DW)
    # stem dX scope: Cout % 4, Cout <= 32, pad 1, even W up to 256
    assert "stem dX" in _native.describe_plan(_d(cin=1, cout=4, w=2, h=1, d=1), _native.LEG_DX)
    assert "stem dX" in _native.describe_plan(_d(cin=1, cout=32, w=256), _native.LEG_DX)
    for bad in (_d(cin=1, cout=6), _d(cin=1, cout=48), _d(cin=1, w=31), _d(cin=1, w=258), _d(cin=1, p=0),
                _d(cin=1, p=2), _d(cin=1, force=1)):
        assert "stem dX" not in _native.describe_plan(bad, _native.LEG_DX)
    # rows whose byte stride is not a multiple of 16, k=1 and 5+ channels stay
    # on the general kernel; forcing the SIMT family still works
    assert "stem" not in _native.describe_plan(_d(cin=3, w=30), _native.LEG_FWD)
    assert _native.workspace_bytes(_d(cin=3, w=30), _native.LEG_FWD) > 0
    assert "stem" not in _native.describe_plan(_d(cin=2, k=1, p=0), _native.LEG_FWD)
    assert "stem" not in _native.describe_plan(_d(cin=5, w=8), _native.LEG_FWD)
    assert _native.plan_kernel(_d(cin=1, force=1), _native.LEG_FWD) == _native.KERNEL_GENERIC


def test_tconv_family():
    # ConvTranspose3d k2s2 forward / dX with Cin, Cout multiples of 8: the
    # tcgen05 transpose-conv kernel, weights packed per task as 64-channel
    # swizzled images (boxes x N columns x 128 B); dW: the tcgen05 split-K
    # kernel, its partials (plus the db partials) in the caller's workspace
    def t(n, cin, cout, d, h, w, force=0):
        return _native.make_desc(n, d, h, w, cin, cout, 2, (0, 0, 0), torch.bfloat16, force)
    for cin, cout, sp, fwd_b, dx_b in ((48, 24, (32, 64, 64), 1 * 192 * 128, 4 * 48 * 128),
                                       (96, 48, (16, 32, 32), 2 * 2 * 192 * 128, 8 * 96 * 128),
                                       (192, 96, (8, 16, 16), 3 * 3 * 256 * 128, 3 * 12 * 64 * 128)):
        dsc = t(4, cin, cout, *sp)
        for leg, nbytes in ((_native.LEG_TFWD, fwd_b), (_native.LEG_TDX, dx_b)):
            assert _native.plan_kernel(dsc, leg) == _native.KERNEL_TC
            assert "tcgen05 tconv" in _native.describe_plan(dsc, leg)
            assert _native.packed_weight_bytes(dsc, leg) == nbytes
            assert _native.workspace_bytes(dsc, leg) == 0
        assert _native.plan_kernel(dsc, _native.LEG_TDW) == _native.KERNEL_TC
        assert "tcgen05 tconv dW" in _native.describe_plan(dsc, _native.LEG_TDW)
        assert _native.workspace_bytes(dsc, _native.LEG_TDW) > 0
    # channel counts off the multiple of 8, or the SIMT family forced
    assert _native.plan_kernel(t(1, 5, 3, 2, 3, 4), _native.LEG_TFWD) == _native.KERNEL_GENERIC
    assert _native.plan_kernel(t(1, 16, 12, 2, 3, 4), _native.LEG_TDX) == _native.KERNEL_GENERIC
    assert _native.plan_kernel(t(1, 16, 8, 2, 3, 4, force=1), _native.LEG_TFWD) == _native.KERNEL_GENERIC
    assert _native.plan_kernel(t(1, 16, 12, 2, 3, 4), _native.LEG_TDW) == _native.KERNEL_GENERIC
    assert _native.plan_kernel(t(1, 16, 8, 2, 3, 4, force=1), _native.LEG_TDW) == _native.KERNEL_GENERIC


def test_descriptor_validation():
    assert _native.plan_kernel(_d(k=5), _native.LEG_FWD) == -2       # unsupported
    assert _native.plan_kernel(_d(k=3), _native.LEG_TFWD) == -2      # tconv needs k=2
    assert _native.plan_kernel(_d(p=-1), _native.LEG_FWD) == -1      # negative pad
    assert _native.plan_kernel(_d(cin=0), _native.LEG_FWD) == -1
    assert _native.plan_kernel(_d(d=1, p=0), _native.LEG_FWD) == -1  # empty output
    bad = _d()
    bad.dtype = 7
    assert _native.plan_kernel(bad, _native.LEG_FWD) == -1


def test_workspace_sizes():
    ws = _native.workspace_bytes(_d(), _native.LEG_DW)
    assert ws > 0 and ws % 256 == 0
    assert _native.workspace_bytes(_d(), _native.LEG_FWD) == 0
    t = _native.make_desc(1, 4, 4, 4, 16, 8, 2, (0, 0, 0), torch.bfloat16)
    assert _native.workspace_bytes(t, _native.LEG_TDW) > 0


def test_packed_sizes():
    # SIMT layout: plain [tap][Cout][Cin]; tcgen05 layouts hold at least the padded weight
    assert _native.packed_weight_bytes(_d(cin=5, cout=7, force=1), _native.LEG_DX) == 5 * 7 * 27 * 2
    assert _native.packed_weight_bytes(_d(cin=5, cout=7), _native.LEG_DX) >= 8 * 5 * 27 * 2
    assert _native.packed_weight_bytes(_d(), _native.LEG_FWD) >= 24 * 24 * 27 * 2


def test_null_descriptor_rejected():
    lib = _native.lib()
    assert lib.r4c_plan_kernel(None, 0) == -1
    assert lib.r4c_conv3d_fwd(None, None, None, None, None, None, 0, None) == -1


def _x(xs, ws, s, p, dl, g, dt=torch.bfloat16):
    return _native.make_convex_desc(xs, ws, (s,) * 3, (p,) * 3, (dl,) * 3, g, dt)


def test_convex_plan_and_sizes():
    # k2s2 downsampling conv: the tcgen05 transpose-conv kernels (packed weight in the workspace)
    d = _x((2, 16, 8, 12, 16), (32, 16, 2, 2, 2), 2, 0, 1, 1)
    assert _native.convex_plan(d) == _native.KERNEL_TC
    assert _native.convex_out_shape(d) == (2, 32, 4, 6, 8)
    lib = _native.lib()
    assert lib.r4c_convex_workspace_size(d, _native.LEG_FWD) > 0
    assert lib.r4c_convex_workspace_size(d, _native.LEG_DW) > 0
    # odd extents, fp32 or odd channels: SIMT
    assert _native.convex_plan(_x((2, 16, 7, 12, 16), (32, 16, 2, 2, 2), 2, 0, 1, 1)) == _native.KERNEL_GENERIC
    assert _native.convex_plan(_x((2, 16, 8, 12, 16), (32, 16, 2, 2, 2), 2, 0, 1, 1, torch.float32)) == \
        _native.KERNEL_GENERIC
    # strided, dilated, grouped: SIMT, dW split-K partials in the workspace only
    g = _x((1, 8, 10, 11, 12), (16, 4, 3, 3, 3), 2, 2, 2, 2)
    assert _native.convex_plan(g) == _native.KERNEL_GENERIC
    assert _native.convex_out_shape(g) == (1, 16, 5, 6, 6)   # (i + 4 - 4 - 1) // 2 + 1
    assert lib.r4c_convex_workspace_size(g, _native.LEG_FWD) == 0
    assert lib.r4c_convex_workspace_size(g, _native.LEG_DW) >= 16 * 4 * 27 * 4
    # invalid: channels not divisible by groups, zero stride
    assert _native.convex_plan(_x((1, 6, 4, 4, 4), (4, 2, 3, 3, 3), 1, 1, 1, 4)) == -1
    assert _native.convex_plan(_x((1, 8, 4, 4, 4), (8, 8, 3, 3, 3), 0, 1, 1, 1)) == -2
