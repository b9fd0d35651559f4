"""Python API surface and CPU behaviour of the drop-ins (no GPU)."""
import os
import subprocess
import sys

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import rdna4_conv3d
from conftest import ROOT
from rdna4_conv3d import Conv3dWmma, ConvTranspose3dWmma, conv3d_plan, conv3d_wmma, swap_conv3d

PKG = os.path.join(ROOT, "rdna4-conv3d-wmma_b200")


def test_public_names_match_reference():
    assert set(rdna4_conv3d.__all__) == {
        "Conv3dWmma", "ConvTranspose3dWmma", "conv3d_plan", "conv3d_wmma", "swap_conv3d",
        "wmma_dw", "wmma_dx", "wmma_fwd", "wmma_ok_dw", "wmma_ok_dx", "wmma_ok_fwd"}
    assert rdna4_conv3d.__version__ == "0.1.0"
    # the function shadows the submodule attribute, like the reference
    assert callable(rdna4_conv3d.conv3d_wmma)
    assert "rdna4_conv3d.conv3d_wmma" in sys.modules


def test_modules_are_state_dict_compatible():
    a = nn.Conv3d(4, 6, 3, padding=1)
    b = Conv3dWmma(4, 6, 3, padding=1)
    b.load_state_dict(a.state_dict())
    assert set(a.state_dict()) == set(b.state_dict())
    t = nn.ConvTranspose3d(6, 3, 2, stride=2)
    u = ConvTranspose3dWmma(6, 3, 2, stride=2)
    u.load_state_dict(t.state_dict())


def test_swap_copies_weights_and_keeps_attributes():
    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.c = nn.Conv3d(4, 8, 3, padding=1)
            self.seq = nn.Sequential(nn.Conv3d(8, 8, 1), nn.ReLU(), nn.Conv3d(8, 2, 3, padding=1,
                                                                              padding_mode="replicate"))
            self.t = nn.ConvTranspose3d(8, 4, 2, stride=2)

    m = M().double()
    w = m.c.weight.data.clone()
    n = swap_conv3d(m)
    assert n == 3
    assert isinstance(m.c, Conv3dWmma) and isinstance(m.seq[0], Conv3dWmma)
    assert type(m.t) is nn.ConvTranspose3d          # ConvTranspose3d is not swapped
    assert torch.equal(m.c.weight.data, w)
    assert m.c.weight.dtype == torch.float64        # dtype preserved
    assert m.seq[2].padding_mode == "replicate"     # padding_mode preserved
    assert swap_conv3d(m) == 0                      # already swapped


def test_cpu_forward_is_stock_path():
    torch.manual_seed(0)
    conv = Conv3dWmma(3, 5, 3, padding=1)
    x = torch.randn(1, 3, 4, 5, 6)
    torch.testing.assert_close(conv(x), F.conv3d(x, conv.weight, conv.bias, 1, 1))
    tr = ConvTranspose3dWmma(5, 2, 2, stride=2)
    y = torch.randn(1, 5, 2, 3, 4)
    torch.testing.assert_close(tr(y), F.conv_transpose3d(y, tr.weight, tr.bias, 2))


def test_conv3d_wmma_groups_fallback():
    torch.manual_seed(0)
    x = torch.randn(1, 4, 4, 4, 4)
    w = torch.randn(4, 2, 3, 3, 3)
    torch.testing.assert_close(conv3d_wmma(x, w, None, 1, 1, 1, 2), F.conv3d(x, w, None, 1, 1, 1, 2))


def test_plan_without_gpu_is_stock():
    assert conv3d_plan(24, 24, 3) == {"fwd": "miopen", "dw": "miopen", "dx": "miopen"}


def _plan_in_subprocess(env_extra):
    env = dict(os.environ)
    env.pop("RDNA4_CONV3D_BACKEND", None)
    env.pop("BIOHUB_CONV3D_BACKEND", None)
    env.update(env_extra)
    code = ("import sys; sys.path.insert(0, %r); from rdna4_conv3d import conv3d_plan; "
            "print(conv3d_plan(24, 24, 3)['fwd'], conv3d_plan(24, 24, 5)['fwd'])" % PKG)
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, check=True)
    return out.stdout.split()


@pytest.mark.parametrize("env,want", [
    ({}, ["miopen", "miopen"]),                                  # hybrid, no sm_100 device
    ({"RDNA4_CONV3D_BACKEND": "wmma"}, ["wmma", "miopen"]),
    ({"RDNA4_CONV3D_BACKEND": "B200"}, ["wmma", "miopen"]),
    ({"BIOHUB_CONV3D_BACKEND": "wmma"}, ["wmma", "miopen"]),      # alias
    ({"RDNA4_CONV3D_BACKEND": "miopen", "BIOHUB_CONV3D_BACKEND": "wmma"}, ["miopen", "miopen"]),
    ({"RDNA4_CONV3D_BACKEND": "torch"}, ["miopen", "miopen"]),
])
def test_backend_env(env, want):
    assert _plan_in_subprocess(env) == want


def test_in_scope_cuda_call_without_gpu_raises():
    """With the kernels forced on but no CUDA tensor, the native layer refuses
    loudly instead of computing on the host."""
    from rdna4_conv3d import _native
    with pytest.raises(_native.NativeError):
        _native.pack_weight(_native.make_desc(1, 4, 4, 4, 8, 8, 3, (1, 1, 1), torch.bfloat16), 0,
                            torch.randn(8, 8, 3, 3, 3))


def test_fuse_bn_relu_structure_and_cpu_fallback():
    """(BatchNorm3d, ReLU) pairs become (BatchNormReLU3d, Identity) with the
    same state_dict; on CPU the module runs stock BatchNorm3d + ReLU."""
    from rdna4_conv3d.bn_relu import BatchNormReLU3d, fuse_bn_relu
    from rdna4_conv3d.unet3d import unet3d
    torch.manual_seed(0)
    stock = unet3d(8, levels=2, wmma=False)
    fused = unet3d(8, levels=2, wmma=False, fuse_bn=True)
    assert sum(isinstance(m, BatchNormReLU3d) for m in fused.modules()) == 6   # 3 blocks x 2
    assert set(stock.state_dict()) == set(fused.state_dict())
    fused.load_state_dict(stock.state_dict())
    x = torch.randn(2, 1, 8, 8, 8).contiguous(memory_format=torch.channels_last_3d)
    torch.testing.assert_close(fused(x), stock(x))
    for a, b in zip(stock.buffers(), fused.buffers()):    # running statistics updated alike
        torch.testing.assert_close(a, b)
    seq = torch.nn.Sequential(torch.nn.BatchNorm3d(4), torch.nn.ReLU(), torch.nn.BatchNorm3d(4))
    assert fuse_bn_relu(seq) == 1 and isinstance(seq[1], torch.nn.Identity)
    assert type(seq[2]) is torch.nn.BatchNorm3d


def test_torch_ops_registered_with_fake_kernels():
    """torch.ops.r4c.* exist and their fake kernels give shapes, dtypes and the
    NDHWC layout without running anything (FakeTensor on a CPU-only host)."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    import rdna4_conv3d  # noqa: F401
    cl = torch.channels_last_3d
    with FakeTensorMode():
        x = torch.empty(2, 24, 8, 16, 16, dtype=torch.bfloat16).contiguous(memory_format=cl)
        w = torch.empty(48, 24, 3, 3, 3)
        y = torch.ops.r4c.conv3d_fwd(x, w, None, [1, 1, 1])
        assert y.shape == (2, 48, 8, 16, 16) and y.dtype == torch.bfloat16
        assert y.is_contiguous(memory_format=cl)
        y0 = torch.ops.r4c.conv3d_fwd(x, w, None, [0, 1, 1])
        assert y0.shape == (2, 48, 6, 16, 16)
        dx = torch.ops.r4c.conv3d_dx(y, w, list(x.shape), [1, 1, 1])
        assert dx.shape == x.shape and dx.is_contiguous(memory_format=cl)
        dw, db = torch.ops.r4c.conv3d_dw(x, y, list(w.shape), [1, 1, 1], True)
        assert dw.shape == w.shape and dw.dtype == torch.float32 and db.shape == (48,)
        _, db0 = torch.ops.r4c.conv3d_dw(x, y, list(w.shape), [1, 1, 1], False)
        assert db0.shape == (0,)
        wt = torch.empty(24, 12, 2, 2, 2)
        t = torch.ops.r4c.tconv_fwd(x, wt, None)
        assert t.shape == (2, 12, 16, 32, 32)
        assert torch.ops.r4c.tconv_dx(t, wt, list(x.shape)).shape == x.shape
        tdw, tdb = torch.ops.r4c.tconv_dw(x, t, list(wt.shape), True)
        assert tdw.shape == wt.shape and tdb.shape == (12,)


def test_unet_fused_skip_path_on_cpu_matches_stock():
    """The fused-skip forward (forward_pool + skip_cat) falls back to stock ops
    on CPU and computes the same network, gradients included."""
    from rdna4_conv3d.unet3d import unet3d
    torch.manual_seed(0)
    stock = unet3d(4, levels=3, wmma=False).double()
    fused = unet3d(4, levels=3, wmma=False, fuse_bn=True).double()
    fused.load_state_dict(stock.state_dict())
    assert fused._fused_skips() and not stock._fused_skips()
    x = torch.randn(2, 1, 8, 8, 8, dtype=torch.float64)
    ys, yf = stock(x), fused(x)
    torch.testing.assert_close(yf, ys)
    gy = torch.randn_like(ys)
    ys.backward(gy)
    yf.backward(gy)
    for (n, a), b in zip(stock.named_parameters(), fused.parameters()):
        torch.testing.assert_close(b.grad, a.grad, msg=n)
