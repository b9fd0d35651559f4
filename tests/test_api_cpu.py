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
