"""Module / autograd behaviour on a B200, against the stock PyTorch path.

Ports the reference's GPU tests (tests/test_conv3d.py:24-75 of the reference:
swap, fallback on unsupported geometry, fp16 parity with its tolerances) and
adds what the reference never pinned: channels_last inputs, autocast, the
k2s2 transpose conv module, and a small UNet's AMP loss trajectory.
"""
import sys

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import oracle as O
from rdna4_conv3d import Conv3dWmma, ConvTranspose3dWmma, conv3d_wmma, swap_conv3d

pytestmark = pytest.mark.gpu


def test_swap_copies_weights_on_cuda(cuda_ready):
    m = nn.Sequential(nn.Conv3d(4, 8, 3, padding=1)).cuda()
    w = m[0].weight.data.clone()
    assert swap_conv3d(m) == 1
    assert isinstance(m[0], Conv3dWmma)
    assert m[0].weight.is_cuda and torch.equal(m[0].weight.data, w)


def test_fallback_matches_conv3d_on_unsupported_geom(cuda_ready):
    torch.manual_seed(0)
    x = torch.randn(1, 4, 8, 8, 8, device="cuda")
    conv = Conv3dWmma(4, 5, 3, stride=2, padding=1).cuda()
    torch.testing.assert_close(conv(x), F.conv3d(x, conv.weight, conv.bias, 2, 1), atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("n,cin,cout,d,h,w,k,pad", [
    (2, 5, 7, 9, 11, 13, 3, 1), (2, 24, 1, 8, 16, 16, 1, 0), (1, 24, 24, 8, 16, 16, 3, 1),
    (1, 1, 24, 8, 16, 16, 3, 1)])
def test_close_to_fp16_stock(cuda_ready, n, cin, cout, d, h, w, k, pad):
    """The reference's own parity test, same tolerances, vs fp16 cuDNN."""
    torch.manual_seed(0)
    x = torch.randn(n, cin, d, h, w, device="cuda", dtype=torch.float16, requires_grad=True)
    wt = torch.randn(cout, cin, k, k, k, device="cuda", dtype=torch.float16, requires_grad=True)
    b = torch.randn(cout, device="cuda", dtype=torch.float16, requires_grad=True)
    x2, w2, b2 = (t.detach().requires_grad_(True) for t in (x, wt, b))
    y = conv3d_wmma(x, wt, b, 1, pad)
    y2 = F.conv3d(x2, w2, b2, 1, pad)
    torch.testing.assert_close(y, y2, atol=2e-2, rtol=8e-2)
    go = torch.randn_like(y2)
    y.backward(go)
    y2.backward(go)
    torch.testing.assert_close(x.grad, x2.grad, atol=8e-2, rtol=8e-2)
    torch.testing.assert_close(wt.grad, w2.grad, atol=0.5, rtol=0.5)
    torch.testing.assert_close(b.grad.float(), b2.grad.float(), atol=0.5, rtol=1e-2)


@pytest.mark.parametrize("layout", ["ncdhw", "ndhwc"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_module_grads_vs_cpu_fp32(cuda_ready, layout, dtype):
    torch.manual_seed(0)
    ref = nn.Conv3d(24, 16, 3, padding=1)
    mod = Conv3dWmma(24, 16, 3, padding=1).cuda()
    mod.load_state_dict(ref.state_dict())
    x = torch.randn(2, 24, 6, 10, 12)
    xg = x.to(dtype).cuda()
    if layout == "ndhwc":
        xg = xg.contiguous(memory_format=torch.channels_last_3d)
    xg.requires_grad_(True)
    y = mod(xg)
    assert y.dtype == dtype and y.is_contiguous(
        memory_format=torch.channels_last_3d if layout == "ndhwc" else torch.contiguous_format)
    go = torch.randn(y.shape)
    y.backward(go.to(dtype).cuda())
    xr = x.to(dtype).float().requires_grad_(True)
    yr = ref(xr)
    yr.backward(go.to(dtype).float())
    assert O.max_rel(y.float().cpu(), yr) <= 2e-2
    assert O.max_rel(xg.grad.float().cpu(), xr.grad) <= 2e-2
    assert O.norm_rel(mod.weight.grad.cpu(), ref.weight.grad) <= 3e-2
    assert O.norm_rel(mod.bias.grad.cpu(), ref.bias.grad) <= 3e-2
    assert mod.weight.grad.dtype == torch.float32


def test_autocast_casts_outside_function(cuda_ready):
    torch.manual_seed(0)
    mod = Conv3dWmma(8, 8, 3, padding=1).cuda()
    x = torch.randn(1, 8, 4, 6, 8, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = mod(x)
        ys = F.conv3d(x, mod.weight, mod.bias, 1, 1)
    assert y.dtype == ys.dtype == torch.bfloat16
    y.float().sum().backward()
    assert mod.weight.grad.dtype == torch.float32


def test_tconv_module(cuda_ready):
    torch.manual_seed(0)
    ref = nn.ConvTranspose3d(16, 8, 2, stride=2)
    mod = ConvTranspose3dWmma(16, 8, 2, stride=2).cuda()
    mod.load_state_dict(ref.state_dict())
    x = torch.randn(2, 16, 3, 4, 5)
    xg = x.to(torch.bfloat16).cuda().requires_grad_(True)
    y = mod(xg)
    go = torch.randn(y.shape)
    y.backward(go.to(torch.bfloat16).cuda())
    xr = x.to(torch.bfloat16).float().requires_grad_(True)
    yr = ref(xr)
    yr.backward(go.to(torch.bfloat16).float())
    assert O.max_rel(y.float().cpu(), yr) <= 2e-2
    assert O.max_rel(xg.grad.float().cpu(), xr.grad) <= 2e-2
    assert O.norm_rel(mod.weight.grad.cpu(), ref.weight.grad) <= 3e-2
    # output_size that disagrees with 2x falls back to the stock module
    out = mod(x.cuda(), output_size=(7, 9, 11))
    assert out.shape[-3:] == (7, 9, 11)
    torch.testing.assert_close(out, ref.cuda()(x.cuda(), output_size=(7, 9, 11)))


def _block(cin, cout, conv):
    return nn.Sequential(conv(cin, cout, 3, padding=1), nn.BatchNorm3d(cout), nn.ReLU(inplace=True),
                         conv(cout, cout, 3, padding=1), nn.BatchNorm3d(cout), nn.ReLU(inplace=True))


class _TinyUNet(nn.Module):
    def __init__(self, conv, tr, base=8):
        super().__init__()
        self.e1 = _block(1, base, conv)
        self.e2 = _block(base, 2 * base, conv)
        self.up = tr(2 * base, base, 2, stride=2)
        self.d1 = _block(2 * base, base, conv)
        self.head = conv(base, 4, 1)

    def forward(self, x):
        a = self.e1(x)
        b = self.e2(F.max_pool3d(a, 2))
        return self.head(self.d1(torch.cat([self.up(b), a], 1)))


def test_unet_amp_loss_parity(cuda_ready):
    """40 AMP steps with Adam: |loss_ours - loss_stock| <= 1e-3 at every step."""
    torch.manual_seed(0)
    stock = _TinyUNet(nn.Conv3d, nn.ConvTranspose3d).cuda()
    ours = _TinyUNet(Conv3dWmma, ConvTranspose3dWmma).cuda()
    ours.load_state_dict(stock.state_dict())
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(2, 1, 16, 32, 32, device="cuda", generator=g)
    tgt = torch.randint(0, 4, (2, 16, 32, 32), device="cuda", generator=g)
    losses = []
    for net in (stock, ours):
        opt = torch.optim.Adam(net.parameters(), lr=1e-3)
        hist = []
        for _ in range(40):
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = F.cross_entropy(net(x), tgt)
            loss.backward()
            opt.step()
            hist.append(float(loss.detach()))
        losses.append(hist)
    diffs = [abs(a - b) for a, b in zip(*losses)]
    assert max(diffs) <= 1e-3, (max(diffs), losses[0][-1], losses[1][-1])   # absolute
