"""UNet3D: the application model the conv hot path is measured in.

The reference's headline protocol (README.md:57-66 of the reference) is one
AMP training step (forward, backward, Adam) of a 3D UNet whose blocks are two
(Conv3d k3 + BatchNorm3d + ReLU) layers, with MaxPool3d(2) down and
ConvTranspose3d k2 s2 up plus a skip concatenation; its benches ship a
two-level version of that model (benches/unet_e2e.py:12-38 of the reference).
This is the full-depth model the benchmark configurations name: ``levels``
resolution levels with ``base * 2**i`` channels (base 24 -> 24/48/96/192), a
1x1x1 head to ``n_classes``.

``conv`` / ``tconv`` choose the layer classes, so the same architecture is
built on stock PyTorch (the parity baseline) or on this package's kernels
(``Conv3dWmma`` / ``ConvTranspose3dWmma``); ``unet3d(..., wmma=True)`` does the
latter. Activations should be channels_last_3d (NDHWC) end to end.
"""
from __future__ import annotations

from typing import List

import torch
import torch.nn as nn

from .conv3d_wmma import Conv3dWmma, ConvTranspose3dWmma


def conv_block(cin: int, cout: int, conv=nn.Conv3d) -> nn.Sequential:
    """Two (k3 pad1 conv + BatchNorm3d + ReLU) layers."""
    return nn.Sequential(
        conv(cin, cout, 3, padding=1), nn.BatchNorm3d(cout), nn.ReLU(inplace=True),
        conv(cout, cout, 3, padding=1), nn.BatchNorm3d(cout), nn.ReLU(inplace=True),
    )


class UNet3D(nn.Module):
    def __init__(self, in_channels: int = 1, n_classes: int = 4, base: int = 24, levels: int = 4,
                 conv=nn.Conv3d, tconv=nn.ConvTranspose3d):
        super().__init__()
        ch = [base * 2 ** i for i in range(levels)]
        self.channels = ch
        self.enc = nn.ModuleList(
            [conv_block(in_channels if i == 0 else ch[i - 1], ch[i], conv) for i in range(levels)])
        self.pool = nn.MaxPool3d(2)
        self.up = nn.ModuleList([tconv(ch[i + 1], ch[i], 2, stride=2) for i in reversed(range(levels - 1))])
        self.dec = nn.ModuleList([conv_block(2 * ch[i], ch[i], conv) for i in reversed(range(levels - 1))])
        self.head = conv(ch[0], n_classes, 1)

    def _fused_skips(self) -> bool:
        from .bn_relu import BatchNormReLU3d
        return all(isinstance(b[-2], BatchNormReLU3d) and isinstance(b[-1], nn.Identity) for b in self.enc)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._fused_skips():
            return self._forward_fused(x)
        skips: List[torch.Tensor] = []
        for i, block in enumerate(self.enc):
            x = block(x if i == 0 else self.pool(x))
            skips.append(x)
        x = skips.pop()
        for up, dec in zip(self.up, self.dec):
            x = dec(torch.cat([up(x), skips.pop()], dim=1))
        return self.head(x)


    def _forward_fused(self, x: torch.Tensor) -> torch.Tensor:
        """Same network, with each encoder level's last BatchNorm+ReLU also
        doing the MaxPool3d(2) and writing its output (the skip connection)
        straight into the channels of the decoder's concatenation buffer; the
        up-conv then writes its output into the buffer's first channels."""
        from .bn_relu import skip_cat
        bufs = []
        last = len(self.enc) - 1
        for i, block in enumerate(self.enc):
            for m in list(block)[:-2]:
                x = m(x)
            if i == last:
                x = block[-2](x)
            else:
                lead = self.channels[i]           # the up-conv at this level outputs ch[i] channels
                buf, x = block[-2].forward_pool(x, lead)
                bufs.append((buf, lead))
        for up, dec in zip(self.up, self.dec):
            buf, lead = bufs.pop()
            # the up-conv writes into the buffer's first channels when it can
            x = dec(up.forward_into(x, buf, lead) if hasattr(up, "forward_into") else skip_cat(up(x), buf, lead))
        return self.head(x)


def unet3d(base: int = 24, levels: int = 4, in_channels: int = 1, n_classes: int = 4, wmma: bool = True,
           device=None, fuse_bn: bool = None) -> UNet3D:
    """The UNet3D on this package's kernels (``wmma=True``) or on stock PyTorch,
    channels_last_3d parameters on ``device``. ``fuse_bn`` (default: same as
    ``wmma``) runs each BatchNorm3d + ReLU pair on the fused kernels; the
    state_dict keys are those of the stock model either way."""
    conv, tconv = (Conv3dWmma, ConvTranspose3dWmma) if wmma else (nn.Conv3d, nn.ConvTranspose3d)
    net = UNet3D(in_channels, n_classes, base, levels, conv, tconv)
    if wmma if fuse_bn is None else fuse_bn:
        from .bn_relu import fuse_bn_relu
        fuse_bn_relu(net)
    if device is not None:
        net = net.to(device)
    net = net.to(memory_format=torch.channels_last_3d)
    if wmma:
        # activations are NDHWC, but conv weights stay in PyTorch's OIDHW
        # order: the packing kernels read that order and the weight
        # gradients come back in it, so neither the packing nor the gradient
        # accumulation needs a layout copy
        for m in net.modules():
            if isinstance(m, (nn.Conv3d, nn.ConvTranspose3d)):
                m.weight.data = m.weight.data.contiguous()
    return net


def conv_flops_per_sample(net: UNet3D, spatial, in_channels: int = 1) -> float:
    """Algorithmic conv + transpose-conv FLOPs of one forward pass of one
    sample (2 * output voxels * Cin * Cout * k^3 per conv; padding MACs not
    counted). Forward + backward is three times this."""
    d, h, w = spatial
    total = 0.0
    for i, block in enumerate(net.enc):
        s = (d >> i) * (h >> i) * (w >> i)
        for m in block:
            if isinstance(m, nn.Conv3d):
                total += 2.0 * s * m.in_channels * m.out_channels * 27
    levels = len(net.enc)
    for j, (up, dec) in enumerate(zip(net.up, net.dec)):
        lvl = levels - 2 - j
        s = (d >> lvl) * (h >> lvl) * (w >> lvl)
        total += 2.0 * (s // 8) * up.in_channels * up.out_channels * 8
        for m in dec:
            if isinstance(m, nn.Conv3d):
                total += 2.0 * s * m.in_channels * m.out_channels * 27
    total += 2.0 * d * h * w * net.head.in_channels * net.head.out_channels
    return total
