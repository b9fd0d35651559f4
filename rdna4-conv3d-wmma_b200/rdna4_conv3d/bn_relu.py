"""BatchNorm3d + ReLU in one pair of fused kernels per direction.

The reference's UNet blocks are Conv3d -> BatchNorm3d -> ReLU on the vendor
library (benches/unet_e2e.py:13-20 of the reference), BatchNorm costing about
11 ms of its step (the reference's docs/DESIGN.md:66). ``BatchNormReLU3d`` is an
``nn.BatchNorm3d`` (same parameters, buffers and state_dict) whose training
forward, on a CUDA NDHWC bf16/fp16 activation with a multiple of 8 channels,
runs the library's r4c_bn_* kernels: one statistics pass, a per-channel
finalize (running statistics updated as BatchNorm3d does), one
normalise+ReLU pass; backward: one reduction pass over dY and x, one dX pass.
Everything else (eval mode, CPU, other layouts or dtypes) runs the stock
BatchNorm3d followed by ReLU.

``fuse_bn_relu(model)`` swaps every (BatchNorm3d, ReLU) pair that follows each
other in an ``nn.Sequential`` for (BatchNormReLU3d, Identity): module names
and state_dict keys stay the same.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native

_HALF = (torch.float16, torch.bfloat16)


class BNReLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, running_mean, running_var, momentum, eps, relu, sums_hook, pivot=None):
        gamma = None if weight is None else weight.detach().float().contiguous()
        beta = None if bias is None else bias.detach().float().contiguous()
        y, mi, ss, count = _native.bn_relu_forward(x, gamma, beta, running_mean, running_var, momentum, eps, relu,
                                                   sums_hook, pivot)
        ctx.save_for_backward(x, mi, ss)
        ctx.count, ctx.relu, ctx.sums_hook = count, relu, sums_hook
        ctx.wdtype = None if weight is None else weight.dtype
        ctx.bdtype = None if bias is None else bias.dtype
        return y

    @staticmethod
    def backward(ctx, gy):
        x, mi, ss = ctx.saved_tensors
        gy = gy.contiguous(memory_format=torch.channels_last_3d)
        if gy.dtype != x.dtype:
            gy = gy.to(x.dtype)
        dx, dg, db = _native.bn_relu_backward(gy, x, mi, ss, ctx.count, ctx.relu, ctx.needs_input_grad[0],
                                              ctx.sums_hook)
        dg = dg.to(ctx.wdtype) if ctx.wdtype is not None and ctx.needs_input_grad[1] else None
        db = db.to(ctx.bdtype) if ctx.bdtype is not None and ctx.needs_input_grad[2] else None
        return dx, dg, db, None, None, None, None, None, None, None


class BNReLUPoolFn(torch.autograd.Function):
    """(buf, p) = (lead empty channels + relu(bn(x)), maxpool2(relu(bn(x))))."""

    @staticmethod
    def forward(ctx, x, weight, bias, running_mean, running_var, momentum, eps, lead, sums_hook=None, pivot=None):
        gamma = None if weight is None else weight.detach().float().contiguous()
        beta = None if bias is None else bias.detach().float().contiguous()
        _, mi, af, count = _native.bn_relu_forward(x, gamma, beta, running_mean, running_var, momentum, eps, True,
                                                   sums_hook, pivot, apply=False)
        buf, p, am = _native.bn_relu_pool_forward(x, mi, af, lead)
        ctx.save_for_backward(x, mi, af, am)
        ctx.count, ctx.lead, ctx.sums_hook = count, lead, sums_hook
        ctx.wdtype = None if weight is None else weight.dtype
        ctx.bdtype = None if bias is None else bias.dtype
        return buf, p

    @staticmethod
    def backward(ctx, gbuf, gp):
        x, mi, af, am = ctx.saved_tensors
        cl = torch.channels_last_3d
        if gbuf is None:
            gbuf = torch.zeros((x.shape[0], ctx.lead + x.shape[1]) + tuple(x.shape[2:]), dtype=x.dtype,
                               device=x.device, memory_format=cl)
        if gp is None:
            gp = torch.zeros((x.shape[0], x.shape[1]) + tuple(s // 2 for s in x.shape[2:]), dtype=x.dtype,
                             device=x.device, memory_format=cl)
        gbuf = gbuf.to(x.dtype).contiguous(memory_format=cl)
        gp = gp.to(x.dtype).contiguous(memory_format=cl)
        dx, dg, db = _native.bn_relu_pool_backward(gbuf, ctx.lead, gp, x, mi, af, ctx.count, ctx.needs_input_grad[0],
                                                   ctx.sums_hook, argmax=am)
        dg = dg.to(ctx.wdtype) if ctx.wdtype is not None and ctx.needs_input_grad[1] else None
        db = db.to(ctx.bdtype) if ctx.bdtype is not None and ctx.needs_input_grad[2] else None
        return dx, dg, db, None, None, None, None, None, None, None


class SkipCatFn(torch.autograd.Function):
    """Write `up` into channels [0, lead) of `buf` in place (the rest of buf
    already holds the skip connection): torch.cat([up, skip], 1) without
    copying the skip."""

    @staticmethod
    def forward(ctx, up, buf, lead):
        buf[:, :lead].copy_(up)
        ctx.mark_dirty(buf)
        ctx.lead = lead
        return buf

    @staticmethod
    def backward(ctx, g):
        return g[:, :ctx.lead], g, None


def skip_cat(up: torch.Tensor, buf: torch.Tensor, lead: int) -> torch.Tensor:
    return SkipCatFn.apply(up, buf, lead)


class BatchNormReLU3d(nn.BatchNorm3d):
    """BatchNorm3d followed by ReLU (``relu=False``: BatchNorm3d alone)."""

    def __init__(self, num_features, eps=1e-5, momentum=0.1, affine=True, track_running_stats=True, relu=True,
                 device=None, dtype=None):
        super().__init__(num_features, eps, momentum, affine, track_running_stats, device=device, dtype=dtype)
        self.relu = relu

    def _sums_hook(self):
        """Per-channel sums reduction across ranks (None: this process's data only)."""
        return None

    def _pivot(self):
        """Statistics pivot shared by every rank (None: the first voxel)."""
        return None

    def _fused_ok(self, x) -> bool:
        from .conv3d_wmma import _wmma_hw
        if not (x.is_cuda and x.dim() == 5 and x.dtype in _HALF and _wmma_hw()):
            return False
        if not (self.training or not self.track_running_stats):
            return False      # eval mode with running statistics: stock path
        if x.shape[1] % 8 or not x.is_contiguous(memory_format=torch.channels_last_3d) or x.data_ptr() % 16:
            return False
        if self.running_mean is not None and self.running_mean.dtype != torch.float32:
            return False
        return True

    def forward(self, x):
        if not self._fused_ok(x):
            y = super().forward(x)
            return F.relu(y) if self.relu else y
        if self.training and self.track_running_stats and self.num_batches_tracked is not None:
            self.num_batches_tracked.add_(1)
            mom = 1.0 / float(self.num_batches_tracked) if self.momentum is None else self.momentum
        else:
            mom = 0.0 if self.momentum is None else self.momentum
        rm = self.running_mean if (self.training and self.track_running_stats) else None
        rv = self.running_var if (self.training and self.track_running_stats) else None
        return BNReLUFn.apply(x, self.weight, self.bias, rm, rv, float(mom), float(self.eps), bool(self.relu),
                              self._sums_hook(), self._pivot())

    def forward_pool(self, x, lead: int):
        """(buf, p): buf an NDHWC tensor of ``lead`` + C channels whose last C
        hold relu(bn(x)) — the skip connection, placed where the decoder's
        concatenation wants it — and p = max_pool3d(relu(bn(x)), 2). One
        fused kernel set on the supported path, stock ops otherwise."""
        even = x.dim() == 5 and all(int(s) % 2 == 0 for s in x.shape[2:])
        if not (self.relu and even and self._fused_ok(x) and self.training and self.track_running_stats):
            y = self.forward(x)
            head = torch.empty((x.shape[0], lead) + tuple(x.shape[2:]), dtype=y.dtype, device=y.device)
            buf = torch.cat([head, y], dim=1).contiguous(memory_format=torch.channels_last_3d)
            return buf, F.max_pool3d(y, 2)
        self.num_batches_tracked.add_(1)
        mom = 1.0 / float(self.num_batches_tracked) if self.momentum is None else self.momentum
        return BNReLUPoolFn.apply(x, self.weight, self.bias, self.running_mean, self.running_var, float(mom),
                                  float(self.eps), int(lead), self._sums_hook(), self._pivot())


def fuse_bn_relu(model: nn.Module) -> int:
    """Replace each (BatchNorm3d, ReLU) pair inside an nn.Sequential with
    (BatchNormReLU3d, Identity), copying the BatchNorm's state. Returns the
    number of pairs fused."""
    count = 0
    for child in model.children():
        count += fuse_bn_relu(child)
    if isinstance(model, nn.Sequential):
        names = list(model._modules.keys())
        for a, b in zip(names, names[1:]):
            bn, act = model._modules[a], model._modules[b]
            if type(bn) is nn.BatchNorm3d and isinstance(act, nn.ReLU):
                ref = bn.weight if bn.affine else bn.running_mean
                new = BatchNormReLU3d(bn.num_features, bn.eps, bn.momentum, bn.affine, bn.track_running_stats,
                                      device=None if ref is None else ref.device,
                                      dtype=None if ref is None else ref.dtype)
                new.load_state_dict(bn.state_dict())
                new.train(bn.training)
                model._modules[a] = new
                model._modules[b] = nn.Identity()
                count += 1
    return count
