"""Multi-GPU execution of the conv hot path over NCCL (NVLink / NVSwitch).

No reference counterpart: the reference is single-GPU only. Two modes:

* Batch-sharded data parallel: every rank runs its own samples; the fp32 dW
  and db of each conv are all-reduced on a side stream right after the dW
  kernel, while the dX kernel of the same layer runs on the compute stream
  (``data_parallel_grads`` / ``GradAllReducer``). Conv parameters handled this
  way must be excluded from DDP (``ddp_ignore_conv_params``).
* Depth-sharded single volume: each rank owns a contiguous slab of D planes;
  every k3 conv exchanges one plane with each D-neighbour into a local halo
  (``halo_exchange`` / ``DepthShardedConv3dFn``) and the weight gradient is
  all-reduced.
"""
from __future__ import annotations

import contextlib
import sys
from typing import List, Optional

import torch
import torch.distributed as dist


def _cw():
    return sys.modules["rdna4_conv3d.conv3d_wmma"]


class _Pending:
    def __init__(self, works, tensors, stream, scale):
        self.works = works
        self.tensors = tensors
        self.stream = stream
        self.scale = scale

    def wait(self):
        for w in self.works:
            w.wait()
        if self.stream is not None:
            torch.cuda.current_stream().wait_stream(self.stream)
            for t in self.tensors:
                t.record_stream(self.stream)
        if self.scale != 1.0:
            for t in self.tensors:
                t.mul_(self.scale)


class GradAllReducer:
    """All-reduce (sum, optionally averaged) of fp32 gradient tensors on a side stream."""

    def __init__(self, group=None, average: bool = True):
        self.group = group
        self.world = dist.get_world_size(group)
        self.average = average
        self.stream = torch.cuda.Stream() if torch.cuda.is_available() else None

    def reduce_async(self, tensors: List[torch.Tensor]) -> Optional[_Pending]:
        tensors = [t for t in tensors if t is not None]
        if not tensors or self.world == 1:
            return None
        scale = 1.0 / self.world if self.average else 1.0
        if self.stream is None or not tensors[0].is_cuda:
            works = [dist.all_reduce(t, group=self.group, async_op=True) for t in tensors]
            return _Pending(works, tensors, None, scale)
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            works = [dist.all_reduce(t, group=self.group, async_op=True) for t in tensors]
        return _Pending(works, tensors, self.stream, scale)


@contextlib.contextmanager
def data_parallel_grads(group=None, average: bool = True):
    """Inside this context, Conv3dWmma / ConvTranspose3dWmma backward passes
    all-reduce their dW/db across `group`, overlapped with the dX kernel."""
    cw = _cw()
    prev = cw._GRAD_REDUCER
    cw._GRAD_REDUCER = GradAllReducer(group, average)
    try:
        yield cw._GRAD_REDUCER
    finally:
        cw._GRAD_REDUCER = prev


def ddp_ignore_conv_params(model: torch.nn.Module) -> List[str]:
    """Names of Conv3dWmma / ConvTranspose3dWmma parameters, registered with
    DDP's ignore list so DDP does not reduce them a second time."""
    from .conv3d_wmma import Conv3dWmma, ConvTranspose3dWmma
    names = []
    for mname, mod in model.named_modules():
        if isinstance(mod, (Conv3dWmma, ConvTranspose3dWmma)):
            for pname, _ in mod.named_parameters(recurse=False):
                names.append(f"{mname}.{pname}" if mname else pname)
    torch.nn.parallel.DistributedDataParallel._set_params_and_buffers_to_ignore_for_model(model, names)
    return names


# ---------------------------------------------------------------------------
# Depth sharding
# ---------------------------------------------------------------------------
def _neighbours(group):
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    prev_r = rank - 1 if rank > 0 else None
    next_r = rank + 1 if rank < world - 1 else None
    to_global = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
    return (None if prev_r is None else to_global(prev_r)), (None if next_r is None else to_global(next_r))


def halo_exchange(x: torch.Tensor, halo: int = 1, group=None) -> torch.Tensor:
    """Return x (N, C, D, H, W) padded along D with `halo` planes from each
    D-neighbour (zeros at the volume ends). Point-to-point over NCCL."""
    prev_r, next_r = _neighbours(group)
    n, c, d, h, w = x.shape
    if d < halo:
        raise ValueError("depth slab thinner than the halo")
    out = torch.empty((n, c, d + 2 * halo, h, w), dtype=x.dtype, device=x.device,
                      memory_format=torch.channels_last_3d).zero_()
    out[:, :, halo:halo + d] = x
    ops = []
    lo = torch.empty((n, c, halo, h, w), dtype=x.dtype, device=x.device) if prev_r is not None else None
    hi = torch.empty((n, c, halo, h, w), dtype=x.dtype, device=x.device) if next_r is not None else None
    if prev_r is not None:
        ops.append(dist.P2POp(dist.isend, x[:, :, :halo].contiguous(), prev_r, group))
        ops.append(dist.P2POp(dist.irecv, lo, prev_r, group))
    if next_r is not None:
        ops.append(dist.P2POp(dist.isend, x[:, :, d - halo:].contiguous(), next_r, group))
        ops.append(dist.P2POp(dist.irecv, hi, next_r, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    if lo is not None:
        out[:, :, :halo] = lo
    if hi is not None:
        out[:, :, halo + d:] = hi
    return out


def halo_reduce(gx_padded: torch.Tensor, halo: int = 1, group=None) -> torch.Tensor:
    """Adjoint of halo_exchange: send the halo planes of a padded gradient back
    to the neighbours that own them and add what comes back into the slab."""
    prev_r, next_r = _neighbours(group)
    n, c, dp, h, w = gx_padded.shape
    d = dp - 2 * halo
    core = gx_padded[:, :, halo:halo + d].contiguous(memory_format=torch.channels_last_3d)
    ops = []
    from_prev = torch.empty((n, c, halo, h, w), dtype=core.dtype, device=core.device) \
        if prev_r is not None else None
    from_next = torch.empty((n, c, halo, h, w), dtype=core.dtype, device=core.device) \
        if next_r is not None else None
    if prev_r is not None:
        ops.append(dist.P2POp(dist.isend, gx_padded[:, :, :halo].contiguous(), prev_r, group))
        ops.append(dist.P2POp(dist.irecv, from_prev, prev_r, group))
    if next_r is not None:
        ops.append(dist.P2POp(dist.isend, gx_padded[:, :, halo + d:].contiguous(), next_r, group))
        ops.append(dist.P2POp(dist.irecv, from_next, next_r, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    if from_prev is not None:
        core[:, :, :halo] += from_prev
    if from_next is not None:
        core[:, :, d - halo:] += from_next
    return core


class DepthShardedConv3dFn(torch.autograd.Function):
    """k3 pad-1 Conv3d over a D-sharded volume: halo exchange, then the local
    conv with D padding 0 (the halo planes stand in for the neighbours'
    data); backward sends the halo part of dX back and all-reduces dW/db."""

    @staticmethod
    def forward(ctx, x, weight, bias, group):
        cw = _cw()
        xp = halo_exchange(x, 1, group)
        if x.is_cuda and cw._wmma_hw():
            y = cw._launch_fwd(xp, weight, bias, (0, 1, 1))
        else:
            y = torch.nn.functional.conv3d(xp, weight.to(xp.dtype),
                                           None if bias is None else bias.to(xp.dtype), 1, (0, 1, 1))
        ctx.save_for_backward(xp, weight)
        ctx.has_bias = bias is not None
        ctx.group = group
        return y

    @staticmethod
    def backward(ctx, go):
        cw = _cw()
        xp, weight = ctx.saved_tensors
        group = ctx.group
        go = go.to(xp.dtype)
        if xp.is_cuda and cw._wmma_hw():
            dw, db = cw._launch_wgrad(xp, go, weight.shape, (0, 1, 1), ctx.has_bias)
        else:
            acc = torch.promote_types(xp.dtype, torch.float32)  # fp32 accumulation, fp64 kept
            dw = torch.nn.grad.conv3d_weight(xp.to(acc), weight.shape, go.to(acc), 1, (0, 1, 1))
            db = go.to(acc).sum(dim=(0, 2, 3, 4)) if ctx.has_bias else None
        red = GradAllReducer(group, average=False)
        pending = red.reduce_async([dw, db])
        if xp.is_cuda and cw._wmma_hw():
            gxp = cw._launch_dgrad(go, weight, xp.shape, (0, 1, 1))
        else:
            gxp = torch.nn.grad.conv3d_input(xp.shape, weight.to(go.dtype), go, 1, (0, 1, 1))
        gx = halo_reduce(gxp, 1, group)
        if pending is not None:
            pending.wait()
        return gx, dw.to(weight.dtype), (None if db is None else db.to(weight.dtype)), None


def depth_sharded_conv3d(x, weight, bias=None, group=None):
    """k=3, pad=1 Conv3d of a D-sharded activation (each rank: its D slab)."""
    if tuple(weight.shape[2:]) != (3, 3, 3):
        raise ValueError("depth sharding is implemented for k=3, pad=1 convs")
    return DepthShardedConv3dFn.apply(x, weight, bias, group)
