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

from .bn_relu import BatchNormReLU3d


def _cw():
    return sys.modules["rdna4_conv3d.conv3d_wmma"]


class _Pending:
    def __init__(self, works, tensors, stream, scale, flat=None):
        self.works = works
        self.tensors = tensors
        self.stream = stream
        self.scale = scale
        self.flat = flat  # reduced (and already scaled) copy of the tensors, one buffer

    def wait(self):
        for w in self.works:
            w.wait()
        if self.stream is not None:
            torch.cuda.current_stream().wait_stream(self.stream)
            for t in self.tensors:
                t.record_stream(self.stream)
            if self.flat is not None:
                self.flat.record_stream(torch.cuda.current_stream())
        if self.flat is not None:
            off = 0
            for t in self.tensors:
                n = t.numel()
                t.copy_(self.flat[off:off + n].view_as(t))
                off += n
        elif self.scale != 1.0:
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
            if len(tensors) == 1 or any(t.dtype != tensors[0].dtype for t in tensors):
                works = [dist.all_reduce(t, group=self.group, async_op=True) for t in tensors]
                return _Pending(works, tensors, self.stream, scale)
            # one collective per call: the tensors (e.g. a layer's dW and db)
            # packed into one buffer, reduced and scaled on the side stream
            flat = torch.cat([t.reshape(-1) for t in tensors])
            dist.all_reduce(flat, group=self.group)
            if scale != 1.0:
                flat.mul_(scale)
        return _Pending([], tensors, self.stream, scale, flat)


class GradSync:
    """Batch-sharded data parallel gradients for a whole model, overlapped
    with the backward pass.

    A post-accumulate-grad hook on every trainable parameter hands its .grad
    to a side stream as soon as autograd has accumulated it; gradients are
    packed into buckets of about ``bucket_bytes`` and each full bucket is
    all-reduced (NCCL over NVLink) while the backward of the earlier layers
    still runs on the compute stream. When the backward pass ends the last
    bucket is flushed, the reduced values are copied back into the .grad
    tensors (divided by the world size when ``average``), and the compute
    stream waits for the side stream once. Every rank runs the same graph, so
    hooks fire and buckets flush in the same order on every rank.

    Each parameter must receive its gradient once per backward pass (true of
    the UNet and of every feed-forward conv net). Conv parameters reduced
    here need no DDP wrapper; buffers (BatchNorm running statistics) are
    not synchronised.
    """

    def __init__(self, model, group=None, average: bool = True, bucket_bytes: int = 8 << 20):
        """``model``: an nn.Module (all its trainable parameters) or an
        iterable of parameters."""
        self.group = group
        self.world = dist.get_world_size(group)
        self.average = average
        self.bucket_bytes = int(bucket_bytes)
        params = model.parameters() if isinstance(model, torch.nn.Module) else model
        self.params = [p for p in params if p.requires_grad]
        self.stream = None
        self.compute = None
        self._bucket: List[torch.Tensor] = []
        self._bucket_nbytes = 0
        self._inflight = []          # (work, flat, grads)
        self._armed = False
        self.buckets_flushed = 0
        self._handles = [p.register_post_accumulate_grad_hook(self._on_grad) for p in self.params]

    def remove(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles = []

    # -- hooks ------------------------------------------------------------
    def _on_grad(self, p: torch.Tensor) -> None:
        if self.world == 1 or p.grad is None:
            return
        g = p.grad
        if not self._armed:
            self._armed = True
            if g.is_cuda:
                self.compute = torch.cuda.current_stream(g.device)
                if self.stream is None:
                    self.stream = torch.cuda.Stream(g.device)
            torch.autograd.Variable._execution_engine.queue_callback(self._finish)
        self._bucket.append(g)
        self._bucket_nbytes += g.numel() * g.element_size()
        if self._bucket_nbytes >= self.bucket_bytes:
            self._flush()

    def _flush(self) -> None:
        grads, self._bucket, self._bucket_nbytes = self._bucket, [], 0
        if not grads:
            return
        self.buckets_flushed += 1
        if self.stream is None:                       # CPU (gloo): synchronous
            flat = torch.cat([g.reshape(-1) for g in grads])
            dist.all_reduce(flat, group=self.group)
            self._inflight.append((None, flat, grads))
            return
        self.stream.wait_stream(self.compute)         # the grads are complete on the compute stream
        with torch.cuda.stream(self.stream):
            flat = torch.cat([g.reshape(-1) for g in grads])
            work = dist.all_reduce(flat, group=self.group, async_op=True)
        self._inflight.append((work, flat, grads))

    def _finish(self) -> None:
        self._flush()
        scale = 1.0 / self.world if self.average else 1.0
        ctx = torch.cuda.stream(self.stream) if self.stream is not None else contextlib.nullcontext()
        with ctx:
            for work, flat, grads in self._inflight:
                if work is not None:
                    work.wait()
                if scale != 1.0:
                    flat.mul_(scale)
                off = 0
                for g in grads:
                    n = g.numel()
                    g.copy_(flat[off:off + n].view_as(g))
                    off += n
                    if self.stream is not None:
                        g.record_stream(self.stream)
        if self.stream is not None:
            self.compute.wait_stream(self.stream)
        self._inflight = []
        self._armed = False


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


def _plane(t: torch.Tensor, i: int, n: int = 1) -> torch.Tensor:
    """Planes [i, i+n) along D as a dense NDHWC tensor (a view when N == 1)."""
    v = t[:, :, i:i + n]
    if v.is_contiguous(memory_format=torch.channels_last_3d):
        return v
    return v.contiguous(memory_format=torch.channels_last_3d)


class _HaloRequest:
    def __init__(self, reqs, lo, hi):
        self.reqs, self.lo, self.hi = reqs, lo, hi

    def wait(self):
        for r in self.reqs:
            r.wait()
        return self.lo, self.hi


def _wire(t: torch.Tensor) -> torch.Tensor:
    """A plane in the layout the backend sends: NCCL takes dense NDHWC
    planes (a view for batch 1), gloo wants the default contiguous layout."""
    if t.is_cuda:
        return _plane(t, 0, t.shape[2])
    return t.contiguous()


def start_halo_exchange(x: torch.Tensor, group=None) -> _HaloRequest:
    """Post the exchange of one D plane with each D-neighbour (NCCL P2P over
    NVLink, gloo on CPU): this rank's first plane goes to the previous rank,
    its last plane to the next one. ``wait()`` returns (lo, hi): the
    neighbours' edge planes, None at the volume ends. The transfer runs on the
    communicator's own stream, so work enqueued before ``wait()`` overlaps it."""
    prev_r, next_r = _neighbours(group)
    n, c, d, h, w = x.shape
    ops = []
    lo = hi = None
    fmt = torch.channels_last_3d if x.is_cuda else torch.contiguous_format
    mk = lambda: torch.empty((n, c, 1, h, w), dtype=x.dtype, device=x.device, memory_format=fmt)  # noqa: E731
    if prev_r is not None:
        lo = mk()
        ops.append(dist.P2POp(dist.isend, _wire(x[:, :, :1]), prev_r, group))
        ops.append(dist.P2POp(dist.irecv, lo, prev_r, group))
    if next_r is not None:
        hi = mk()
        ops.append(dist.P2POp(dist.isend, _wire(x[:, :, d - 1:]), next_r, group))
        ops.append(dist.P2POp(dist.irecv, hi, next_r, group))
    reqs = dist.batch_isend_irecv(ops) if ops else []
    return _HaloRequest(reqs, lo, hi)


def halo_exchange(x: torch.Tensor, halo: int = 1, group=None) -> torch.Tensor:
    """x (N, C, D, H, W) padded along D with one plane from each D-neighbour
    (zeros at the volume ends). Kept for callers that want the padded slab;
    the depth-sharded conv itself never builds it."""
    if halo != 1:
        raise ValueError("the halo is one plane (k=3 convs)")
    lo, hi = start_halo_exchange(x, group).wait()
    z = torch.zeros_like(_plane(x, 0))
    return torch.cat([z if lo is None else lo, x, z if hi is None else hi], dim=2)


def halo_reduce(gx_padded: torch.Tensor, halo: int = 1, group=None) -> torch.Tensor:
    """Adjoint of halo_exchange: send the halo planes of a padded gradient back
    to the neighbours that own them and add what comes back into the slab."""
    if halo != 1:
        raise ValueError("the halo is one plane (k=3 convs)")
    prev_r, next_r = _neighbours(group)
    n, c, dp, h, w = gx_padded.shape
    d = dp - 2
    core = gx_padded[:, :, 1:1 + d].contiguous(memory_format=torch.channels_last_3d)
    ops = []
    from_prev = torch.empty((n, c, 1, h, w), dtype=core.dtype, device=core.device) if prev_r is not None else None
    from_next = torch.empty((n, c, 1, h, w), dtype=core.dtype, device=core.device) if next_r is not None else None
    if prev_r is not None:
        ops.append(dist.P2POp(dist.isend, gx_padded[:, :, :1].contiguous(), prev_r, group))
        ops.append(dist.P2POp(dist.irecv, from_prev, prev_r, group))
    if next_r is not None:
        ops.append(dist.P2POp(dist.isend, gx_padded[:, :, 1 + d:].contiguous(), next_r, group))
        ops.append(dist.P2POp(dist.irecv, from_next, next_r, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    if from_prev is not None:
        core[:, :, :1] += from_prev
    if from_next is not None:
        core[:, :, d - 1:] += from_next
    return core


class _ConvOps:
    """The three conv legs with per-axis padding: the B200 kernels for CUDA
    tensors, stock PyTorch (any dtype, fp64 included) otherwise."""

    def __init__(self, t: torch.Tensor):
        self.native = t.is_cuda and _cw()._wmma_hw()

    def fwd(self, x, w, b, pads, out=None):
        if self.native:
            return _cw()._launch_fwd(x, w, b, pads, out=out)
        y = torch.nn.functional.conv3d(x, w.to(x.dtype), None if b is None else b.to(x.dtype), 1, pads)
        if out is not None:
            out.copy_(y)
            return out
        return y

    def dgrad(self, go, w, x_shape, pads, out=None):
        if self.native:
            return _cw()._launch_dgrad(go, w, x_shape, pads, out=out)
        gx = torch.nn.grad.conv3d_input(tuple(x_shape), w.to(go.dtype), go.contiguous(), 1, pads)
        if out is not None:
            out.copy_(gx)
            return out
        return gx

    def wgrad(self, x, go, w_shape, pads, want_db):
        if self.native:
            return _cw()._launch_wgrad(x, go, w_shape, pads, want_db)
        acc = torch.promote_types(x.dtype, torch.float32)   # fp32 accumulation, fp64 kept
        dw = torch.nn.grad.conv3d_weight(x.to(acc), tuple(w_shape), go.to(acc).contiguous(), 1, pads)
        return dw, (go.to(acc).sum(dim=(0, 2, 3, 4)) if want_db else None)


def _write(dst: torch.Tensor, i: int, n: int):
    """Planes [i, i+n) of ``dst`` as an output buffer for a kernel: the view
    itself when it is dense NDHWC (batch 1), else None (compute, then copy)."""
    v = dst[:, :, i:i + n]
    return v if v.is_contiguous(memory_format=torch.channels_last_3d) else None


def _into(dst: torch.Tensor, i: int, n: int, fn):
    buf = _write(dst, i, n)
    r = fn(buf)
    if buf is None:
        dst[:, :, i:i + n] = r


class DepthShardedConv3dFn(torch.autograd.Function):
    """k3 pad-1 Conv3d of a D-sharded volume, interior first.

    Forward: the edge planes go to the D-neighbours (NCCL P2P) while the
    interior output planes 1..d-2 are computed from the local slab alone
    (D padding 0, written straight into the output); when the halo planes
    have arrived, output planes 0 and d-1 are computed from the three-plane
    stacks [lo, x0, x1] and [x_{d-2}, x_{d-1}, hi]. No padded copy of the
    slab is made. Backward does the same with dY's edge planes for dX (the
    interior planes come from dY alone, forward padding (2, 1, 1) on d-2
    planes), and dW = dW(x, dY, pad 1) plus the two halo-plane terms it
    misses, all-reduced (sum) over the group with db.
    """

    @staticmethod
    def forward(ctx, x, weight, bias, group):
        ops = _ConvOps(x)
        n, c, d, h, w = x.shape
        if d < 2:
            raise ValueError("each rank needs at least two planes of the depth-sharded volume")
        if ops.native:
            x = _cw()._as_ndhwc(x)
        req = start_halo_exchange(x, group)
        cout = int(weight.shape[0])
        y = torch.empty((n, cout, d, h, w), dtype=x.dtype, device=x.device, memory_format=torch.channels_last_3d)
        if d > 2:
            _into(y, 1, d - 2, lambda buf: ops.fwd(x, weight, bias, (0, 1, 1), buf))
        lo, hi = req.wait()
        z = torch.zeros_like(_plane(x, 0))
        lo3 = torch.cat([z if lo is None else lo, _plane(x, 0, 2)], dim=2)
        hi3 = torch.cat([_plane(x, d - 2, 2), z if hi is None else hi], dim=2)
        _into(y, 0, 1, lambda buf: ops.fwd(lo3, weight, bias, (0, 1, 1), buf))
        _into(y, d - 1, 1, lambda buf: ops.fwd(hi3, weight, bias, (0, 1, 1), buf))
        ctx.save_for_backward(x, weight, *(t for t in (lo, hi) if t is not None))
        ctx.has = (lo is not None, hi is not None)
        ctx.has_bias = bias is not None
        ctx.group = group
        return y

    @staticmethod
    def backward(ctx, go):
        saved = list(ctx.saved_tensors)
        x, weight = saved[0], saved[1]
        rest = saved[2:]
        lo = rest.pop(0) if ctx.has[0] else None
        hi = rest.pop(0) if ctx.has[1] else None
        group = ctx.group
        ops = _ConvOps(x)
        go = go.to(x.dtype)
        if ops.native:
            go = _cw()._as_ndhwc(go)
        n, c, d, h, w = x.shape
        req = start_halo_exchange(go, group)
        # dW over the slab with the volume's own padding, then the two terms
        # that pair a halo plane with an edge plane of dY (kd = 0 / kd = 2)
        dw, db = ops.wgrad(x, go, weight.shape, (1, 1, 1), ctx.has_bias)
        if lo is not None:
            dlo, _ = ops.wgrad(torch.cat([lo, _plane(x, 0, 2)], dim=2), _plane(go, 0), weight.shape, (0, 1, 1), False)
            dw[:, :, 0] += dlo[:, :, 0]
        if hi is not None:
            dhi, _ = ops.wgrad(torch.cat([_plane(x, d - 2, 2), hi], dim=2), _plane(go, d - 1), weight.shape,
                               (0, 1, 1), False)
            dw[:, :, 2] += dhi[:, :, 2]
        pending = GradAllReducer(group, average=False).reduce_async([dw, db])
        gx = torch.empty(x.shape, dtype=x.dtype, device=x.device, memory_format=torch.channels_last_3d)
        if d > 2:
            _into(gx, 1, d - 2, lambda buf: ops.dgrad(go, weight, (n, c, d - 2, h, w), (2, 1, 1), buf))
        glo, ghi = req.wait()
        z = torch.zeros_like(_plane(go, 0))
        g_lo3 = torch.cat([z if glo is None else glo, _plane(go, 0, 2)], dim=2)
        g_hi3 = torch.cat([_plane(go, d - 2, 2), z if ghi is None else ghi], dim=2)
        _into(gx, 0, 1, lambda buf: ops.dgrad(g_lo3, weight, (n, c, 1, h, w), (2, 1, 1), buf))
        _into(gx, d - 1, 1, lambda buf: ops.dgrad(g_hi3, weight, (n, c, 1, h, w), (2, 1, 1), buf))
        if pending is not None:
            pending.wait()
        return gx, dw.to(weight.dtype), (None if db is None else db.to(weight.dtype)), None


def depth_sharded_conv3d(x, weight, bias=None, group=None):
    """k=3, pad=1 Conv3d of a D-sharded activation (each rank: its D slab).
    Under autocast the activation is cast to the autocast dtype here (the
    weight is packed from its own dtype), as ``conv3d_wmma`` does."""
    if tuple(weight.shape[2:]) != (3, 3, 3):
        raise ValueError("depth sharding is implemented for k=3, pad=1 convs")
    x, weight, bias = _cw()._autocast_args(x, weight, bias)
    return DepthShardedConv3dFn.apply(x, weight, bias, group)


# ---------------------------------------------------------------------------
# Modules for a depth-sharded model
# ---------------------------------------------------------------------------
class _SyncBNFn(torch.autograd.Function):
    """Batch norm whose statistics span every rank of ``group`` (fp32, or fp64 for fp64 inputs)."""

    @staticmethod
    def forward(ctx, x, weight, bias, running_mean, running_var, momentum, eps, group, training):
        dims = (0, 2, 3, 4)
        acc = torch.promote_types(x.dtype, torch.float32)    # fp32 statistics (fp64 kept)
        xf = x.to(acc)
        c = x.shape[1]
        if training:
            cnt = torch.tensor([xf.numel() // c], dtype=acc, device=x.device)
            s = torch.cat([xf.sum(dims), cnt])
            dist.all_reduce(s, group=group)
            total = s[-1]
            mean = s[:c] / total
            sq = ((xf - mean.view(1, c, 1, 1, 1)) ** 2).sum(dims)
            dist.all_reduce(sq, group=group)
            var = sq / total
            if running_mean is not None:
                with torch.no_grad():
                    running_mean.mul_(1 - momentum).add_(mean.to(running_mean.dtype), alpha=momentum)
                    unbiased = var * total / torch.clamp(total - 1, min=1)
                    running_var.mul_(1 - momentum).add_(unbiased.to(running_var.dtype), alpha=momentum)
        else:
            mean, var, total = running_mean.to(acc).clone(), running_var.to(acc).clone(), None
        invstd = torch.rsqrt(var + eps)
        shape = (1, c, 1, 1, 1)
        xhat = (xf - mean.view(shape)) * invstd.view(shape)
        wf = weight.to(acc) if weight is not None else torch.ones(c, dtype=acc, device=x.device)
        bf = bias.to(acc) if bias is not None else torch.zeros(c, dtype=acc, device=x.device)
        y = (xhat * wf.view(shape) + bf.view(shape)).to(x.dtype)
        ctx.save_for_backward(x, mean, invstd, wf)
        ctx.total = total
        ctx.group = group
        ctx.has_affine = (weight is not None, bias is not None)
        ctx.wdtype = None if weight is None else weight.dtype
        ctx.bdtype = None if bias is None else bias.dtype
        return y

    @staticmethod
    def backward(ctx, gy):
        x, mean, invstd, wf = ctx.saved_tensors
        c = x.shape[1]
        shape = (1, c, 1, 1, 1)
        dims = (0, 2, 3, 4)
        gf = gy.to(mean.dtype)
        xhat = (x.to(mean.dtype) - mean.view(shape)) * invstd.view(shape)
        # whole-volume sums: they give dgamma / dbeta and, in training, the
        # terms of dX that come from the shared statistics
        s = torch.cat([gf.sum(dims), (gf * xhat).sum(dims)])
        dist.all_reduce(s, group=ctx.group)
        sum_g, sum_gx = s[:c], s[c:]
        scale = (wf * invstd).view(shape)
        if ctx.total is not None:
            total = ctx.total
            gx = scale * (gf - (sum_g / total).view(shape) - xhat * (sum_gx / total).view(shape))
        else:
            gx = gf * scale
        gw = sum_gx.to(ctx.wdtype) if ctx.has_affine[0] else None
        gb = sum_g.to(ctx.bdtype) if ctx.has_affine[1] else None
        return gx.to(gy.dtype), gw, gb, None, None, None, None, None, None


class DepthShardedBatchNorm3d(torch.nn.BatchNorm3d):
    """BatchNorm3d whose batch statistics (and their gradient sums) are
    all-reduced over ``group``: every rank holds one D slab of the same
    volume, so the statistics must be the whole volume's. Weight and bias
    gradients come out as whole-volume sums (no further reduction)."""

    def __init__(self, *args, group=None, **kw):
        super().__init__(*args, **kw)
        self.group = group

    def forward(self, x):
        if not (dist.is_available() and dist.is_initialized()):
            return super().forward(x)
        training = self.training or not self.track_running_stats
        if self.training and self.num_batches_tracked is not None:
            self.num_batches_tracked.add_(1)
        mom = 0.1 if self.momentum is None else self.momentum
        return _SyncBNFn.apply(x, self.weight, self.bias, self.running_mean if self.track_running_stats else None,
                               self.running_var if self.track_running_stats else None, mom, self.eps, self.group,
                               training)


class DepthShardedBatchNormReLU3d(BatchNormReLU3d):
    """BatchNormReLU3d (fused kernels) over a D-sharded volume: the
    per-channel sums are all-reduced over ``group`` between the statistics
    pass and the finalize (and between the backward sums and the dX pass),
    with the running mean as the pivot every rank shares (the running
    statistics are updated identically on every rank). dgamma / dbeta come
    out as whole-volume sums."""

    def __init__(self, *args, group=None, **kw):
        super().__init__(*args, **kw)
        self.group = group
        # whole-volume voxel count per local count: the finalize kernels take
        # the count from the host, and reading an all-reduced count back each
        # call would stall the host once per layer and step
        self._totals = {}

    def _sums_hook(self):
        if not (dist.is_available() and dist.is_initialized()):
            return None
        group, C, totals = self.group, self.num_features, self._totals

        def hook(sums, count):
            dist.all_reduce(sums[:2 * C], group=group)
            if count is None:
                return None
            # Every rank calls this in the same order with its own slab, so
            # all ranks meet a new slab shape (and run this collective) at the
            # same call; later calls with the same shapes reuse the total.
            if count not in totals:
                t = torch.tensor([count], dtype=torch.float64, device=sums.device)
                dist.all_reduce(t, group=group)
                totals[count] = float(t.item())
            return totals[count]
        return hook

    def _pivot(self):
        if self.running_mean is None or not (dist.is_available() and dist.is_initialized()):
            return None
        return self.running_mean.detach().float().contiguous()


class DepthShardedConv3d(torch.nn.Conv3d):
    """Conv3d (k=3, pad=1) over a D-sharded volume; other geometries run
    locally (k=1 convs need no halo)."""

    def __init__(self, *args, group=None, **kw):
        super().__init__(*args, **kw)
        self.group = group

    def forward(self, x):
        if self.kernel_size == (3, 3, 3) and self.padding == (1, 1, 1) and self.stride == (1, 1, 1) \
                and self.dilation == (1, 1, 1) and self.groups == 1 and dist.is_initialized():
            return depth_sharded_conv3d(x, self.weight, self.bias, self.group)
        from .conv3d_wmma import conv3d_wmma
        if x.is_cuda:
            return conv3d_wmma(x, self.weight, self.bias, self.stride, self.padding, self.dilation, self.groups)
        return super().forward(x)


def depth_shard_model(model: torch.nn.Module, group=None) -> List[torch.nn.Parameter]:
    """Convert a model in place for depth sharding over ``group``: every k3
    pad-1 Conv3d becomes a DepthShardedConv3d (halo exchange), every
    BatchNorm3d a DepthShardedBatchNorm3d and every fused BatchNormReLU3d a
    DepthShardedBatchNormReLU3d (statistics over the whole volume).
    Pooling, k2s2 transpose convs, concatenation and k1 convs need no
    exchange. Returns the parameters whose gradients are still per-slab
    partial sums (the transpose convs and k1 convs): reduce them with
    ``GradSync(params, average=False)``."""
    partial: List[torch.nn.Parameter] = []

    def convert(mod):
        for name, child in list(mod.named_children()):
            if isinstance(child, torch.nn.Conv3d) and not isinstance(child, DepthShardedConv3d) \
                    and child.kernel_size == (3, 3, 3) and child.padding == (1, 1, 1):
                new = DepthShardedConv3d(child.in_channels, child.out_channels, 3, padding=1,
                                         bias=child.bias is not None, group=group,
                                         device=child.weight.device, dtype=child.weight.dtype)
                with torch.no_grad():
                    new.weight.copy_(child.weight)
                    if child.bias is not None:
                        new.bias.copy_(child.bias)
                setattr(mod, name, new)
            elif isinstance(child, BatchNormReLU3d) and not isinstance(child, DepthShardedBatchNormReLU3d):
                ref = child.weight if child.affine else child.running_mean
                new = DepthShardedBatchNormReLU3d(child.num_features, child.eps, child.momentum, child.affine,
                                                  child.track_running_stats, relu=child.relu, group=group,
                                                  device=None if ref is None else ref.device,
                                                  dtype=None if ref is None else ref.dtype)
                new.load_state_dict(child.state_dict())
                setattr(mod, name, new)
            elif isinstance(child, torch.nn.BatchNorm3d) and not isinstance(child, DepthShardedBatchNorm3d) \
                    and not isinstance(child, BatchNormReLU3d):
                ref = child.weight if child.affine else child.running_mean
                new = DepthShardedBatchNorm3d(child.num_features, child.eps, child.momentum, child.affine,
                                              child.track_running_stats, group=group,
                                              device=None if ref is None else ref.device,
                                              dtype=None if ref is None else ref.dtype)
                new.load_state_dict(child.state_dict())
                setattr(mod, name, new)
            elif isinstance(child, (torch.nn.Conv3d, torch.nn.ConvTranspose3d)) \
                    and not isinstance(child, DepthShardedConv3d):
                partial.extend(p for p in child.parameters(recurse=False) if p.requires_grad)
            else:
                convert(child)

    convert(model)
    return partial
