"""Cross-entropy over NDHWC logits on the native kernels (r4c_ce_*).

``cross_entropy(logits, target)`` is ``F.cross_entropy(logits, target)``
(reduction 'mean', no class weights, ``ignore_index``) for channels_last_3d
bf16/fp16 logits on a CUDA device: one kernel pass forward (per-voxel
log-sum-exp in fp32, deterministic mean) and one backward, with no fp32
copy of the logits and no layout change. Other inputs take F.cross_entropy.
No reference counterpart: the reference's training step computes its loss
with stock PyTorch (benches/unet_e2e.py:41-52).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _native


class CrossEntropyNDHWCFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, ignore_index):
        loss_count = _native.ce_forward(logits, target, ignore_index)
        ctx.save_for_backward(logits, target, loss_count)
        ctx.ignore_index = ignore_index
        return loss_count[0].clone()

    @staticmethod
    def backward(ctx, grad):
        logits, target, loss_count = ctx.saved_tensors
        dz = None
        if ctx.needs_input_grad[0]:
            dz = _native.ce_backward(logits, target, ctx.ignore_index, loss_count, grad)
        return dz, None, None


def _native_ok(logits: torch.Tensor, target: torch.Tensor) -> bool:
    return (logits.is_cuda and logits.dim() == 5 and logits.dtype in (torch.bfloat16, torch.float16)
            and logits.is_contiguous(memory_format=torch.channels_last_3d)
            and target.dtype == torch.int64 and target.is_contiguous() and target.device == logits.device
            and tuple(target.shape) == (logits.shape[0],) + tuple(logits.shape[2:]))


def cross_entropy(logits: torch.Tensor, target: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    """Mean cross-entropy of (N, C, D, H, W) logits against (N, D, H, W) labels."""
    if _native_ok(logits, target):
        return CrossEntropyNDHWCFn.apply(logits, target, int(ignore_index))
    return F.cross_entropy(logits, target, ignore_index=ignore_index)
