"""``torch.ops.r4c.*``: the C-ABI legs as registered PyTorch operators.

Each op calls the same library entry point as the autograd Functions in
conv3d_wmma.py (through _native), and has a fake (meta) implementation that
gives shapes, dtypes and the NDHWC layout without running anything, so the
ops can be traced (FakeTensor, torch.compile, torch.export) and their shapes
checked on a machine without a GPU. Reference counterpart: the pybind
``fwd_k3`` op of the HIP extension (conv3d_wmma_hip.hip:148-195) and the
Triton launchers it sat beside; the reference registers no torch op.

    r4c::conv3d_fwd(x, weight, bias?, padding[3]) -> y
    r4c::conv3d_dx(go, weight, x_shape[5], padding[3]) -> dx
    r4c::conv3d_dw(x, go, weight_shape[5], padding[3], want_db) -> (dw fp32, db fp32; empty when not wanted)
    r4c::tconv_fwd(x, weight, bias?) -> y                        (k=2 s=2 p=0)
    r4c::tconv_dx(go, weight, x_shape[5]) -> dx
    r4c::tconv_dw(x, go, weight_shape[5], want_db) -> (dw fp32, db fp32)

Activations are NDHWC (channels_last_3d) bf16 / fp16; weights in PyTorch's
layout, any float dtype (packed by the library). Outputs are channels_last_3d.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

_CL = torch.channels_last_3d


def _osz(i: int, k: int, p: int) -> int:
    return i + 2 * p - (k - 1)


def _cw():
    import sys
    return sys.modules["rdna4_conv3d.conv3d_wmma"]


@torch.library.custom_op("r4c::conv3d_fwd", mutates_args=())
def conv3d_fwd(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], padding: List[int]) -> torch.Tensor:
    return _cw()._launch_fwd(x, weight, bias, tuple(padding))


@conv3d_fwd.register_fake
def _(x, weight, bias, padding):
    k = weight.shape[2]
    n, _, d, h, w = x.shape
    shape = (n, weight.shape[0], _osz(d, k, padding[0]), _osz(h, k, padding[1]), _osz(w, k, padding[2]))
    return torch.empty(shape, dtype=x.dtype, device=x.device, memory_format=_CL)


@torch.library.custom_op("r4c::conv3d_dx", mutates_args=())
def conv3d_dx(go: torch.Tensor, weight: torch.Tensor, x_shape: List[int], padding: List[int]) -> torch.Tensor:
    return _cw()._launch_dgrad(go, weight, tuple(x_shape), tuple(padding))


@conv3d_dx.register_fake
def _(go, weight, x_shape, padding):
    return torch.empty(tuple(x_shape), dtype=go.dtype, device=go.device, memory_format=_CL)


@torch.library.custom_op("r4c::conv3d_dw", mutates_args=())
def conv3d_dw(x: torch.Tensor, go: torch.Tensor, weight_shape: List[int], padding: List[int],
              want_db: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    dw, db = _cw()._launch_wgrad(x, go, tuple(weight_shape), tuple(padding), want_db)
    if db is None:
        db = torch.empty(0, dtype=torch.float32, device=x.device)
    return dw, db


@conv3d_dw.register_fake
def _(x, go, weight_shape, padding, want_db):
    dw = x.new_empty(tuple(weight_shape), dtype=torch.float32)
    db = x.new_empty((weight_shape[0] if want_db else 0,), dtype=torch.float32)
    return dw, db


@torch.library.custom_op("r4c::tconv_fwd", mutates_args=())
def tconv_fwd(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
    return _cw().transpose_k2s2_fwd(x, weight, bias)


@tconv_fwd.register_fake
def _(x, weight, bias):
    n, _, d, h, w = x.shape
    return torch.empty((n, weight.shape[1], 2 * d, 2 * h, 2 * w), dtype=x.dtype, device=x.device, memory_format=_CL)


@torch.library.custom_op("r4c::tconv_dx", mutates_args=())
def tconv_dx(go: torch.Tensor, weight: torch.Tensor, x_shape: List[int]) -> torch.Tensor:
    return _cw().transpose_k2s2_dx(tuple(x_shape), weight, go)


@tconv_dx.register_fake
def _(go, weight, x_shape):
    return torch.empty(tuple(x_shape), dtype=go.dtype, device=go.device, memory_format=_CL)


@torch.library.custom_op("r4c::tconv_dw", mutates_args=())
def tconv_dw(x: torch.Tensor, go: torch.Tensor, weight_shape: List[int], want_db: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    dw, db = _cw().transpose_k2s2_dw(x, tuple(weight_shape), go, want_db)
    if db is None:
        db = torch.empty(0, dtype=torch.float32, device=x.device)
    return dw, db


@tconv_dw.register_fake
def _(x, go, weight_shape, want_db):
    dw = x.new_empty(tuple(weight_shape), dtype=torch.float32)
    db = x.new_empty((weight_shape[1] if want_db else 0,), dtype=torch.float32)
    return dw, db
