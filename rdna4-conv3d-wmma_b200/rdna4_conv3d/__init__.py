"""Drop-in 3D convolution on NVIDIA B200 (sm_100a) tensor cores.

Same public surface as the reference ``rdna4_conv3d`` package
(src/rdna4_conv3d/__init__.py:10-37): k=1 and k=3 stride-1 Conv3d and k=2 s=2
ConvTranspose3d run on hand-written tcgen05/TMA CUDA kernels through the C-ABI
library ``libr4c_conv3d.so``; unsupported geometries fall back to
``torch.nn.functional.conv3d``.

As in the reference, binding the function ``conv3d_wmma`` here shadows the
submodule attribute of the same name; reach the module via ``sys.modules``.
"""

from rdna4_conv3d.conv3d_wmma import (
    Conv3dWmma,
    ConvTranspose3dWmma,
    conv3d_plan,
    conv3d_wmma,
    swap_conv3d,
    wmma_dw,
    wmma_dx,
    wmma_fwd,
    wmma_ok_dw,
    wmma_ok_dx,
    wmma_ok_fwd,
)

from rdna4_conv3d import ops as _ops  # noqa: E402,F401  (registers torch.ops.r4c.*)

__version__ = "0.1.0"
__all__ = [
    "Conv3dWmma",
    "ConvTranspose3dWmma",
    "conv3d_plan",
    "conv3d_wmma",
    "swap_conv3d",
    "wmma_dw",
    "wmma_dx",
    "wmma_fwd",
    "wmma_ok_dw",
    "wmma_ok_dx",
    "wmma_ok_fwd",
]
