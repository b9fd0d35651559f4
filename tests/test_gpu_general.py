"""Conv3d of any geometry (r4c_convex_* entry points) on a B200.

Strided, dilated, grouped and non-cubic convs — the geometries the
reference sends to the vendor library (conv3d_wmma.py:1241-1242 of the
reference) — against the reference's CPU path (stock PyTorch fp32 conv) on
the same rounded inputs. The k=2 stride-2 conv runs on the tcgen05
transpose-conv kernels (roles swapped), the rest on SIMT kernels.
Tolerances as for the in-scope legs: forward / dX max-rel 2e-2, dW / db
norm-rel 3e-2 (fp32 inputs: 1e-4).
"""
import pytest
import torch
import torch.nn.functional as F

import oracle as O

pytestmark = pytest.mark.gpu

# x shape, w shape, stride, padding, dilation, groups
CASES = [
    ((2, 16, 8, 12, 16), (32, 16, 2, 2, 2), 2, 0, 1, 1),        # k2s2 downsample: tcgen05 transpose-conv kernels
    ((4, 24, 64, 128, 128), (48, 24, 2, 2, 2), 2, 0, 1, 1),     # k2s2 at the UNet's first level
    ((1, 48, 16, 32, 32), (96, 48, 2, 2, 2), 2, 0, 1, 1),
    ((2, 8, 9, 10, 11), (16, 8, 3, 3, 3), 2, 1, 1, 1),          # k3 stride 2 pad 1
    ((1, 6, 7, 8, 9), (5, 6, 3, 3, 3), (1, 2, 3), (1, 0, 2), 1, 1),
    ((1, 4, 9, 9, 9), (6, 4, 5, 5, 5), 1, 2, 1, 1),             # k5
    ((1, 8, 10, 11, 12), (8, 8, 3, 3, 3), 1, 2, 2, 1),          # dilation 2
    ((1, 8, 8, 8, 8), (16, 4, 3, 3, 3), 1, 1, 1, 2),            # groups 2
    ((2, 12, 6, 7, 8), (12, 1, 3, 3, 3), 1, 1, 1, 12),          # depthwise
    ((1, 8, 6, 9, 10), (8, 8, (3, 1, 1)), 1, (1, 0, 0), 1, 1),  # non-cubic kernel
    ((1, 5, 7, 7, 7), (3, 5, 2, 2, 2), 2, 0, 1, 1),             # k2s2 with odd channels / extents: SIMT
    ((0, 8, 4, 4, 4), (8, 8, 3, 3, 3), 2, 1, 1, 1),             # empty batch
]


def _wshape(ws):
    if len(ws) == 3:
        return (ws[0], ws[1]) + tuple(ws[2])
    return ws


def _ids():
    return [f"x{'x'.join(map(str, c[0]))}_w{'x'.join(map(str, _wshape(c[1])))}_s{c[2]}_p{c[3]}_d{c[4]}_g{c[5]}"
            for c in CASES]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=["bf16", "fp16", "fp32"])
@pytest.mark.parametrize("case", CASES, ids=_ids())
def test_general_conv_legs(cuda_ready, case, dtype):
    from rdna4_conv3d import _native
    from rdna4_conv3d.conv3d_wmma import conv3d_general
    xs, ws, stride, pad, dil, groups = case
    ws = _wshape(ws)
    if dtype == torch.float32 and xs[0] * xs[2] * xs[3] * xs[4] > 1_000_000:
        pytest.skip("fp32 SIMT path covered on the smaller shapes")
    g = torch.Generator().manual_seed(sum(xs) + sum(ws))
    x = torch.randn(*xs, generator=g).to(dtype)
    w = (torch.randn(*ws, generator=g) / (ws[1] * ws[2] * ws[3] * ws[4]) ** 0.5).to(dtype)
    b = torch.randn(ws[0], generator=g).to(dtype)
    yref = F.conv3d(x.float(), w.float(), b.float(), stride, pad, dil, groups)
    go = torch.randn(yref.shape, generator=g).to(dtype)
    xg = x.cuda().contiguous(memory_format=torch.channels_last_3d).requires_grad_(True)
    wg = w.cuda().requires_grad_(True)
    bg = b.cuda().requires_grad_(True)
    n0 = _native.launch_count()
    y = conv3d_general(xg, wg, bg, stride, pad, dil, groups)
    y.backward(go.cuda())
    torch.cuda.synchronize()
    assert y.shape == yref.shape and y.dtype == dtype
    if xs[0] == 0:
        return
    assert _native.launch_count() > n0
    xr = x.float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    br = b.float().requires_grad_(True)
    F.conv3d(xr, wr, br, stride, pad, dil, groups).backward(go.float())
    tol_w = 1e-4 if dtype == torch.float32 else 3e-2
    assert O.max_rel(y.float().cpu(), yref) <= (1e-4 if dtype == torch.float32 else 2e-2)
    assert O.max_rel(xg.grad.float().cpu(), xr.grad) <= (1e-4 if dtype == torch.float32 else 2e-2)
    assert O.norm_rel(wg.grad.float().cpu(), wr.grad) <= tol_w
    assert O.norm_rel(bg.grad.float().cpu(), br.grad) <= tol_w


def test_k2s2_routes_to_tensor_cores(cuda_ready):
    """Conv3dWmma with k=2 stride 2 (bf16 / autocast) runs the tcgen05 path;
    fp32 without autocast stays with the vendor library."""
    from rdna4_conv3d import Conv3dWmma, _native
    m = Conv3dWmma(24, 48, 2, stride=2).cuda()
    x = torch.randn(2, 24, 8, 16, 16, device="cuda").contiguous(memory_format=torch.channels_last_3d)
    d = _native.make_convex_desc(x.shape, m.weight.shape, (2, 2, 2), (0, 0, 0), (1, 1, 1), 1, torch.bfloat16)
    assert _native.convex_plan(d) == _native.KERNEL_TC
    n0 = _native.launch_count()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
    assert _native.launch_count() > n0 and y.dtype == torch.bfloat16
    torch.testing.assert_close(y.float(), F.conv3d(x, m.weight, m.bias, 2).float(), atol=3e-2, rtol=3e-2)
    n1 = _native.launch_count()
    m(x)                       # fp32, no autocast: stock conv
    assert _native.launch_count() == n1
