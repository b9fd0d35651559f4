"""Parity at the sizes the benchmark times.

Every layer that bench.py times is run here at its full batch-4 size through
the same launch path (default planner, first-call plan tuner on, the split
counts and multi-wave persistent schedules that size selects), and compared
with the reference's CPU path (stock PyTorch fp32 conv on the host, see
oracle/oracle.py) fed the same bf16-rounded inputs. North-star tolerances,
written here:
  forward and dX : max|out - ref| / max|ref| <= 2e-2
  dW, db         : ||out - ref|| / ||ref||   <= 3e-2
dW and db are fp32 accumulations of identical inputs, so they also meet a
much tighter 1e-3 bound; it is asserted as well.

Also here: the isolated public API (wmma_fwd / wmma_dw / wmma_dx, the path
bench.py's e2e number goes through) with its layout and dtype contract, and
per-axis padding (0, 1, 1), the form the depth-sharded conv uses.
Reference test being extended: tests/test_conv3d.py:47-75.
"""
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

FWD_TOL = 2e-2
DW_TOL = 3e-2
DW_TIGHT = 1e-3
BATCH = 4

# (cin, cout, (D, H, W), k) — identical to bench.py's TRUNK
TRUNK = [
    (1, 24, (64, 128, 128), 3),
    (24, 24, (64, 128, 128), 3),
    (48, 48, (32, 64, 64), 3),
    (96, 96, (16, 32, 32), 3),
    (192, 192, (8, 16, 16), 3),
    (48, 24, (64, 128, 128), 1),
    (96, 48, (32, 64, 64), 1),
    (192, 96, (16, 32, 32), 1),
]
# ConvTranspose3d k2 s2 from these inputs
TCONV = [
    (192, 96, (8, 16, 16)),
    (96, 48, (16, 32, 32)),
    (48, 24, (32, 64, 64)),
]


def _cw():
    import sys
    return sys.modules["rdna4_conv3d.conv3d_wmma"]


def _cl(t):
    return t.contiguous(memory_format=torch.channels_last_3d)


def _trunk_inputs(cin, cout, spatial, k, seed):
    """Seeded N(0,1) activations / grad_out and default nn.Conv3d init, rounded to bf16."""
    g = torch.Generator().manual_seed(seed)
    d, h, w = spatial
    x = torch.randn(BATCH, cin, d, h, w, generator=g).to(torch.bfloat16)
    go = torch.randn(BATCH, cout, d, h, w, generator=g).to(torch.bfloat16)
    torch.manual_seed(seed)
    conv = torch.nn.Conv3d(cin, cout, k, padding=(k - 1) // 2)
    return x, go, conv.weight.detach().to(torch.bfloat16), conv.bias.detach().to(torch.bfloat16)


@pytest.mark.parametrize("layer", TRUNK, ids=[f"k{k} {a}->{b}" for a, b, _, k in TRUNK])
def test_trunk_layer_full_size(cuda_ready, layer):
    cin, cout, spatial, k = layer
    pad = (k - 1) // 2
    cw = _cw()
    x, go, wt, b = _trunk_inputs(cin, cout, spatial, k, seed=cin * 1000 + cout)
    xg, gg = _cl(x.cuda()), _cl(go.cuda())
    wg, bg = wt.cuda(), b.cuda()
    p3 = (pad,) * 3
    y = cw._launch_fwd(xg, wg, bg, p3).cpu()
    dw, db = cw._launch_wgrad(xg, gg, wg.shape, p3, True)
    dx = cw._launch_dgrad(gg, wg, xg.shape, p3).cpu()
    dw, db = dw.cpu(), db.cpu()
    del xg, gg
    from rdna4_conv3d import _native
    assert _native.device_error() == 0

    e_y = O.max_rel(y, O.torch_conv_fwd(x, wt, b, pad))
    e_dx = O.max_rel(dx, O.torch_conv_dx(x.shape, wt, go, pad))
    e_dw = O.norm_rel(dw, O.torch_conv_dw(x, go, wt.shape, pad))
    e_db = O.norm_rel(db, go.float().sum(dim=(0, 2, 3, 4)))
    assert e_y <= FWD_TOL, e_y
    assert e_dx <= FWD_TOL, e_dx
    assert e_dw <= DW_TOL and e_db <= DW_TOL, (e_dw, e_db)
    assert e_dw <= DW_TIGHT and e_db <= DW_TIGHT, (e_dw, e_db)


@pytest.mark.parametrize("layer", TCONV, ids=[f"T {a}->{b}" for a, b, _ in TCONV])
def test_tconv_layer_full_size(cuda_ready, layer):
    cin, cout, (d, h, w) = layer
    cw = _cw()
    g = torch.Generator().manual_seed(cin)
    x = torch.randn(BATCH, cin, d, h, w, generator=g).to(torch.bfloat16)
    go = torch.randn(BATCH, cout, 2 * d, 2 * h, 2 * w, generator=g).to(torch.bfloat16)
    torch.manual_seed(cin)
    m = torch.nn.ConvTranspose3d(cin, cout, 2, stride=2)
    wt, b = m.weight.detach().to(torch.bfloat16), m.bias.detach().to(torch.bfloat16)
    xg, gg, wg, bg = _cl(x.cuda()), _cl(go.cuda()), wt.cuda(), b.cuda()
    y = cw.transpose_k2s2_fwd(xg, wg, bg).cpu()
    dx = cw.transpose_k2s2_dx(xg.shape, wg, gg).cpu()
    dw, db = cw.transpose_k2s2_dw(xg, wg.shape, gg, True)
    dw, db = dw.cpu(), db.cpu()
    dxr, dwr = O.torch_tconv_grads(x, wt, go)
    assert O.max_rel(y, O.torch_tconv_fwd(x, wt, b)) <= FWD_TOL
    assert O.max_rel(dx, dxr) <= FWD_TOL
    assert O.norm_rel(dw, dwr) <= DW_TIGHT
    assert O.norm_rel(db, go.float().sum(dim=(0, 2, 3, 4))) <= DW_TIGHT


# ---------------------------------------------------------------------------
# The isolated API (reference conv3d_wmma.py:1368-1409)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("layout", ["ncdhw", "ndhwc"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("case", [(2, 24, 24, 16, 32, 32, 3, 1), (1, 48, 24, 8, 16, 16, 1, 0),
                                  (1, 1, 24, 8, 16, 16, 3, 1), (1, 16, 8, 5, 6, 7, 3, 2)],
                         ids=["cfg1", "k1", "stem", "pad2"])
def test_isolated_api(cuda_ready, case, dtype, layout):
    from rdna4_conv3d import wmma_dw, wmma_dx, wmma_fwd
    n, cin, cout, d, h, w, k, pad = case
    g = torch.Generator().manual_seed(11)
    x = torch.randn(n, cin, d, h, w, generator=g).to(dtype)
    wt = (torch.randn(cout, cin, k, k, k, generator=g) / (cin * k ** 3) ** 0.5).to(dtype)
    b = torch.randn(cout, generator=g).to(dtype)
    o = tuple(s + 2 * pad - (k - 1) for s in (d, h, w))
    go = torch.randn(n, cout, *o, generator=g).to(dtype)
    xg, gg = x.cuda(), go.cuda()
    if layout == "ndhwc":
        xg, gg = _cl(xg), _cl(gg)
    # the reference's rule (conv3d_wmma.py:1379-1381): NDHWC out when x is
    # channels_last_3d-contiguous, which a one-channel NCDHW tensor also is
    cl_in = xg.is_contiguous(memory_format=torch.channels_last_3d)
    fmt = torch.channels_last_3d if cl_in else torch.contiguous_format
    y = wmma_fwd(xg, wt.cuda(), b.cuda(), 1, pad)
    dw = wmma_dw(xg, wt.cuda(), gg, 1, pad)
    dx = wmma_dx(xg, wt.cuda(), gg, 1, pad)
    torch.cuda.synchronize()
    assert y.shape == (n, cout) + o and y.dtype == dtype and y.is_contiguous(memory_format=fmt)
    assert dx.shape == x.shape and dx.dtype == dtype and dx.is_contiguous(memory_format=fmt)
    assert dw.shape == wt.shape and dw.dtype == go.dtype and dw.is_contiguous()
    assert O.max_rel(y.cpu(), O.torch_conv_fwd(x, wt, b, pad)) <= FWD_TOL
    assert O.max_rel(dx.cpu(), O.torch_conv_dx(x.shape, wt, go, pad)) <= FWD_TOL
    # dW comes back rounded to go's dtype (the reference's wmma_dw contract)
    assert O.norm_rel(dw.cpu(), O.torch_conv_dw(x, go, wt.shape, pad)) <= DW_TOL


def test_isolated_api_rejects_out_of_scope(cuda_ready):
    from rdna4_conv3d import wmma_dw, wmma_fwd
    x = torch.randn(1, 8, 4, 4, 4, device="cuda", dtype=torch.bfloat16)
    w5 = torch.randn(8, 8, 5, 5, 5, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        wmma_fwd(x, w5, None, 1, 2)
    w3 = torch.randn(8, 8, 3, 3, 3, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        wmma_dw(x, w3, x, 2, 1)


# ---------------------------------------------------------------------------
# Per-axis padding: the depth-sharded conv runs the local slab with D pad 0
# (the halo planes stand in for the neighbours), so fwd/dW see (0, 1, 1) and
# dX sees (2, 1, 1) after the k-1-p flip.
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("pads", [(0, 1, 1), (1, 0, 1), (2, 1, 0), (0, 2, 1)], ids=str)
@pytest.mark.parametrize("case", [(1, 24, 24, 6, 16, 16), (2, 48, 48, 5, 8, 12), (1, 1, 24, 6, 8, 16),
                                  (1, 96, 96, 4, 8, 8)], ids=["24", "48", "stem", "96"])
def test_per_axis_padding(cuda_ready, case, pads):
    n, cin, cout, d, h, w = case
    cw = _cw()
    g = torch.Generator().manual_seed(5)
    x = torch.randn(n, cin, d, h, w, generator=g).to(torch.bfloat16)
    wt = (torch.randn(cout, cin, 3, 3, 3, generator=g) / (cin * 27) ** 0.5).to(torch.bfloat16)
    b = torch.randn(cout, generator=g).to(torch.bfloat16)
    o = tuple(s + 2 * p - 2 for s, p in zip((d, h, w), pads))
    go = torch.randn(n, cout, *o, generator=g).to(torch.bfloat16)
    xg, gg = _cl(x.cuda()), _cl(go.cuda())
    y = cw._launch_fwd(xg, wt.cuda(), b.cuda(), pads).cpu()
    dx = cw._launch_dgrad(gg, wt.cuda(), xg.shape, pads).cpu()
    dw, db = cw._launch_wgrad(xg, gg, wt.shape, pads, True)
    assert y.shape == (n, cout) + o
    assert O.max_rel(y, O.torch_conv_fwd(x, wt, b, pads)) <= FWD_TOL
    assert O.max_rel(dx, O.torch_conv_dx(x.shape, wt, go, pads)) <= FWD_TOL
    assert O.norm_rel(dw.cpu(), O.torch_conv_dw(x, go, wt.shape, pads)) <= DW_TIGHT
    assert O.norm_rel(db.cpu(), go.float().sum(dim=(0, 2, 3, 4))) <= DW_TIGHT
