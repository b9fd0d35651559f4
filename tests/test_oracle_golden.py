"""Pin the C oracle against the reference's own outputs (CPU only).

The golden fixtures were produced by the reference's Triton kernels
(tests/golden/make_golden.py). They are fp16 outputs of fp32-accumulated
GEMMs, so the oracle (fp32) must agree to fp16 output rounding. The oracle is
also checked against the reference's CPU path (stock PyTorch fp32).
"""
import glob
import os

import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN_DIR

FILES = sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def _load(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


def test_fixtures_present():
    names = {os.path.basename(f) for f in FILES}
    assert "ref_k3_c24_c24.npz" in names and "tconv_c16_c8.npz" in names
    assert len(FILES) >= 9


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f)[:-4] for f in FILES])
def test_oracle_matches_reference_kernels(path):
    g = _load(path)
    n, cin, cout, d, h, w, k, pad = (int(v) for v in g["meta"])
    x = torch.from_numpy(g["x"]).float()
    wt = torch.from_numpy(g["w"]).float()
    b = torch.from_numpy(g["b"]).float()
    go = torch.from_numpy(g["go"]).float()
    if k == 2:
        y = O.c_tconv_fwd(x, wt, b)
        dx = O.c_tconv_dx(x.shape, wt, go)
        dw = O.c_tconv_dw(x, go, cout)
    else:
        y = O.c_conv_fwd(x, wt, b, pad)
        dx = O.c_conv_dx(x.shape, wt, go, pad)
        dw = O.c_conv_dw(x, go, wt.shape, pad)
    # fp16 output rounding of the reference: half an ulp of |y|max ~ 2.5e-4 rel.
    assert O.max_rel(y, torch.from_numpy(g["y"])) < 2e-3
    assert O.norm_rel(dw, torch.from_numpy(g["dw"])) < 2e-3
    if "dx" in g:
        assert O.max_rel(dx, torch.from_numpy(g["dx"])) < 2e-3


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f)[:-4] for f in FILES])
def test_oracle_matches_torch_cpu(path):
    g = _load(path)
    n, cin, cout, d, h, w, k, pad = (int(v) for v in g["meta"])
    x = torch.from_numpy(g["x"]).float()
    wt = torch.from_numpy(g["w"]).float()
    b = torch.from_numpy(g["b"]).float()
    go = torch.from_numpy(g["go"]).float()
    if k == 2:
        dxr, dwr = O.torch_tconv_grads(x, wt, go)
        assert O.max_rel(O.c_tconv_fwd(x, wt, b), O.torch_tconv_fwd(x, wt, b)) < 1e-5
        assert O.max_rel(O.c_tconv_dx(x.shape, wt, go), dxr) < 1e-5
        assert O.norm_rel(O.c_tconv_dw(x, go, cout), dwr) < 1e-5
    else:
        assert O.max_rel(O.c_conv_fwd(x, wt, b, pad), O.torch_conv_fwd(x, wt, b, pad)) < 1e-5
        assert O.max_rel(O.c_conv_dx(x.shape, wt, go, pad), O.torch_conv_dx(x.shape, wt, go, pad)) < 1e-5
        assert O.norm_rel(O.c_conv_dw(x, go, wt.shape, pad), O.torch_conv_dw(x, go, wt.shape, pad)) < 1e-5
    assert O.max_rel(O.c_bias_grad(go), go.sum(dim=(0, 2, 3, 4))) < 1e-5


def test_reference_k3_dx_pad_bug_documented():
    """The reference's k3 dX reuses the forward padding; for pad 0 that gives
    the wrong shape. The oracle (and the B200 kernels) use pad' = 2 - pad."""
    torch.manual_seed(0)
    x = torch.randn(1, 4, 5, 6, 7)
    wt = torch.randn(3, 4, 3, 3, 3)
    go = torch.randn(1, 3, 3, 4, 5)
    dx = O.c_conv_dx(x.shape, wt, go, 0)
    assert dx.shape == x.shape
    assert O.max_rel(dx, O.torch_conv_dx(x.shape, wt, go, 0)) < 1e-5
    # what the reference computes: conv3d(dY, rot180(W)^T, pad 0) -> wrong size
    wf = wt.flip(2, 3, 4).transpose(0, 1)
    assert torch.nn.functional.conv3d(go, wf, None, 1, 0).shape != x.shape


def test_split_order_is_deterministic():
    torch.manual_seed(1)
    x = torch.randn(2, 8, 4, 5, 6)
    go = torch.randn(2, 8, 4, 5, 6)
    a = O.c_conv_dw(x, go, (8, 8, 3, 3, 3), 1, split=7)
    b = O.c_conv_dw(x, go, (8, 8, 3, 3, 3), 1, split=7)
    assert torch.equal(a, b)
