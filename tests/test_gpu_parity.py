"""Kernel parity on a B200: every leg against the oracle, through the product path.

Oracle: the reference's CPU path (stock PyTorch fp32 on CPU; oracle/oracle.py)
fed the same bf16/fp16-rounded inputs, plus the golden vectors the reference's
own Triton kernels produced (tests/golden). Tolerances are the north-star
ones, written here:
  forward and dX : max|out - ref| / max|ref| <= 2e-2
  dW, db         : ||out - ref|| / ||ref||   <= 3e-2
"""
import glob
import os

import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN_DIR

pytestmark = pytest.mark.gpu

FWD_TOL = 2e-2
DW_TOL = 3e-2

# n, cin, cout, d, h, w, k, pad
CONV_CASES = [
    (2, 24, 24, 16, 32, 32, 3, 1),
    (2, 5, 7, 9, 11, 13, 3, 1),        # reference test shapes
    (2, 24, 1, 8, 16, 16, 1, 0),
    (1, 24, 24, 8, 16, 16, 3, 1),
    (1, 1, 24, 8, 16, 16, 3, 1),
    (1, 16, 8, 6, 7, 9, 3, 0),         # pad 0 / pad 2
    (1, 8, 16, 4, 5, 6, 3, 2),
    (1, 24, 24, 5, 9, 11, 3, 0),
    (1, 24, 24, 5, 9, 11, 3, 2),
    (1, 16, 8, 4, 5, 6, 1, 1),         # k1 with padding
    (1, 48, 48, 8, 16, 16, 3, 1),      # trunk channel counts, reduced volume
    (1, 96, 96, 4, 8, 8, 3, 1),
    (1, 192, 192, 4, 8, 8, 3, 1),
    (1, 48, 24, 8, 16, 16, 1, 0),
    (1, 96, 48, 4, 8, 8, 1, 0),
    (1, 192, 96, 4, 8, 8, 1, 0),
    (1, 8, 8, 3, 3, 3, 3, 1),          # one 8-channel chunk
    (1, 40, 16, 4, 6, 10, 3, 1),       # five chunks (odd pairing)
    (2, 24, 48, 3, 5, 130, 3, 1),      # W above 128
    (1, 8, 8, 2, 2, 300, 3, 1),        # W split into two tiles
    (1, 16, 200, 3, 4, 5, 3, 1),       # Cout not a multiple of 16
    (1, 32, 256, 2, 4, 8, 3, 1),       # Cout = 256
    (0, 24, 24, 4, 4, 4, 3, 1),        # empty batch
    # stem kernel (forward, 1..4 input channels, W*Cin a multiple of 8)
    (2, 2, 16, 5, 9, 12, 3, 1),
    (1, 3, 8, 4, 6, 8, 3, 0),
    (1, 4, 32, 3, 5, 10, 3, 2),
    (1, 1, 24, 3, 4, 200, 3, 1),       # brick row of 200 columns
    (1, 1, 24, 2, 3, 296, 3, 1),       # two brick columns
    (1, 4, 24, 2, 3, 100, 3, 1),       # Cin=4: 50-column bricks
    (1, 1, 48, 6, 7, 16, 3, 1),        # Cout 48: five M tiles per unit
    (1, 1, 7, 3, 5, 8, 3, 1),          # Cout 7: scalar stores
    (1, 2, 256, 2, 3, 8, 3, 1),        # Cout 256
    # stem dX kernel (one input channel, Cout % 4 == 0 up to 32, pad 1, even W <= 256)
    (2, 1, 24, 11, 37, 128, 3, 1),     # two rows per stage, ragged strips and plane slabs
    (1, 1, 8, 5, 6, 64, 3, 1),         # four rows per stage
    (1, 1, 32, 4, 9, 256, 3, 1),       # one row of 128 pairs per stage, 4 K steps
    (1, 1, 12, 3, 3, 6, 3, 1),         # 12 rows per stage, pairs straddle warps
    (1, 1, 4, 2, 2, 2, 3, 1),          # one pair per row
    (1, 1, 20, 7, 10, 150, 3, 1),      # 75 pairs: idle lanes in every stage
]
TCONV_CASES = [
    (2, 16, 8, 3, 4, 5),
    (1, 48, 24, 2, 4, 6),
    (1, 192, 96, 2, 4, 4),
    (1, 96, 48, 4, 4, 4),
    (1, 5, 3, 2, 3, 4),
    (0, 16, 8, 2, 2, 2),
    # tcgen05 transpose conv (Cin, Cout multiples of 8): tiles of R rows x W,
    # x segments for W > 128, N split into tasks, 2*Cout over two box groups
    (1, 8, 16, 1, 3, 130),
    (2, 48, 24, 2, 5, 64),
    (1, 192, 96, 3, 8, 16),
    (1, 96, 48, 2, 4, 32),
    # 2 tasks of N = 256: the output staging would leave one load stage, so
    # per-thread stores
    (1, 128, 64, 2, 4, 32),
    (1, 24, 40, 2, 3, 7),
    # last M tile of 8 channels: db from the dW kernel's ones row there
    (1, 136, 16, 2, 3, 8),
    # last M tile of 104 channels: db from the db kernel by default
    (1, 104, 16, 2, 2, 8),
]


def _cw():
    import sys
    return sys.modules["rdna4_conv3d.conv3d_wmma"]


def _ids(cases):
    return ["x".join(str(v) for v in c) for c in cases]


def _inputs(n, cin, cout, d, h, w, k, pad, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, cin, d, h, w, generator=g).to(dtype)
    wt = (torch.randn(cout, cin, k, k, k, generator=g) / (cin * k ** 3) ** 0.5).to(dtype)
    b = torch.randn(cout, generator=g).to(dtype)
    od, oh, ow = d + 2 * pad - (k - 1), h + 2 * pad - (k - 1), w + 2 * pad - (k - 1)
    go = torch.randn(n, cout, od, oh, ow, generator=g).to(dtype)
    return x, wt, b, go


def _run_conv(x, wt, b, go, pad):
    cw = _cw()
    dev = "cuda"
    xg, wg, bg, gg = (t.to(dev) for t in (x, wt, b, go))
    y = cw._launch_fwd(xg, wg, bg, (pad,) * 3)
    dx = cw._launch_dgrad(gg, wg, xg.shape, (pad,) * 3)
    dw, db = cw._launch_wgrad(xg, gg, wg.shape, (pad,) * 3, True)
    torch.cuda.synchronize()
    return y.cpu(), dx.cpu(), dw.cpu(), db.cpu()


@pytest.mark.parametrize("force", [0, 1], ids=["auto", "simt"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("case", CONV_CASES, ids=_ids(CONV_CASES))
def test_conv_legs_match_oracle(cuda_ready, case, dtype, force, monkeypatch):
    n, cin, cout, d, h, w, k, pad = case
    if force == 1 and cin * cout * d * h * w * k ** 3 > 40_000_000:
        pytest.skip("SIMT path covered on the smaller shapes")
    monkeypatch.setattr(_cw(), "_FORCE_KERNEL", force)
    x, wt, b, go = _inputs(*case, dtype)
    y, dx, dw, db = _run_conv(x, wt, b, go, pad)
    assert y.shape == (n, cout, d + 2 * pad - (k - 1), h + 2 * pad - (k - 1), w + 2 * pad - (k - 1))
    assert dx.shape == x.shape and dw.shape == wt.shape and dw.dtype == torch.float32
    if n == 0:
        assert float(dw.abs().sum()) == 0.0 and float(db.abs().sum()) == 0.0
        return
    yr = O.torch_conv_fwd(x, wt, b, pad)
    dxr = O.torch_conv_dx(x.shape, wt, go, pad)
    dwr = O.torch_conv_dw(x, go, wt.shape, pad)
    dbr = go.float().sum(dim=(0, 2, 3, 4))
    assert O.max_rel(y, yr) <= FWD_TOL
    assert O.max_rel(dx, dxr) <= FWD_TOL
    assert O.norm_rel(dw, dwr) <= DW_TOL
    assert O.norm_rel(db, dbr) <= DW_TOL
    # fp32 accumulation of identical inputs: far inside the stated bounds
    assert O.norm_rel(dw, dwr) <= 1e-4


# dW in both layouts of the tcgen05 weight-gradient kernel: 8-channel chunks
# and wide swizzled channel groups (R4C_DW_WIDE forces one; with the wide
# one, groups and dY boxes past Cin / Cout are padded with zero channels)
DW_CASES = [
    (1, 48, 48, 4, 8, 8, 3, 1),
    (1, 32, 16, 3, 5, 20, 3, 1),       # one 32-channel group, ragged W
    (2, 96, 96, 3, 6, 10, 3, 1),
    (1, 192, 192, 2, 4, 8, 3, 1),
    (1, 64, 24, 3, 4, 9, 3, 0),        # pad 0, Cout 24 (8-channel dY chunks)
    (1, 192, 96, 4, 8, 8, 1, 0),       # k1
    (1, 48, 24, 4, 8, 8, 1, 0),
    (1, 128, 40, 2, 3, 140, 3, 1),     # W split into two tiles
    (1, 40, 40, 3, 5, 16, 1, 0),       # padded channel group (40 of 64) and dY box (40 of 64)
    (1, 24, 24, 3, 5, 16, 3, 1),       # padded 32-channel group and dY box (24 real)
    (2, 24, 24, 3, 4, 128, 3, 1),      # fold: K = 144 positions, two M tiles (trunk 24->24 row)
    (1, 16, 8, 4, 5, 6, 3, 1),         # rows: 16-channel atoms (8 per M tile), 16-channel dY atoms
    (1, 64, 64, 3, 5, 24, 3, 1),       # rows: two M tiles, N = 192, one kw per task
    (2, 48, 24, 4, 6, 300, 3, 1),      # rows: W split into tiles, Cin padded to 64
    (1, 8, 16, 4, 5, 6, 3, 2),         # pad 2
    (1, 16, 8, 3, 4, 200, 3, 0),       # pad 0, K = 208 positions
]


@pytest.mark.parametrize("layout", ["chunks", "fold", "wide", "rows"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("case", DW_CASES, ids=_ids(DW_CASES))
def test_dw_layouts_match_oracle(cuda_ready, case, dtype, layout, monkeypatch):
    # chunks: 8-channel chunks, one MMA per kw; fold: the same with kw folded
    # into N (three kw-shifted dY copies; k3 rows that fit one W tile);
    # wide: swizzled channel groups; rows: one stage per input row (three
    # input planes as A, three dY rows as B; k3 pad 1, forced for every
    # channel count here — other geometries fall back to the default plan)
    n, cin, cout, d, h, w, k, pad = case
    monkeypatch.setenv("R4C_DW_WIDE", "1" if layout == "wide" else "0")
    monkeypatch.setenv("R4C_DW_FOLD", "1" if layout == "fold" else "0")
    monkeypatch.setenv("R4C_DW_STRIP", "1" if layout == "rows" else "0")
    cw = _cw()
    x, wt, b, go = _inputs(*case, dtype)
    dw, db = cw._launch_wgrad(x.cuda(), go.cuda(), wt.shape, (pad,) * 3, True)
    torch.cuda.synchronize()
    dwr = O.torch_conv_dw(x, go, wt.shape, pad)
    assert O.norm_rel(dw.cpu(), dwr) <= 1e-4
    assert O.norm_rel(db.cpu(), go.float().sum(dim=(0, 2, 3, 4))) <= 1e-4


@pytest.mark.parametrize("force", [0, 1], ids=["auto", "simt"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("case", TCONV_CASES, ids=_ids(TCONV_CASES))
def test_tconv_legs_match_oracle(cuda_ready, case, dtype, force, monkeypatch):
    n, cin, cout, d, h, w = case
    cw = _cw()
    monkeypatch.setattr(cw, "_FORCE_KERNEL", force)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(n, cin, d, h, w, generator=g).to(dtype)
    wt = (torch.randn(cin, cout, 2, 2, 2, generator=g) / cin ** 0.5).to(dtype)
    b = torch.randn(cout, generator=g).to(dtype)
    go = torch.randn(n, cout, 2 * d, 2 * h, 2 * w, generator=g).to(dtype)
    xg, wg, bg, gg = (t.cuda() for t in (x, wt, b, go))
    y = cw.transpose_k2s2_fwd(xg, wg, bg).cpu()
    dx = cw.transpose_k2s2_dx(xg.shape, wg, gg).cpu()
    dw, db = cw.transpose_k2s2_dw(xg, wg.shape, gg, True)
    dw, db = dw.cpu(), db.cpu()
    assert y.shape == (n, cout, 2 * d, 2 * h, 2 * w) and dx.shape == x.shape and dw.shape == wt.shape
    if n == 0:
        return
    dxr, dwr = O.torch_tconv_grads(x, wt, go)
    assert O.max_rel(y, O.torch_tconv_fwd(x, wt, b)) <= FWD_TOL
    assert O.max_rel(dx, dxr) <= FWD_TOL
    assert O.norm_rel(dw, dwr) <= 1e-4
    assert O.norm_rel(db, go.float().sum(dim=(0, 2, 3, 4))) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("case", [(1, 104, 16, 2, 2, 8), (1, 96, 48, 2, 4, 32)], ids=["104x16", "96x48"])
def test_tconv_dw_db_fill_opt_in(cuda_ready, case, dtype, tmp_path):
    """R4C_TCONV_DBFILL=1: db from a 1 written into the zero fill of a last
    M tile of 72-120 channels, checked against the same oracle as the default.
    The library reads the switch once per process, so the GPU leg runs in a
    child process started with it set."""
    import subprocess
    import sys
    n, cin, cout, d, h, w = case
    g = torch.Generator().manual_seed(1)
    x = torch.randn(n, cin, d, h, w, generator=g).to(dtype)
    wt = (torch.randn(cin, cout, 2, 2, 2, generator=g) / cin ** 0.5).to(dtype)
    go = torch.randn(n, cout, 2 * d, 2 * h, 2 * w, generator=g).to(dtype)
    torch.save({"x": x, "wshape": tuple(wt.shape), "go": go}, tmp_path / "in.pt")
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rdna4-conv3d-wmma_b200")
    code = (
        "import sys, torch; sys.path.insert(0, %r)\n"
        "import rdna4_conv3d\n"
        "cw = sys.modules['rdna4_conv3d.conv3d_wmma']\n"
        "t = torch.load(%r)\n"
        "dw, db = cw.transpose_k2s2_dw(t['x'].cuda(), t['wshape'], t['go'].cuda(), True)\n"
        "torch.save({'dw': dw.cpu(), 'db': db.cpu()}, %r)\n"
    ) % (pkg, str(tmp_path / "in.pt"), str(tmp_path / "out.pt"))
    env = dict(os.environ, R4C_TCONV_DBFILL="1")
    subprocess.run([sys.executable, "-c", code], env=env, check=True, timeout=600)
    out = torch.load(tmp_path / "out.pt")
    _, dwr = O.torch_tconv_grads(x, wt, go)
    assert O.norm_rel(out["dw"], dwr) <= 1e-4
    assert O.norm_rel(out["db"], go.float().sum(dim=(0, 2, 3, 4))) <= 1e-4


GOLDEN =sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_matches_reference_golden(cuda_ready, path):
    """fp16 kernels vs the reference's fp16 Triton outputs on identical inputs."""
    z = np.load(path)
    n, cin, cout, d, h, w, k, pad = (int(v) for v in z["meta"])
    cw = _cw()
    x, wt, b, go = (torch.from_numpy(z[key]).cuda() for key in ("x", "w", "b", "go"))
    if k == 2:
        y = cw.transpose_k2s2_fwd(x, wt, b)
        dx = cw.transpose_k2s2_dx(x.shape, wt, go)
        dw, _ = cw.transpose_k2s2_dw(x, wt.shape, go)
    else:
        y = cw._launch_fwd(x, wt, b, (pad,) * 3)
        dx = cw._launch_dgrad(go, wt, x.shape, (pad,) * 3)
        dw, _ = cw._launch_wgrad(x, go, wt.shape, (pad,) * 3, False)
    assert O.max_rel(y.cpu(), torch.from_numpy(z["y"])) < 4e-3
    assert O.norm_rel(dw.cpu(), torch.from_numpy(z["dw"])) < 2e-3
    if "dx" in z.files:
        assert O.max_rel(dx.cpu(), torch.from_numpy(z["dx"])) < 4e-3


def test_small_cases_match_c_oracle(cuda_ready):
    """The C restatement of the reference algorithm agrees with the kernels too."""
    for case in [(1, 24, 24, 4, 6, 8, 3, 1), (1, 5, 7, 3, 4, 5, 3, 0), (1, 16, 8, 3, 4, 5, 1, 0)]:
        n, cin, cout, d, h, w, k, pad = case
        x, wt, b, go = _inputs(*case, torch.bfloat16, seed=3)
        y, dx, dw, db = _run_conv(x, wt, b, go, pad)
        assert O.max_rel(y, O.c_conv_fwd(x, wt, b, pad)) <= FWD_TOL
        assert O.max_rel(dx, O.c_conv_dx(x.shape, wt, go, pad)) <= FWD_TOL
        assert O.norm_rel(dw, O.c_conv_dw(x, go, wt.shape, pad)) <= 1e-4
        assert O.norm_rel(db, O.c_bias_grad(go)) <= 1e-4


def test_deterministic_dw(cuda_ready):
    """Split-K partials are summed in a fixed order: bitwise-identical reruns."""
    cw = _cw()
    x, wt, b, go = _inputs(2, 24, 24, 16, 32, 32, 3, 1, torch.bfloat16)
    xg, gg = x.cuda(), go.cuda()
    a, da = cw._launch_wgrad(xg, gg, wt.shape, (1, 1, 1), True)
    c, dc = cw._launch_wgrad(xg, gg, wt.shape, (1, 1, 1), True)
    assert torch.equal(a, c) and torch.equal(da, dc)


def test_kernel_families_used(cuda_ready):
    """The tcgen05 family serves the trunk shapes (no silent SIMT routing)."""
    cw = _cw()
    for shape, cout, k in [((4, 24, 64, 128, 128), 24, 3), ((4, 48, 32, 64, 64), 48, 3),
                           ((4, 96, 16, 32, 32), 96, 3), ((4, 192, 8, 16, 16), 192, 3),
                           ((4, 48, 64, 128, 128), 24, 1)]:
        fam = cw.conv3d_kernels(shape, cout, k, 1 if k == 3 else 0)
        assert fam["fwd"] == "tcgen05" and fam["dx"] == "tcgen05" and fam["dw"] == "tcgen05", (shape, fam)


def test_no_device_error_flag(cuda_ready):
    from rdna4_conv3d import _native
    assert _native.device_error() == 0


# Two input planes per pipeline stage (pps=2) forced on and off through the
# plan override, with odd and even plane counts per unit, k1 and k3.
PPS_CASES = [
    (2, 24, 24, 16, 32, 32, 3, 1),
    (2, 24, 24, 5, 9, 11, 3, 0),
    (2, 24, 24, 5, 9, 11, 3, 2),
    (1, 48, 48, 8, 16, 16, 3, 1),
    (1, 16, 8, 6, 7, 9, 3, 1),
    (1, 40, 16, 4, 6, 10, 3, 1),
    (2, 24, 48, 3, 5, 130, 3, 1),
    (1, 48, 24, 8, 16, 16, 1, 0),
]


@pytest.mark.parametrize("plan", ["pps=2", "pps=2,P=3", "pps=2,P=2,stg=0", "pps=1"])
@pytest.mark.parametrize("case", PPS_CASES, ids=_ids(PPS_CASES))
def test_conv_planes_per_stage(cuda_ready, case, plan, monkeypatch):
    from rdna4_conv3d import _native
    n, cin, cout, d, h, w, k, pad = case
    monkeypatch.setenv("R4C_TC_PLAN", plan)
    x, wt, b, go = _inputs(*case, torch.bfloat16, seed=5)
    desc = _native.make_desc(n, d, h, w, cin, cout, k, (pad,) * 3, torch.bfloat16)
    if "tcgen05 conv" not in _native.describe_plan(desc, _native.LEG_FWD):
        pytest.skip("no plan of this form for the shape")
    y, dx, dw, db = _run_conv(x, wt, b, go, pad)
    assert O.max_rel(y, O.torch_conv_fwd(x, wt, b, pad)) <= FWD_TOL
    assert O.max_rel(dx, O.torch_conv_dx(x.shape, wt, go, pad)) <= FWD_TOL
    assert _native.device_error() == 0
