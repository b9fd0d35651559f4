"""Parity oracle for the Conv3d hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` leg
may import this module; the product (``rdna4_conv3d``) never does.

Two checkers live here:

* ``c_*`` — ctypes wrappers of ``conv3d_oracle.c``, a plain-C restatement of
  the reference's implicit-GEMM algorithm (packed-weight layouts, tap-major K
  order, split-K partials summed in split order). Pinned against golden
  vectors that the reference's own Triton kernels produced
  (tests/golden/make_golden.py).
* ``torch_*`` — the reference's CPU path: on CPU tensors ``Conv3dWmma`` is
  ``nn.Conv3d.forward`` (src/rdna4_conv3d/conv3d_wmma.py:1437-1438) and the
  fallback gradients are ``torch.nn.grad.conv3d_input/_weight``
  (conv3d_wmma.py:1299-1314), all in fp32 here.

All helpers take and return NCDHW fp32 torch tensors.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import torch
import torch.nn.functional as F

_DIR = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_DIR, "liboracle_conv3d.so")
_lib = None


def build() -> str:
    src = os.path.join(_DIR, "conv3d_oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _DIR], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_SO)
        fp = ctypes.POINTER(ctypes.c_float)
        i = ctypes.c_int
        L.oracle_pack_weight.argtypes = [fp, i, i, i, fp]
        L.oracle_unpack_weight.argtypes = [fp, i, i, i, fp]
        L.oracle_conv_fwd.argtypes = [fp, i, i, i, i, i, fp, i, i, i, i, i, fp, fp]
        L.oracle_conv_dgrad.argtypes = [fp, i, i, i, i, i, fp, i, i, i, i, i, fp]
        L.oracle_conv_wgrad.argtypes = [fp, fp, i, i, i, i, i, i, i, i, i, i, i, fp]
        L.oracle_bias_grad.argtypes = [fp, ctypes.c_int64, i, fp]
        L.oracle_tr_pack_w.argtypes = [fp, i, i, fp]
        L.oracle_tr_unpack_w.argtypes = [fp, i, i, fp]
        L.oracle_tconv_fwd.argtypes = [fp, i, i, i, i, i, fp, i, fp, fp]
        L.oracle_tconv_dx.argtypes = [fp, i, i, i, i, i, fp, i, fp]
        L.oracle_tconv_dw.argtypes = [fp, fp, i, i, i, i, i, i, i, fp]
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.detach().to(torch.float32).cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _ndhwc(t: torch.Tensor) -> np.ndarray:
    return _f32(t.detach().float().permute(0, 2, 3, 4, 1))


def _ncdhw(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a).permute(0, 4, 1, 2, 3).contiguous()


def _t3(v):
    return (v, v, v) if isinstance(v, int) else tuple(int(x) for x in v)


def _osz(i, k, p):
    return i + 2 * p - (k - 1)


# ---------------------------------------------------------------------------
# C restatement
# ---------------------------------------------------------------------------
def c_pack_weight(w: torch.Tensor) -> np.ndarray:
    cout, cin, k = int(w.shape[0]), int(w.shape[1]), int(w.shape[2])
    src = _f32(w)
    out = np.empty((k ** 3 * cin, cout), np.float32)
    lib().oracle_pack_weight(_p(src), cout, cin, k, _p(out))
    return out


def c_conv_fwd(x: torch.Tensor, w: torch.Tensor, b=None, padding=0) -> torch.Tensor:
    n, cin, d, h, ww = (int(s) for s in x.shape)
    cout, k = int(w.shape[0]), int(w.shape[2])
    pd, ph, pw = _t3(padding)
    xs, wp = _ndhwc(x), c_pack_weight(w)
    bs = None if b is None else _f32(b)
    y = np.empty((n, _osz(d, k, pd), _osz(h, k, ph), _osz(ww, k, pw), cout), np.float32)
    lib().oracle_conv_fwd(_p(xs), n, d, h, ww, cin, _p(wp), cout, k, pd, ph, pw,
                          None if bs is None else _p(bs), _p(y))
    return _ncdhw(y)


def c_conv_dx(x_shape, w: torch.Tensor, go: torch.Tensor, padding=0) -> torch.Tensor:
    n, cin, d, h, ww = (int(s) for s in x_shape)
    cout, k = int(w.shape[0]), int(w.shape[2])
    pd, ph, pw = _t3(padding)
    gs, wp = _ndhwc(go), c_pack_weight(w)
    dx = np.empty((n, d, h, ww, cin), np.float32)
    lib().oracle_conv_dgrad(_p(gs), n, d, h, ww, cin, _p(wp), cout, k, pd, ph, pw, _p(dx))
    return _ncdhw(dx)


def c_conv_dw(x: torch.Tensor, go: torch.Tensor, w_shape, padding=0, split=4) -> torch.Tensor:
    n, cin, d, h, ww = (int(s) for s in x.shape)
    cout, k = int(w_shape[0]), int(w_shape[2])
    pd, ph, pw = _t3(padding)
    xs, gs = _ndhwc(x), _ndhwc(go)
    dwp = np.empty((k ** 3 * cin, cout), np.float32)
    lib().oracle_conv_wgrad(_p(xs), _p(gs), n, d, h, ww, cin, cout, k, pd, ph, pw, split, _p(dwp))
    out = np.empty((cout, cin, k, k, k), np.float32)
    lib().oracle_unpack_weight(_p(dwp), cout, cin, k, _p(out))
    return torch.from_numpy(out)


def c_bias_grad(go: torch.Tensor) -> torch.Tensor:
    gs = _ndhwc(go)
    cout = int(go.shape[1])
    db = np.empty((cout,), np.float32)
    lib().oracle_bias_grad(_p(gs), int(gs.size // max(cout, 1)), cout, _p(db))
    return torch.from_numpy(db)


def c_tr_pack(w: torch.Tensor) -> np.ndarray:
    cin, cout = int(w.shape[0]), int(w.shape[1])
    out = np.empty((cin, 8 * cout), np.float32)
    lib().oracle_tr_pack_w(_p(_f32(w)), cin, cout, _p(out))
    return out


def c_tconv_fwd(x: torch.Tensor, w: torch.Tensor, b=None) -> torch.Tensor:
    n, cin, d, h, ww = (int(s) for s in x.shape)
    cout = int(w.shape[1])
    xs, wp = _ndhwc(x), c_tr_pack(w)
    bs = None if b is None else _f32(b)
    y = np.empty((n, 2 * d, 2 * h, 2 * ww, cout), np.float32)
    lib().oracle_tconv_fwd(_p(xs), n, d, h, ww, cin, _p(wp), cout, None if bs is None else _p(bs), _p(y))
    return _ncdhw(y)


def c_tconv_dx(x_shape, w: torch.Tensor, go: torch.Tensor) -> torch.Tensor:
    n, cin, d, h, ww = (int(s) for s in x_shape)
    cout = int(w.shape[1])
    gs, wp = _ndhwc(go), c_tr_pack(w)
    dx = np.empty((n, d, h, ww, cin), np.float32)
    lib().oracle_tconv_dx(_p(gs), n, d, h, ww, cin, _p(wp), cout, _p(dx))
    return _ncdhw(dx)


def c_tconv_dw(x: torch.Tensor, go: torch.Tensor, cout: int, split=4) -> torch.Tensor:
    n, cin, d, h, ww = (int(s) for s in x.shape)
    xs, gs = _ndhwc(x), _ndhwc(go)
    dwp = np.empty((cin, 8 * cout), np.float32)
    lib().oracle_tconv_dw(_p(xs), _p(gs), n, d, h, ww, cin, cout, split, _p(dwp))
    out = np.empty((cin, cout, 2, 2, 2), np.float32)
    lib().oracle_tr_unpack_w(_p(dwp), cin, cout, _p(out))
    return torch.from_numpy(out)


# ---------------------------------------------------------------------------
# The reference's CPU path (stock PyTorch, fp32)
# ---------------------------------------------------------------------------
def torch_conv_fwd(x, w, b=None, padding=0):
    return F.conv3d(x.float().cpu(), w.float().cpu(), None if b is None else b.float().cpu(), 1, padding)


def torch_conv_dx(x_shape, w, go, padding=0):
    return torch.nn.grad.conv3d_input(tuple(x_shape), w.float().cpu(), go.float().cpu().contiguous(), 1,
                                      padding, 1, 1)


def torch_conv_dw(x, go, w_shape, padding=0):
    return torch.nn.grad.conv3d_weight(x.float().cpu(), tuple(w_shape), go.float().cpu().contiguous(), 1,
                                       padding, 1, 1)


def torch_tconv_fwd(x, w, b=None):
    return F.conv_transpose3d(x.float().cpu(), w.float().cpu(), None if b is None else b.float().cpu(), 2)


def torch_tconv_grads(x, w, go):
    xr = x.detach().float().cpu().requires_grad_(True)
    wr = w.detach().float().cpu().requires_grad_(True)
    F.conv_transpose3d(xr, wr, None, 2).backward(go.float().cpu())
    return xr.grad, wr.grad


# ---------------------------------------------------------------------------
# Error metrics used by the parity tests
# ---------------------------------------------------------------------------
def max_rel(out: torch.Tensor, ref: torch.Tensor) -> float:
    """max |out - ref| / max |ref| (normalised max error)."""
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    den = ref.abs().max().item()
    return (out - ref).abs().max().item() / (den if den > 0 else 1.0)


def norm_rel(out: torch.Tensor, ref: torch.Tensor) -> float:
    """||out - ref||_2 / ||ref||_2."""
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    den = ref.norm().item()
    return (out - ref).norm().item() / (den if den > 0 else 1.0)
