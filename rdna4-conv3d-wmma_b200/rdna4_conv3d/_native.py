"""ctypes binding of the B200 C-ABI library (``libr4c_conv3d.so``).

This module is the only place Python touches the native kernels. It is the
reference-side binding of ``include/r4c_conv3d.h``: it turns torch tensors into
plain pointers and sizes, passes torch's current CUDA stream, and turns status
codes into exceptions. There is deliberately no host fallback: if the library
is missing or the call fails, the caller gets an exception.

Reference counterpart: the JIT loader of the HIP extension
(src/rdna4_conv3d/hip_backend.py:1-37) and the Triton launchers it sat next to
(src/rdna4_conv3d/conv3d_wmma.py:1015-1227, 1453-1542).
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Tuple

import torch

_LIB_NAME = "libr4c_conv3d.so"
_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), _LIB_NAME)
_lib = None
_lock = threading.Lock()

# Must match include/r4c_conv3d.h.
R4C_OK = 0
R4C_BF16, R4C_F16, R4C_F32 = 0, 1, 2
LEG_FWD, LEG_DX, LEG_DW, LEG_TFWD, LEG_TDX, LEG_TDW = range(6)
KERNEL_NONE, KERNEL_GENERIC, KERNEL_TC = 0, 1, 2


class ConvDesc(ctypes.Structure):
    _fields_ = [
        ("n", ctypes.c_int32), ("d", ctypes.c_int32), ("h", ctypes.c_int32), ("w", ctypes.c_int32),
        ("cin", ctypes.c_int32), ("cout", ctypes.c_int32), ("k", ctypes.c_int32),
        ("pad_d", ctypes.c_int32), ("pad_h", ctypes.c_int32), ("pad_w", ctypes.c_int32),
        ("dtype", ctypes.c_int32), ("force_kernel", ctypes.c_int32),
    ]


class ConvexDesc(ctypes.Structure):
    """r4c_convex_desc: Conv3d of any geometry (include/r4c_conv3d.h)."""
    _fields_ = [(name, ctypes.c_int32) for name in (
        "n", "d", "h", "w", "cin", "cout", "groups", "kd", "kh", "kw", "sd", "sh", "sw",
        "pd", "ph", "pw", "dd", "dh", "dw", "dtype")]


class NativeError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""


def library_path() -> str:
    return _LIB_PATH


def _bind(lib) -> None:
    P = ctypes.c_void_p
    D = ctypes.POINTER(ConvDesc)
    X = ctypes.POINTER(ConvexDesc)
    sz = ctypes.c_size_t
    i = ctypes.c_int
    i64 = ctypes.c_int64
    dbl = ctypes.c_double
    flt = ctypes.c_float
    sig = {
        "r4c_strerror": ([i], ctypes.c_char_p),
        "r4c_version": ([], i),
        "r4c_device_error": ([P, i], i),
        "r4c_watchdog_selftest": ([ctypes.c_uint64, P], i),
        "r4c_launch_count": ([], ctypes.c_uint64),
        "r4c_plan_kernel": ([D, i], i),
        "r4c_describe_plan": ([D, i, ctypes.c_char_p, sz], i),
        "r4c_packed_weight_bytes": ([D, i], sz),
        "r4c_workspace_size": ([D, i], sz),
        "r4c_pack_weight": ([D, i, P, i, P, P], i),
        "r4c_conv3d_fwd": ([D, P, P, P, P, P, sz, P], i),
        "r4c_conv3d_dx": ([D, P, P, P, P, sz, P], i),
        "r4c_conv3d_dw": ([D, P, P, P, P, P, sz, P], i),
        "r4c_tconv_fwd": ([D, P, P, P, P, P, sz, P], i),
        "r4c_tconv_fwd_pitched": ([D, P, P, P, P, i, P, sz, P], i),
        "r4c_tconv_dx": ([D, P, P, P, P, sz, P], i),
        "r4c_tconv_dw": ([D, P, P, P, P, P, sz, P], i),
        "r4c_bn_workspace_size": ([i64, i], sz),
        "r4c_bn_stats": ([P, i64, i, i, P, P, P, sz, P], i),
        "r4c_bn_finalize": ([P, dbl, i, P, P, flt, flt, P, P, P, P, P], i),
        "r4c_bn_relu_fwd": ([P, P, P, P, i64, i, i, i, P], i),
        "r4c_bn_relu_bwd_sums": ([P, P, P, P, i64, i, i, i, P, P, sz, P], i),
        "r4c_bn_relu_bwd_dx": ([P, P, P, P, P, P, dbl, i64, i, i, i, P, P, P, P], i),
        "r4c_channel_slice_copy": ([P, i, P, i64, i, i, P], i),
        "r4c_bn_relu_pool_fwd": ([P, P, i, P, P, P, i, i, i, i, i, i, P], i),
        "r4c_bn_relu_pool_fwd_cat": ([P, P, i, P, P, P, P, i, i, i, i, i, i, P], i),
        "r4c_bn_pool_workspace_size": ([i, i, i, i, i], sz),
        "r4c_bn_relu_pool_bwd_sums": ([P, i, P, P, P, P, P, i, i, i, i, i, i, P, P, sz, P], i),
        "r4c_bn_relu_pool_bwd_dx": ([P, i, P, P, P, P, P, P, P, dbl, i, i, i, i, i, i, P, P, P, P], i),
        "r4c_ce_workspace_size": ([i64], sz),
        "r4c_ce_fwd": ([P, P, i64, i, i, i64, P, P, sz, P], i),
        "r4c_ce_bwd": ([P, P, i64, i, i, i64, P, P, P, P], i),
        "r4c_convex_plan": ([X], i),
        "r4c_convex_workspace_size": ([X, i], sz),
        "r4c_convex_fwd": ([X, P, P, P, P, P, sz, P], i),
        "r4c_convex_dx": ([X, P, P, P, P, sz, P], i),
        "r4c_convex_dw": ([X, P, P, P, P, P, sz, P], i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res


def lib():
    """Load (once) and return the native library; raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise NativeError(
                    f"rdna4_conv3d native library not built: {_LIB_PATH} is missing "
                    "(run `python -m rdna4_conv3d.build` or __graft_entry__.build())")
            handle = ctypes.CDLL(_LIB_PATH)
            _bind(handle)
            _lib = handle
    return _lib


def available() -> bool:
    try:
        lib()
        return True
    except (NativeError, OSError):
        return False


def strerror(status: int) -> str:
    return lib().r4c_strerror(int(status)).decode()


def _check(status: int, what: str) -> None:
    if status != R4C_OK:
        raise NativeError(f"{what} failed: {strerror(status)} (status {status})")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return R4C_BF16
    if dt == torch.float16:
        return R4C_F16
    if dt == torch.float32:
        return R4C_F32
    raise NativeError(f"unsupported dtype {dt}")


def make_desc(n, d, h, w, cin, cout, k, pad, dtype: torch.dtype, force_kernel: int = 0) -> ConvDesc:
    pd, ph, pw = pad
    return ConvDesc(int(n), int(d), int(h), int(w), int(cin), int(cout), int(k),
                    int(pd), int(ph), int(pw), dtype_code(dtype), int(force_kernel))


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _require_cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise NativeError("rdna4_conv3d native kernels need CUDA tensors")
        dev = t.device if dev is None else dev
    return dev


def plan_kernel(desc: ConvDesc, leg: int) -> int:
    return int(lib().r4c_plan_kernel(ctypes.byref(desc), leg))


def describe_plan(desc: ConvDesc, leg: int) -> str:
    buf = ctypes.create_string_buffer(512)
    lib().r4c_describe_plan(ctypes.byref(desc), leg, buf, 512)
    return buf.value.decode()


def workspace_bytes(desc: ConvDesc, leg: int) -> int:
    return int(lib().r4c_workspace_size(ctypes.byref(desc), leg))


def packed_weight_bytes(desc: ConvDesc, leg: int) -> int:
    return int(lib().r4c_packed_weight_bytes(ctypes.byref(desc), leg))


def _workspace(desc: ConvDesc, leg: int, device) -> Tuple[Optional[torch.Tensor], int]:
    nb = workspace_bytes(desc, leg)
    if nb == 0:
        return None, 0
    return torch.empty(nb, dtype=torch.uint8, device=device), nb


def pack_weight(desc: ConvDesc, leg: int, weight: torch.Tensor) -> torch.Tensor:
    """Pack a PyTorch-layout weight for one leg (r4c_pack_weight)."""
    dev = _require_cuda(weight)
    w = weight.contiguous()
    nbytes = packed_weight_bytes(desc, leg)
    if nbytes == 0:
        raise NativeError("descriptor rejected by r4c_packed_weight_bytes")
    out = torch.empty(nbytes // 2, dtype=torch.bfloat16 if desc.dtype == R4C_BF16 else torch.float16,
                      device=dev)
    with torch.cuda.device(dev):
        st = lib().r4c_pack_weight(ctypes.byref(desc), leg, _ptr(w), dtype_code(w.dtype), _ptr(out),
                                   _stream(dev))
    _check(st, "r4c_pack_weight")
    return out


def _ndhwc_empty(n, c, d, h, w, device, dtype) -> torch.Tensor:
    return torch.empty((n, c, d, h, w), device=device, dtype=dtype, memory_format=torch.channels_last_3d)


def _check_out(out: torch.Tensor, shape, dtype) -> torch.Tensor:
    """A caller-given output must be a dense NDHWC buffer of the right size."""
    if (tuple(out.shape) != tuple(shape) or out.dtype != dtype or not out.is_cuda
            or not out.is_contiguous(memory_format=torch.channels_last_3d) or out.data_ptr() % 16):
        raise NativeError(f"out must be a 16-byte aligned channels_last_3d {dtype} tensor of shape {tuple(shape)}")
    return out


def conv_fwd(desc: ConvDesc, x_cl: torch.Tensor, w_packed: torch.Tensor, bias: Optional[torch.Tensor],
             out_shape, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    dev = _require_cuda(x_cl, w_packed, bias)
    od, oh, ow = out_shape
    if out is None:
        y = _ndhwc_empty(desc.n, desc.cout, od, oh, ow, dev, x_cl.dtype)
    else:
        y = _check_out(out, (desc.n, desc.cout, od, oh, ow), x_cl.dtype)
    ws, nb = _workspace(desc, LEG_FWD, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_conv3d_fwd(ctypes.byref(desc), _ptr(x_cl), _ptr(w_packed), _ptr(bias), _ptr(y),
                                  _ptr(ws), nb, _stream(dev))
    _check(st, "r4c_conv3d_fwd")
    return y


def conv_dx(desc: ConvDesc, go_cl: torch.Tensor, w_packed: torch.Tensor,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    dev = _require_cuda(go_cl, w_packed)
    if out is None:
        dx = _ndhwc_empty(desc.n, desc.cin, desc.d, desc.h, desc.w, dev, go_cl.dtype)
    else:
        dx = _check_out(out, (desc.n, desc.cin, desc.d, desc.h, desc.w), go_cl.dtype)
    ws, nb = _workspace(desc, LEG_DX, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_conv3d_dx(ctypes.byref(desc), _ptr(go_cl), _ptr(w_packed), _ptr(dx), _ptr(ws), nb,
                                 _stream(dev))
    _check(st, "r4c_conv3d_dx")
    return dx


def conv_dw(desc: ConvDesc, x_cl: torch.Tensor, go_cl: torch.Tensor, want_db: bool):
    """fp32 OIDHW weight gradient and (optionally) fp32 bias gradient."""
    dev = _require_cuda(x_cl, go_cl)
    k = desc.k
    dw = torch.empty((desc.cout, desc.cin, k, k, k), dtype=torch.float32, device=dev)
    db = torch.empty((desc.cout,), dtype=torch.float32, device=dev) if want_db else None
    ws, nb = _workspace(desc, LEG_DW, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_conv3d_dw(ctypes.byref(desc), _ptr(x_cl), _ptr(go_cl), _ptr(dw), _ptr(db), _ptr(ws), nb,
                                 _stream(dev))
    _check(st, "r4c_conv3d_dw")
    return dw, db


def tconv_fwd(desc: ConvDesc, x_cl: torch.Tensor, w_packed: torch.Tensor,
              bias: Optional[torch.Tensor]) -> torch.Tensor:
    dev = _require_cuda(x_cl, w_packed, bias)
    y = _ndhwc_empty(desc.n, desc.cout, 2 * desc.d, 2 * desc.h, 2 * desc.w, dev, x_cl.dtype)
    ws, nb = _workspace(desc, LEG_TFWD, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_tconv_fwd(ctypes.byref(desc), _ptr(x_cl), _ptr(w_packed), _ptr(bias), _ptr(y),
                                 _ptr(ws), nb, _stream(dev))
    _check(st, "r4c_tconv_fwd")
    return y


def tconv_fwd_into(desc: ConvDesc, x_cl: torch.Tensor, w_packed: torch.Tensor, bias: Optional[torch.Tensor],
                   buf: torch.Tensor) -> None:
    """The transpose conv's output written into channels [0, Cout) of ``buf``,
    a dense NDHWC buffer with more channels (r4c_tconv_fwd_pitched)."""
    dev = _require_cuda(x_cl, w_packed, bias, buf)
    pitch = int(buf.shape[1])
    if (tuple(buf.shape) != (desc.n, pitch, 2 * desc.d, 2 * desc.h, 2 * desc.w) or buf.dtype != x_cl.dtype
            or not buf.is_contiguous(memory_format=torch.channels_last_3d) or buf.data_ptr() % 16 or pitch < desc.cout):
        raise NativeError("buf must be a 16-byte aligned channels_last_3d tensor (N, >= Cout, 2D, 2H, 2W) of x's dtype")
    ws, nb = _workspace(desc, LEG_TFWD, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_tconv_fwd_pitched(ctypes.byref(desc), _ptr(x_cl), _ptr(w_packed), _ptr(bias), _ptr(buf),
                                         pitch, _ptr(ws), nb, _stream(dev))
    _check(st, "r4c_tconv_fwd_pitched")


def tconv_dx(desc: ConvDesc, go_cl: torch.Tensor, w_packed: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(go_cl, w_packed)
    dx = _ndhwc_empty(desc.n, desc.cin, desc.d, desc.h, desc.w, dev, go_cl.dtype)
    ws, nb = _workspace(desc, LEG_TDX, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_tconv_dx(ctypes.byref(desc), _ptr(go_cl), _ptr(w_packed), _ptr(dx), _ptr(ws), nb,
                                _stream(dev))
    _check(st, "r4c_tconv_dx")
    return dx


def tconv_dw(desc: ConvDesc, x_cl: torch.Tensor, go_cl: torch.Tensor, want_db: bool):
    dev = _require_cuda(x_cl, go_cl)
    dw = torch.empty((desc.cin, desc.cout, 2, 2, 2), dtype=torch.float32, device=dev)
    db = torch.empty((desc.cout,), dtype=torch.float32, device=dev) if want_db else None
    ws, nb = _workspace(desc, LEG_TDW, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_tconv_dw(ctypes.byref(desc), _ptr(x_cl), _ptr(go_cl), _ptr(dw), _ptr(db), _ptr(ws), nb,
                                _stream(dev))
    _check(st, "r4c_tconv_dw")
    return dw, db


# ---------------------------------------------------------------------------
# Conv3d of any geometry (r4c_convex_*)
# ---------------------------------------------------------------------------
def make_convex_desc(x_shape, w_shape, stride, padding, dilation, groups, dtype: torch.dtype) -> ConvexDesc:
    n, cin, d, h, w = (int(v) for v in x_shape)
    cout, _, kd, kh, kw = (int(v) for v in w_shape)
    return ConvexDesc(n, d, h, w, cin, cout, int(groups), kd, kh, kw, *(int(v) for v in stride),
                      *(int(v) for v in padding), *(int(v) for v in dilation), dtype_code(dtype))


def convex_out_shape(desc: ConvexDesc):
    o = lambda i, k, s, p, dl: (i + 2 * p - dl * (k - 1) - 1) // s + 1  # noqa: E731
    return (desc.n, desc.cout, o(desc.d, desc.kd, desc.sd, desc.pd, desc.dd), o(desc.h, desc.kh, desc.sh, desc.ph, desc.dh),
            o(desc.w, desc.kw, desc.sw, desc.pw, desc.dw))


def convex_plan(desc: ConvexDesc) -> int:
    return int(lib().r4c_convex_plan(ctypes.byref(desc)))


def _convex_ws(desc: ConvexDesc, leg: int, device):
    nb = int(lib().r4c_convex_workspace_size(ctypes.byref(desc), leg))
    if nb == 0:
        return None, 0
    return torch.empty(nb, dtype=torch.uint8, device=device), nb


def convex_fwd(desc: ConvexDesc, x_cl: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
    dev = _require_cuda(x_cl, w, bias)
    shp = convex_out_shape(desc)
    y = _ndhwc_empty(*shp, dev, x_cl.dtype)
    ws, nb = _convex_ws(desc, LEG_FWD, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_convex_fwd(ctypes.byref(desc), _ptr(x_cl), _ptr(w), _ptr(bias), _ptr(y), _ptr(ws), nb,
                                  _stream(dev))
    _check(st, "r4c_convex_fwd")
    return y


def convex_dx(desc: ConvexDesc, go_cl: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(go_cl, w)
    dx = _ndhwc_empty(desc.n, desc.cin, desc.d, desc.h, desc.w, dev, go_cl.dtype)
    ws, nb = _convex_ws(desc, LEG_DX, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_convex_dx(ctypes.byref(desc), _ptr(go_cl), _ptr(w), _ptr(dx), _ptr(ws), nb, _stream(dev))
    _check(st, "r4c_convex_dx")
    return dx


def convex_dw(desc: ConvexDesc, x_cl: torch.Tensor, go_cl: torch.Tensor, want_db: bool):
    dev = _require_cuda(x_cl, go_cl)
    dw = torch.empty((desc.cout, desc.cin // desc.groups, desc.kd, desc.kh, desc.kw), dtype=torch.float32, device=dev)
    db = torch.empty((desc.cout,), dtype=torch.float32, device=dev) if want_db else None
    ws, nb = _convex_ws(desc, LEG_DW, dev)
    with torch.cuda.device(dev):
        st = lib().r4c_convex_dw(ctypes.byref(desc), _ptr(x_cl), _ptr(go_cl), _ptr(dw), _ptr(db), _ptr(ws), nb,
                                 _stream(dev))
    _check(st, "r4c_convex_dw")
    return dw, db


# ---------------------------------------------------------------------------
# BatchNorm3d + ReLU (r4c_bn_*)
# ---------------------------------------------------------------------------
def bn_relu_forward(x_cl: torch.Tensor, gamma, beta, running_mean, running_var, momentum: float, eps: float,
                    relu: bool, sums_hook=None, pivot=None, apply: bool = True):
    """Training forward. Returns (y, mean_invstd, affine, count).
    ``sums_hook(sums, count)``, when given, may all-reduce the per-channel
    sums in place before they are finalised and returns the total count (a
    volume sharded over ranks: every rank then passes the same ``pivot``)."""
    dev = _require_cuda(x_cl)
    C = int(x_cl.shape[1])
    vox = x_cl.numel() // C
    L = lib()
    f32 = dict(dtype=torch.float32, device=dev)
    ws = torch.empty(int(L.r4c_bn_workspace_size(vox, C)), dtype=torch.uint8, device=dev)
    sums = torch.empty(3 * C, **f32)
    mi = torch.empty(2 * C, **f32)
    ss = torch.empty(2 * C, **f32)
    y = torch.empty_like(x_cl, memory_format=torch.channels_last_3d) if apply else None
    dt = dtype_code(x_cl.dtype)
    with torch.cuda.device(dev):
        st = L.r4c_bn_stats(_ptr(x_cl), vox, C, dt, _ptr(pivot), _ptr(sums), _ptr(ws), ws.numel(), _stream(dev))
        _check(st, "r4c_bn_stats")
        count = float(vox)
        if sums_hook is not None:
            count = float(sums_hook(sums, count))
        st = L.r4c_bn_finalize(_ptr(sums), count, C, _ptr(gamma), _ptr(beta), float(eps), float(momentum),
                               _ptr(running_mean), _ptr(running_var), _ptr(mi), _ptr(ss), _stream(dev))
        _check(st, "r4c_bn_finalize")
        if apply:
            st = L.r4c_bn_relu_fwd(_ptr(x_cl), _ptr(y), _ptr(mi), _ptr(ss), vox, C, dt, 1 if relu else 0,
                                   _stream(dev))
            _check(st, "r4c_bn_relu_fwd")
    return (y if apply else None), mi, ss, count


def bn_relu_backward(dy_cl: torch.Tensor, x_cl: torch.Tensor, mean_invstd, affine, count: float, relu: bool,
                     need_dx: bool = True, sums_hook=None):
    """(dx or None, dgamma, dbeta), fp32 parameter gradients."""
    dev = _require_cuda(dy_cl, x_cl)
    C = int(x_cl.shape[1])
    vox = x_cl.numel() // C
    L = lib()
    f32 = dict(dtype=torch.float32, device=dev)
    ws = torch.empty(int(L.r4c_bn_workspace_size(vox, C)), dtype=torch.uint8, device=dev)
    sums = torch.empty(2 * C, **f32)
    dg = torch.empty(C, **f32)
    db = torch.empty(C, **f32)
    coef = torch.empty(3 * C, **f32)
    dx = torch.empty_like(x_cl, memory_format=torch.channels_last_3d) if need_dx else None
    dt = dtype_code(x_cl.dtype)
    with torch.cuda.device(dev):
        st = L.r4c_bn_relu_bwd_sums(_ptr(dy_cl), _ptr(x_cl), _ptr(mean_invstd), _ptr(affine), vox, C, dt,
                                    1 if relu else 0, _ptr(sums), _ptr(ws), ws.numel(), _stream(dev))
        _check(st, "r4c_bn_relu_bwd_sums")
        if sums_hook is not None:
            sums_hook(sums, None)
        st = L.r4c_bn_relu_bwd_dx(_ptr(dy_cl), _ptr(x_cl), _ptr(dx), _ptr(mean_invstd), _ptr(affine),
                                  _ptr(sums), float(count), vox, C, dt, 1 if relu else 0, _ptr(dg), _ptr(db),
                                  _ptr(coef), _stream(dev))
        _check(st, "r4c_bn_relu_bwd_dx")
    return dx, dg, db


def channel_slice_dense(t: torch.Tensor) -> Optional[torch.Tensor]:
    """A dense channels_last_3d copy of ``t`` when ``t`` is a channel slice of
    a wider NDHWC tensor (voxel stride = pitch >= C, channel stride 1), made
    by the library's slice copy; None when ``t`` is not such a slice or the
    copy's alignment rules do not hold."""
    if t.dim() != 5 or not t.is_cuda or t.dtype not in (torch.bfloat16, torch.float16):
        return None
    n, C, d, h, w = (int(v) for v in t.shape)
    sn, sc, sd, sh, sw = t.stride()
    pitch = sw
    if (sc != 1 or C % 8 or pitch % 8 or pitch < C or sh != pitch * w or sd != pitch * w * h
            or (n > 1 and sn != pitch * w * h * d) or t.data_ptr() % 16):
        return None
    dev = t.device
    out = _ndhwc_empty(n, C, d, h, w, dev, t.dtype)
    with torch.cuda.device(dev):
        st = lib().r4c_channel_slice_copy(_ptr(t), pitch, _ptr(out), n * d * h * w, C, dtype_code(t.dtype),
                                          _stream(dev))
    _check(st, "r4c_channel_slice_copy")
    return out


def bn_relu_pool_forward(x_cl: torch.Tensor, mean_invstd, affine, lead: int):
    """(buf, p, argmax): buf is a new NDHWC tensor of lead + C channels whose
    channels [lead, lead + C) hold relu(bn(x)) (the first lead channels zero
    when lead is a multiple of 8, else unwritten: the caller's), p the 2x2x2
    max-pool of those channels, argmax the windows' argmax for the backward
    (int16 storage of the uint16 fields; None when lead is not a multiple of 8)."""
    dev = _require_cuda(x_cl)
    n, C, d, h, w = (int(v) for v in x_cl.shape)
    buf = _ndhwc_empty(n, lead + C, d, h, w, dev, x_cl.dtype)
    p = _ndhwc_empty(n, C, d // 2, h // 2, w // 2, dev, x_cl.dtype)
    am = None
    with torch.cuda.device(dev):
        if lead % 8 == 0:
            # whole voxels in one pass (channels [0, lead) zero until the up-conv writes them)
            am = torch.empty(n * (d // 2) * (h // 2) * (w // 2) * (C // 4), dtype=torch.int16, device=dev)
            st = lib().r4c_bn_relu_pool_fwd_cat(_ptr(x_cl), _ptr(buf), lead, _ptr(p), _ptr(am), _ptr(mean_invstd),
                                                _ptr(affine), n, d, h, w, C, dtype_code(x_cl.dtype), _stream(dev))
        else:
            yptr = ctypes.c_void_p(buf.data_ptr() + lead * buf.element_size())
            st = lib().r4c_bn_relu_pool_fwd(_ptr(x_cl), yptr, lead + C, _ptr(p), _ptr(mean_invstd), _ptr(affine),
                                            n, d, h, w, C, dtype_code(x_cl.dtype), _stream(dev))
    _check(st, "r4c_bn_relu_pool_fwd")
    return buf, p, am


def bn_relu_pool_backward(gbuf_cl: torch.Tensor, lead: int, gp_cl: torch.Tensor, x_cl: torch.Tensor, mean_invstd,
                          affine, count: float, need_dx: bool = True, sums_hook=None, argmax=None):
    """(dx or None, dgamma, dbeta) from dY = channels [lead, lead + C) of gbuf
    and dP = gp; argmax: the forward's (None: recomputed from x)."""
    dev = _require_cuda(gbuf_cl, gp_cl, x_cl)
    n, C, d, h, w = (int(v) for v in x_cl.shape)
    L = lib()
    f32 = dict(dtype=torch.float32, device=dev)
    ws = torch.empty(int(L.r4c_bn_pool_workspace_size(n, d, h, w, C)), dtype=torch.uint8, device=dev)
    sums = torch.empty(2 * C, **f32)
    dg = torch.empty(C, **f32)
    db = torch.empty(C, **f32)
    coef = torch.empty(3 * C, **f32)
    dx = _ndhwc_empty(n, C, d, h, w, dev, x_cl.dtype) if need_dx else None
    dt = dtype_code(x_cl.dtype)
    pitch = int(gbuf_cl.shape[1])
    gyptr = ctypes.c_void_p(gbuf_cl.data_ptr() + lead * gbuf_cl.element_size())
    with torch.cuda.device(dev):
        st = L.r4c_bn_relu_pool_bwd_sums(gyptr, pitch, _ptr(gp_cl), _ptr(argmax), _ptr(x_cl), _ptr(mean_invstd),
                                         _ptr(affine),
                                         n, d, h, w, C, dt, _ptr(sums), _ptr(ws), ws.numel(), _stream(dev))
        _check(st, "r4c_bn_relu_pool_bwd_sums")
        if sums_hook is not None:
            sums_hook(sums, None)
        st = L.r4c_bn_relu_pool_bwd_dx(gyptr, pitch, _ptr(gp_cl), _ptr(argmax), _ptr(x_cl), _ptr(dx),
                                       _ptr(mean_invstd),
                                       _ptr(affine), _ptr(sums), float(count), n, d, h, w, C, dt, _ptr(dg), _ptr(db),
                                       _ptr(coef), _stream(dev))
        _check(st, "r4c_bn_relu_pool_bwd_dx")
    return dx, dg, db


def launch_count() -> int:
    """Kernels launched by the native library so far in this process."""
    return int(lib().r4c_launch_count())


def watchdog_selftest(limit_ns: int, device=None) -> None:
    """Launch the bounded-wait self-test (a wait that runs out after limit_ns)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _check(lib().r4c_watchdog_selftest(int(limit_ns), _stream(dev)), "r4c_watchdog_selftest")


def device_error(device=None, clear: bool = True) -> int:
    """Read (and clear) the kernels' device-side timeout flag."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        return int(lib().r4c_device_error(_stream(dev), 1 if clear else 0))


# ---------------------------------------------------------------------------
# Cross-entropy over NDHWC logits (r4c_ce_*)
# ---------------------------------------------------------------------------
def ce_forward(logits_cl: torch.Tensor, target: torch.Tensor, ignore_index: int) -> torch.Tensor:
    """(mean loss, counted voxels) as a 2-float device tensor."""
    dev = _require_cuda(logits_cl, target)
    C = int(logits_cl.shape[1])
    vox = logits_cl.numel() // C
    L = lib()
    ws = torch.empty(int(L.r4c_ce_workspace_size(vox)), dtype=torch.uint8, device=dev)
    out = torch.empty(2, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = L.r4c_ce_fwd(_ptr(logits_cl), _ptr(target), vox, C, dtype_code(logits_cl.dtype), int(ignore_index),
                          _ptr(out), _ptr(ws), ws.numel(), _stream(dev))
    _check(st, "r4c_ce_fwd")
    return out


def ce_backward(logits_cl: torch.Tensor, target: torch.Tensor, ignore_index: int, loss_count: torch.Tensor,
                grad: torch.Tensor) -> torch.Tensor:
    """d(loss)/d(logits), NDHWC in the logits' dtype; ``grad`` a device scalar."""
    dev = _require_cuda(logits_cl, target)
    C = int(logits_cl.shape[1])
    vox = logits_cl.numel() // C
    g = grad.detach().to(torch.float32).reshape(1).contiguous()
    dz = torch.empty_like(logits_cl, memory_format=torch.channels_last_3d)
    with torch.cuda.device(dev):
        st = lib().r4c_ce_bwd(_ptr(logits_cl), _ptr(target), vox, C, dtype_code(logits_cl.dtype), int(ignore_index),
                              _ptr(loss_count), _ptr(g), _ptr(dz), _stream(dev))
    _check(st, "r4c_ce_bwd")
    return dz
