"""Implicit-GEMM Conv3d / ConvTranspose3d for NVIDIA B200 (sm_100a).

Drop-in for the reference package's module of the same name
(src/rdna4_conv3d/conv3d_wmma.py). The public surface is the same:
``Conv3dWmma``, ``ConvTranspose3dWmma``, ``swap_conv3d``, ``conv3d_wmma``,
``conv3d_plan``, ``wmma_fwd/dw/dx`` and ``wmma_ok_fwd/dw/dx``. The device work
goes through the C-ABI library ``libr4c_conv3d.so`` (tcgen05 + TMA kernels for
channel counts that are multiples of 8, SIMT CUDA kernels otherwise).

Layouts handed to the kernels:
  activations : NDHWC (channels_last_3d), bf16 / fp16
  weights     : PyTorch layout; the library packs them per leg
  dW / db     : fp32 from the kernels (deterministic split-K reduction)

Backend selection keeps the reference's environment variable:
  RDNA4_CONV3D_BACKEND = hybrid (default) | wmma | b200 | miopen | torch | hip
  (BIOHUB_CONV3D_BACKEND is read as an alias.) ``hybrid`` and ``hip`` run the
  B200 kernels on an sm_100 device; ``wmma`` and ``b200`` force them;
  ``miopen`` / ``torch`` force the stock PyTorch path. The value is read once
  at import, like the reference (conv3d_wmma.py:68-76).

Geometries outside k in {1,3}, stride 1, dilation 1, groups 1 fall back to
``F.conv3d`` exactly as the reference does; in-scope geometries on a CUDA
tensor never fall back: a missing or failing native library raises.
"""
from __future__ import annotations

import os
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native

_HALF = (torch.float16, torch.bfloat16)


# ---------------------------------------------------------------------------
# Device / backend selection (reference: conv3d_wmma.py:44-139)
# ---------------------------------------------------------------------------
def _is_rdna4() -> bool:
    """True on AMD gfx120x. Kept for API parity; never true on a B200 box."""
    if not torch.cuda.is_available():
        return False
    name = getattr(torch.cuda.get_device_properties(0), "gcnArchName", "") or ""
    return "gfx120" in name


def _is_b200() -> bool:
    """True when the current CUDA device is an sm_100 (B200-class) GPU."""
    if not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability() == (10, 0)


def _t3(v) -> Tuple[int, int, int]:
    if isinstance(v, int):
        return (v, v, v)
    return tuple(int(x) for x in v)


def _backend_name() -> str:
    """Backend requested through the environment ('hybrid' when unset)."""
    for var in ("RDNA4_CONV3D_BACKEND", "BIOHUB_CONV3D_BACKEND"):
        val = os.environ.get(var)
        if val:
            return val.lower()
    return "hybrid"


_BACKEND = _backend_name()


def _wmma_hw() -> bool:
    """Whether the tensor-core path is selected for this process."""
    if _BACKEND in ("miopen", "torch"):
        return False
    if _BACKEND in ("wmma", "b200"):
        return True
    return _is_b200()


def conv3d_backend() -> str:
    """Concrete backend behind the 'wmma' plan value: 'b200' or 'torch'."""
    return "b200" if _wmma_hw() else "torch"


def _geom_ok(kernel_size, stride, dilation, groups) -> bool:
    """k in {1,3} cubic, stride 1, dilation 1, groups 1 (reference :89-95)."""
    if int(groups) != 1:
        return False
    if _t3(stride) != (1, 1, 1) or _t3(dilation) != (1, 1, 1):
        return False
    return _t3(kernel_size) in ((1, 1, 1), (3, 3, 3))


def wmma_ok_fwd(cin, cout, kernel_size, stride=1, dilation=1, groups=1) -> bool:
    return _wmma_hw() and _geom_ok(kernel_size, stride, dilation, groups)


def wmma_ok_dw(cin, cout, kernel_size, stride=1, dilation=1, groups=1) -> bool:
    return wmma_ok_fwd(cin, cout, kernel_size, stride, dilation, groups)


def wmma_ok_dx(cin, cout, kernel_size, stride=1, dilation=1, groups=1) -> bool:
    """Every in-scope dX geometry (skinny Cin/Cout included) takes the kernels.

    The reference settled this end to end (conv3d_wmma.py:104-126): routing
    skinny dX legs to the vendor library looked cheaper in isolation and cost
    time and memory inside a real training step.
    """
    return wmma_ok_fwd(cin, cout, kernel_size, stride, dilation, groups)


def conv3d_plan(cin, cout, kernel_size, stride=1, dilation=1, groups=1) -> dict:
    """Which backend runs each leg: 'wmma' (tensor-core kernels) or 'miopen' (stock)."""
    legs = (("fwd", wmma_ok_fwd), ("dw", wmma_ok_dw), ("dx", wmma_ok_dx))
    return {leg: ("wmma" if ok(cin, cout, kernel_size, stride, dilation, groups) else "miopen")
            for leg, ok in legs}


def conv3d_kernels(x_shape, cout: int, kernel_size, padding=0, dtype=torch.bfloat16) -> dict:
    """Kernel family ('tcgen05' / 'simt') the library picks per leg for a shape."""
    n, cin, d, h, w = (int(v) for v in x_shape)
    k = _t3(kernel_size)[0]
    desc = _native.make_desc(n, d, h, w, cin, cout, k, _t3(padding), dtype)
    names = {_native.KERNEL_TC: "tcgen05", _native.KERNEL_GENERIC: "simt"}
    out = {}
    for leg, code in (("fwd", _native.LEG_FWD), ("dx", _native.LEG_DX), ("dw", _native.LEG_DW)):
        r = _native.plan_kernel(desc, code)
        out[leg] = names.get(r, f"error{r}")
    return out


# ---------------------------------------------------------------------------
# RDNA4 tile tables of the reference (conv3d_wmma.py:146-238). The B200
# kernels plan their own tiles inside the native library (r4c_plan_kernel);
# these pure functions stay importable with the reference's known answers
# because its CPU tests call them.
# ---------------------------------------------------------------------------
def _pick_bk(K: int) -> int:
    """BLOCK_K in {16, 32} with the least padded K; ties keep 16 below K=32."""
    padded = {bk: -(-K // bk) * bk for bk in (16, 32)}
    if padded[16] != padded[32]:
        return 16 if padded[16] < padded[32] else 32
    return 16 if K < 32 else 32


def _pick_tiles(M: int, N: int, K: int, kind: str = "fwd") -> Tuple[int, int, int, int, int]:
    """(BLOCK_M, BLOCK_N, BLOCK_K, num_warps, num_stages) of the RDNA4 kernels."""
    stages = 2
    if kind == "wgrad":
        bm = 16 if M <= 16 else (32 if M <= 32 else 64)
        bn = 16 if N < 32 else (32 if N < 64 else 64)
        bk, warps = (32, 8) if 16 < M <= 32 else (64, 4)
        return bm, bn, bk, warps, stages
    if N <= 32:
        bn = 16 if N <= 16 else 32
    elif N <= 48 and M < 65536:
        bn = 32
    else:
        bn = 64
    if M >= 65536:
        bm, warps = 128, 8
    elif M >= 64:
        bm, warps = 64, 4
    else:
        bm, warps = 32, 4
    return bm, bn, _pick_bk(K), warps, stages


def _split_k(M, N, K, bm, bn, bk, target_blocks=512) -> int:
    """Split-K factor of the reference's wgrad launch, clamped to [1, 32]."""
    tiles = max(1, (-(-M // bm)) * (-(-N // bn)))
    want = max(1, -(-target_blocks // tiles))
    cap = max(1, K // max(bk * 32, 1))
    return int(max(1, min(want, cap, 32)))


def _out_size(L, k, stride, pad, dil):
    return (L + 2 * pad - dil * (k - 1) - 1) // stride + 1


# ---------------------------------------------------------------------------
# Launch helpers
# ---------------------------------------------------------------------------
def _as_ndhwc(t: torch.Tensor) -> torch.Tensor:
    """channels_last_3d, contiguous and 16-byte aligned (TMA needs the alignment)."""
    if not t.is_contiguous(memory_format=torch.channels_last_3d):
        t = t.contiguous(memory_format=torch.channels_last_3d)
    if t.data_ptr() % 16 != 0:
        t = t.clone(memory_format=torch.channels_last_3d)
    return t


# Kernel family override for tests and benchmarks: 0 = let the library choose,
# 1 = SIMT kernels, 2 = tcgen05 kernels where they apply.
_FORCE_KERNEL = int(os.environ.get("R4C_FORCE_KERNEL", "0") or 0)


def _desc(x_shape, cout: int, k: int, padding, dtype: torch.dtype) -> _native.ConvDesc:
    n, cin, d, h, w = (int(v) for v in x_shape)
    return _native.make_desc(n, d, h, w, cin, int(cout), int(k), _t3(padding), dtype, _FORCE_KERNEL)


# ---------------------------------------------------------------------------
# Packed-weight cache. A packed weight is valid while the source weight is
# unchanged; the key holds (data_ptr, autograd version counter, optimizer
# generation). The version counter catches in-place writes made through
# autograd-visible ops (copy_, load_state_dict, non-fused optimizers); the
# generation, bumped by a global optimizer step hook, catches optimizers that
# write parameters without bumping it (fused Adam). Writes made through
# ``weight.data`` bypass both: call ``clear_packed_weight_cache()`` after them,
# or set R4C_PACK_CACHE=0.
# ---------------------------------------------------------------------------
_PACK_CACHE_ON = os.environ.get("R4C_PACK_CACHE", "1") != "0"
_OPT_GENERATION = [0]
_PACK_CACHE_MAX = 8          # packed layouts kept per weight tensor


def _bump_generation(*_args, **_kw):
    _OPT_GENERATION[0] += 1


try:
    from torch.optim.optimizer import register_optimizer_step_post_hook as _reg_hook
    _reg_hook(_bump_generation)
except ImportError:  # pragma: no cover - very old PyTorch: no hook, no cache
    _PACK_CACHE_ON = False


def clear_packed_weight_cache() -> None:
    """Invalidate every cached packed weight (after writes through ``.data``)."""
    _bump_generation()


def _packed_weight(desc: _native.ConvDesc, leg: int, weight: torch.Tensor) -> torch.Tensor:
    if not _PACK_CACHE_ON or torch.cuda.is_current_stream_capturing():
        return _native.pack_weight(desc, leg, weight)
    key = (leg, bytes(desc), weight.data_ptr(), weight._version, _OPT_GENERATION[0], weight.dtype)
    cache = getattr(weight, "_r4c_packed", None)
    if cache is not None:
        hit = cache.get(key)
        if hit is not None:
            return hit
        # entries of an older weight state are dead: keep only the current state's
        cache = {k: v for k, v in cache.items() if k[2:5] == key[2:5]}
    else:
        cache = {}
    wp = _native.pack_weight(desc, leg, weight)
    if len(cache) >= _PACK_CACHE_MAX:
        cache.pop(next(iter(cache)))
    cache[key] = wp
    try:
        weight._r4c_packed = cache
    except (AttributeError, RuntimeError):  # tensors that refuse attributes: no caching
        pass
    return wp


def _launch_fwd(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], padding,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y (NDHWC) = conv3d(x, weight) + bias on the B200 kernels. The weight
    may be fp32 (packing rounds it to x's dtype) or x's dtype. ``out``, when
    given, is a dense NDHWC buffer the result is written into."""
    k = int(weight.shape[2])
    cout = int(weight.shape[0])
    desc = _desc(x.shape, cout, k, padding, x.dtype)
    wp = _packed_weight(desc, _native.LEG_FWD, weight)
    pd, ph, pw = _t3(padding)
    osz = (_out_size(x.shape[2], k, 1, pd, 1), _out_size(x.shape[3], k, 1, ph, 1),
           _out_size(x.shape[4], k, 1, pw, 1))
    b = None if bias is None else bias.to(x.dtype).contiguous()
    return _native.conv_fwd(desc, _as_ndhwc(x), wp, b, osz, out)


def _launch_dgrad(go: torch.Tensor, weight: torch.Tensor, x_shape, padding,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dX (NDHWC) of a stride-1 conv: conv of dY with the flipped weight, pad k-1-p."""
    k = int(weight.shape[2])
    desc = _desc(x_shape, int(weight.shape[0]), k, padding, go.dtype)
    wp = _packed_weight(desc, _native.LEG_DX, weight)
    return _native.conv_dx(desc, _as_ndhwc(go), wp, out)


def _launch_wgrad(x: torch.Tensor, go: torch.Tensor, weight_shape, padding, want_db: bool):
    """(dW fp32 OIDHW, db fp32 or None)."""
    k = int(weight_shape[2])
    desc = _desc(x.shape, int(weight_shape[0]), k, padding, x.dtype)
    return _native.conv_dw(desc, _as_ndhwc(x), _as_ndhwc(go), want_db)


# Optional gradient reducer (data parallel): set by rdna4_conv3d.distributed.
# backward() hands it the fp32 dW/db right after they are computed and waits
# for the reduction only after dX has been launched.
_GRAD_REDUCER = None


def _reduce_async(tensors):
    red = _GRAD_REDUCER
    if red is None:
        return None
    return red.reduce_async([t for t in tensors if t is not None])


# ---------------------------------------------------------------------------
# Autograd + nn.Conv3d drop-in (reference: conv3d_wmma.py:1233-1319)
# ---------------------------------------------------------------------------
class Conv3dWmmaFn(torch.autograd.Function):
    """Conv3d with B200 kernels for fwd, dX and dW. Tensors are saved in
    setup_context (required for AMP on recent PyTorch)."""

    @staticmethod
    def forward(x, weight, bias, stride, padding, dilation):
        cin, cout = int(x.shape[1]), int(weight.shape[0])
        ks = tuple(int(s) for s in weight.shape[2:])
        if not wmma_ok_fwd(cin, cout, ks, stride, dilation, 1):
            w_c = weight if weight.dtype == x.dtype else weight.to(x.dtype)
            b_c = bias if bias is None or bias.dtype == x.dtype else bias.to(x.dtype)
            return F.conv3d(x, w_c, b_c, stride, padding, dilation)
        compute_dtype = x.dtype
        xc = x if compute_dtype in _HALF else x.to(torch.float16)
        y = _launch_fwd(xc, weight, bias, padding)
        if not x.is_contiguous(memory_format=torch.channels_last_3d):
            y = y.contiguous()
        if compute_dtype not in _HALF:
            y = y.to(compute_dtype)
        return y

    @staticmethod
    def setup_context(ctx, inputs, output):
        x, weight, bias, stride, padding, dilation = inputs
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        ctx.bias_dtype = None if bias is None else bias.dtype
        ctx.stride, ctx.padding, ctx.dilation = stride, padding, dilation
        ctx.kernel_size = tuple(int(s) for s in weight.shape[2:])
        ctx.x_layout = (torch.channels_last_3d if x.is_contiguous(memory_format=torch.channels_last_3d)
                        else torch.contiguous_format)

    @staticmethod
    def backward(ctx, grad_out):
        x, weight = ctx.saved_tensors
        stride, padding, dilation, ks = ctx.stride, ctx.padding, ctx.dilation, ctx.kernel_size
        cin, cout = int(x.shape[1]), int(weight.shape[0])
        go = grad_out if grad_out.dtype in _HALF else grad_out.to(torch.float16)
        x_c = x if x.dtype in _HALF else x.to(torch.float16)
        if go.dtype != x_c.dtype:
            go = go.to(x_c.dtype)
        if x.is_cuda and wmma_ok_dw(cin, cout, ks, stride, dilation, 1):
            go = _as_ndhwc(go)        # one dense NDHWC copy for both kernel legs
        need_x, need_w, need_b = ctx.needs_input_grad[:3]
        want_db = ctx.has_bias and need_b
        dx_leg = need_x and wmma_ok_dx(cin, cout, ks, stride, dilation, 1)
        dw_leg = need_w and wmma_ok_dw(cin, cout, ks, stride, dilation, 1)

        # dW and db first, so a data-parallel reduction overlaps the dX kernel.
        dw = db = None
        if need_w:
            if dw_leg:
                dw, db = _launch_wgrad(x_c, go, weight.shape, padding, want_db)
            else:
                w_c = weight if weight.dtype in _HALF else weight.to(x_c.dtype)
                dw = torch.nn.grad.conv3d_weight(x_c, weight.shape, go.contiguous(), stride, padding,
                                                 dilation, 1).float()
                del w_c
        if want_db and db is None:
            db = go.float().sum(dim=(0, 2, 3, 4))
        handle = _reduce_async([dw, db])

        gx = None
        if need_x:
            if dx_leg:
                gx = _launch_dgrad(go, weight, x.shape, padding)
            else:
                w_c = weight.to(go.dtype)
                gx = torch.nn.grad.conv3d_input(x.shape, w_c, go.contiguous(), stride, padding, dilation, 1)
            if gx.dtype != x.dtype:
                gx = gx.to(x.dtype)
            if ctx.x_layout == torch.contiguous_format:
                gx = gx.contiguous()
        if handle is not None:
            handle.wait()
        if dw is not None and dw.dtype != weight.dtype:
            dw = dw.to(weight.dtype)
        if db is not None and ctx.bias_dtype is not None and db.dtype != ctx.bias_dtype:
            db = db.to(ctx.bias_dtype)
        return gx, dw, db, None, None, None


def _autocast_dtype():
    """Half dtype autocast would run a CUDA conv in, or None when autocast is off.

    Custom Functions bypass autocast (it hooks ATen ops), so the cast is done
    here, outside the Function, exactly where autocast would put it: the
    output then stays in the autocast dtype and dW flows back to fp32 master
    weights through the cast (reference conv3d_wmma.py:1322-1358).
    """
    try:
        if not torch.is_autocast_enabled("cuda"):
            return None
        dt = torch.get_autocast_dtype("cuda")
    except TypeError:  # older PyTorch without the device argument
        if not torch.is_autocast_enabled():
            return None
        dt = torch.get_autocast_gpu_dtype()
    return dt if dt in _HALF else None


def _autocast_args(x, weight, bias):
    """Cast the activation to the autocast dtype here, outside the Function,
    so the output comes out in that dtype as autocast would make it.

    The weight and bias go in uncast: packing rounds the weight to the
    compute dtype (the same values ``weight.to(dt)`` would hold) and dW / db
    come back in fp32 straight into the fp32 master parameters, without the
    half-precision rounding that a cast's backward would add (the reference
    rounds dW to the compute dtype, conv3d_wmma.py:1213-1214; keeping fp32 is
    the more accurate side of the same result).
    """
    dt = _autocast_dtype()
    if dt is None or not x.is_cuda:
        return x, weight, bias
    return (x if x.dtype == dt else x.to(dt)), weight, bias


def conv3d_wmma(x, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
    """Functional Conv3d; same arguments as F.conv3d (integer/tuple padding)."""
    if x.is_cuda and _wmma_hw() and not isinstance(padding, str):
        cin, cout = int(x.shape[1]), int(weight.shape[0])
        if _k2s2_ok(x, cin, cout, weight.shape[2:], stride, padding, dilation, groups) or (
                _GENERAL and not _geom_ok(tuple(weight.shape[2:]), stride, dilation, groups)):
            return conv3d_general(x, weight, bias, stride, padding, dilation, groups)
    if groups != 1:
        return F.conv3d(x, weight, bias, stride, padding, dilation, groups)
    x, weight, bias = _autocast_args(x, weight, bias)
    return Conv3dWmmaFn.apply(x, weight, bias, _t3(stride), _t3(padding), _t3(dilation))


def _check_isolated(weight, stride, dilation):
    ks = tuple(int(s) for s in weight.shape[2:])
    if not _geom_ok(ks, stride, dilation, 1):
        raise ValueError(f"geometry outside the kernel scope: k={ks} stride={stride} dilation={dilation}")


def wmma_fwd(x, weight, bias=None, stride=1, padding=0, dilation=1):
    """Isolated forward leg (no autograd). NCDHW out unless x is channels_last_3d."""
    st, pd, dl = _t3(stride), _t3(padding), _t3(dilation)
    _check_isolated(weight, st, dl)
    y = _launch_fwd(x, weight, bias, pd)
    if x.is_contiguous(memory_format=torch.channels_last_3d):
        return y
    return y.contiguous()


def wmma_dw(x, weight, go, stride=1, padding=0, dilation=1):
    """Isolated weight gradient, OIDHW like nn.Conv3d.weight.grad, in go's dtype."""
    st, pd, dl = _t3(stride), _t3(padding), _t3(dilation)
    _check_isolated(weight, st, dl)
    dw, _ = _launch_wgrad(x, go.to(x.dtype), weight.shape, pd, False)
    return dw.to(go.dtype)


def wmma_dx(x, weight, go, stride=1, padding=0, dilation=1):
    """Isolated input gradient; NCDHW out unless x is channels_last_3d."""
    st, pd, dl = _t3(stride), _t3(padding), _t3(dilation)
    ks = tuple(int(s) for s in weight.shape[2:])
    cin, cout = int(x.shape[1]), int(weight.shape[0])
    cl = x.is_contiguous(memory_format=torch.channels_last_3d)
    if not wmma_ok_dx(cin, cout, ks, st, dl, 1):
        w = weight if weight.dtype == go.dtype else weight.to(go.dtype)
        gx = torch.nn.grad.conv3d_input(x.shape, w, go.contiguous(), st, pd, dl, 1)
        return gx.contiguous(memory_format=torch.channels_last_3d) if cl else gx.contiguous()
    gx = _launch_dgrad(go, weight, x.shape, pd)
    return gx if cl else gx.contiguous()


# ---------------------------------------------------------------------------
# Any other geometry (per-axis kernel size, stride, padding, dilation,
# groups): the r4c_convex_* entry points. k=2 stride-2 pad-0 convs with
# channels that are multiples of 8 run on the tcgen05 transpose-conv kernels
# (the downsampling conv is the transpose of the k2s2 up-conv); the rest on
# SIMT kernels. The reference sends all of these to the vendor library
# (conv3d_wmma.py:1241-1242), and so does Conv3dWmma by default, except the
# k2s2 form; RDNA4_CONV3D_GENERAL=1 routes the rest here too.
# ---------------------------------------------------------------------------
_GENERAL = os.environ.get("RDNA4_CONV3D_GENERAL", "0").lower() in ("1", "simt", "on", "true")


def _k2s2_ok(x, cin, cout, kernel_size, stride, padding, dilation, groups) -> bool:
    """k=2, stride 2, pad 0 conv on the tcgen05 transpose-conv kernels (bf16 /
    fp16 activations, or autocast on; fp32 stays with the vendor library)."""
    if x.dtype not in _HALF and _autocast_dtype() is None:
        return False
    x_shape = x.shape
    if _t3(kernel_size) != (2, 2, 2) or _t3(stride) != (2, 2, 2) or _t3(padding) != (0, 0, 0):
        return False
    if _t3(dilation) != (1, 1, 1) or int(groups) != 1 or cin % 8 or cout % 8:
        return False
    return all(int(v) % 2 == 0 for v in x_shape[2:])


def _convex_desc(x_shape, w_shape, stride, padding, dilation, groups, dtype):
    return _native.make_convex_desc(x_shape, w_shape, _t3(stride), _t3(padding), _t3(dilation), groups, dtype)


class Conv3dGeneralFn(torch.autograd.Function):
    """Conv3d of any geometry on the r4c_convex_* kernels. Computes in x's
    dtype (bf16 / fp16 / fp32); dW and db in fp32."""

    @staticmethod
    def forward(x, weight, bias, stride, padding, dilation, groups):
        xc = _as_ndhwc(x)
        w = weight.to(x.dtype).contiguous()
        b = None if bias is None else bias.to(x.dtype).contiguous()
        desc = _convex_desc(x.shape, weight.shape, stride, padding, dilation, groups, x.dtype)
        y = _native.convex_fwd(desc, xc, w, b)
        if not x.is_contiguous(memory_format=torch.channels_last_3d):
            y = y.contiguous()
        return y

    @staticmethod
    def setup_context(ctx, inputs, output):
        x, weight, bias, stride, padding, dilation, groups = inputs
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        ctx.bias_dtype = None if bias is None else bias.dtype
        ctx.geom = (stride, padding, dilation, groups)
        ctx.x_layout = (torch.channels_last_3d if x.is_contiguous(memory_format=torch.channels_last_3d)
                        else torch.contiguous_format)

    @staticmethod
    def backward(ctx, grad_out):
        x, weight = ctx.saved_tensors
        stride, padding, dilation, groups = ctx.geom
        go = _as_ndhwc(grad_out.to(x.dtype))
        desc = _convex_desc(x.shape, weight.shape, stride, padding, dilation, groups, x.dtype)
        need_x, need_w, need_b = ctx.needs_input_grad[:3]
        dw = db = None
        if need_w or (need_b and ctx.has_bias):
            dw, db = _native.convex_dw(desc, _as_ndhwc(x), go, bool(ctx.has_bias and need_b))
        handle = _reduce_async([dw, db])
        gx = None
        if need_x:
            gx = _native.convex_dx(desc, go, weight.to(x.dtype).contiguous())
            if ctx.x_layout == torch.contiguous_format:
                gx = gx.contiguous()
        if handle is not None:
            handle.wait()
        if dw is not None:
            dw = dw.to(weight.dtype) if need_w else None
        if db is not None and ctx.bias_dtype is not None:
            db = db.to(ctx.bias_dtype)
        return gx, dw, db, None, None, None, None


def conv3d_general(x, weight, bias=None, stride=1, padding=0, dilation=1, groups=1):
    """Conv3d of any geometry (integer or per-axis stride / padding /
    dilation, groups) on this library's kernels, CUDA tensors only. Under
    autocast the activation and weight are cast to the autocast dtype here,
    outside the Function, as for conv3d_wmma."""
    if not x.is_cuda:
        raise ValueError("conv3d_general runs on CUDA tensors")
    dt = _autocast_dtype()
    if dt is not None and x.dtype != dt:
        x = x.to(dt)
    return Conv3dGeneralFn.apply(x, weight, bias, _t3(stride), _t3(padding), _t3(dilation), int(groups))


def swap_conv3d(module: nn.Module) -> int:
    """Replace every plain ``nn.Conv3d`` under ``module`` with ``Conv3dWmma``.

    Weights and bias are copied; the new module keeps the old one's device,
    dtype and padding_mode (the reference built it on the default device,
    conv3d_wmma.py:1412-1430). Returns how many modules were swapped.
    """
    count = 0
    for name, child in list(module.named_children()):
        if type(child) is nn.Conv3d:
            new = Conv3dWmma(
                child.in_channels, child.out_channels, child.kernel_size,
                stride=child.stride, padding=child.padding, dilation=child.dilation,
                groups=child.groups, bias=child.bias is not None, padding_mode=child.padding_mode,
                device=child.weight.device, dtype=child.weight.dtype,
            )
            with torch.no_grad():
                new.weight.copy_(child.weight)
                if child.bias is not None:
                    new.bias.copy_(child.bias)
            new.train(child.training)
            setattr(module, name, new)
            count += 1
        else:
            count += swap_conv3d(child)
    return count


class Conv3dWmma(nn.Conv3d):
    """Drop-in ``nn.Conv3d``: B200 kernels for in-scope geometry on CUDA tensors."""

    def forward(self, x):
        if not x.is_cuda or self.padding_mode != "zeros" or isinstance(self.padding, str):
            return super().forward(x)
        cin, cout = int(x.shape[1]), int(self.weight.shape[0])
        if _wmma_hw() and (_k2s2_ok(x, cin, cout, self.kernel_size, self.stride, self.padding,
                                    self.dilation, self.groups)
                           or (_GENERAL and not _geom_ok(self.kernel_size, self.stride, self.dilation, self.groups))):
            return conv3d_general(x, self.weight, self.bias, self.stride, self.padding, self.dilation, self.groups)
        if self.groups != 1:
            return super().forward(x)
        plan = conv3d_plan(cin, cout, self.kernel_size, self.stride, self.dilation, self.groups)
        if all(v == "miopen" for v in plan.values()):
            return super().forward(x)
        return conv3d_wmma(x, self.weight, self.bias, self.stride, self.padding, self.dilation, 1)


# ---------------------------------------------------------------------------
# ConvTranspose3d k=2 s=2 p=0 (reference: conv3d_wmma.py:1446-1595)
# ---------------------------------------------------------------------------
def _tdesc(x_shape, cout: int, dtype) -> _native.ConvDesc:
    n, cin, d, h, w = (int(v) for v in x_shape)
    return _native.make_desc(n, d, h, w, cin, int(cout), 2, (0, 0, 0), dtype, _FORCE_KERNEL)


def transpose_k2s2_fwd(x, weight, bias=None):
    """weight in PyTorch ConvTranspose3d layout (Cin, Cout, 2, 2, 2); NDHWC out."""
    desc = _tdesc(x.shape, int(weight.shape[1]), x.dtype)
    wp = _packed_weight(desc, _native.LEG_TFWD, weight)
    b = None if bias is None else bias.to(x.dtype).contiguous()
    return _native.tconv_fwd(desc, _as_ndhwc(x), wp, b)


def transpose_k2s2_dx(x_shape, weight, go):
    desc = _tdesc(x_shape, int(weight.shape[1]), go.dtype)
    wp = _packed_weight(desc, _native.LEG_TDX, weight)
    return _native.tconv_dx(desc, _as_ndhwc(go), wp)


def transpose_k2s2_dw(x, weight_shape, go, want_db: bool = False):
    """(dW fp32 (Cin, Cout, 2, 2, 2), db fp32 or None)."""
    desc = _tdesc(x.shape, int(weight_shape[1]), x.dtype)
    return _native.tconv_dw(desc, _as_ndhwc(x), _as_ndhwc(go.to(x.dtype)), want_db)


class ConvTranspose3dWmmaFn(torch.autograd.Function):
    @staticmethod
    def forward(x, weight, bias):
        compute_dtype = x.dtype
        xc = x if compute_dtype in _HALF else x.to(torch.float16)
        y = transpose_k2s2_fwd(xc, weight, bias)
        if not x.is_contiguous(memory_format=torch.channels_last_3d):
            y = y.contiguous()
        if compute_dtype not in _HALF:
            y = y.to(compute_dtype)
        return y

    @staticmethod
    def setup_context(ctx, inputs, output):
        x, weight, bias = inputs
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        ctx.bias_dtype = None if bias is None else bias.dtype
        ctx.x_layout = (torch.channels_last_3d if x.is_contiguous(memory_format=torch.channels_last_3d)
                        else torch.contiguous_format)

    @staticmethod
    def backward(ctx, grad_out):
        return _tconv_backward(ctx, grad_out)


def _tconv_backward(ctx, grad_out):
    """(dX, dW, db) of the k2s2 transpose conv saved in ctx (x, weight)."""
    x, weight = ctx.saved_tensors
    need_x, need_w, need_b = ctx.needs_input_grad[:3]
    x_c = x if x.dtype in _HALF else x.to(torch.float16)
    go = grad_out.to(x_c.dtype) if grad_out.dtype != x_c.dtype else grad_out
    # one dense NDHWC copy shared by both legs when dY arrives as a view
    # (e.g. the channel slice of a concatenation's gradient: the library's
    # slice copy, else PyTorch's)
    if not go.is_contiguous(memory_format=torch.channels_last_3d):
        dense = _native.channel_slice_dense(go)
        if dense is not None:
            go = dense
    go = _as_ndhwc(go)
    want_db = ctx.has_bias and need_b
    dw = db = None
    if need_w:
        dw, db = transpose_k2s2_dw(x_c, weight.shape, go, want_db)
    if want_db and db is None:
        db = go.float().sum(dim=(0, 2, 3, 4))
    handle = _reduce_async([dw, db])
    gx = None
    if need_x:
        gx = transpose_k2s2_dx(x.shape, weight, go)
        if gx.dtype != x.dtype:
            gx = gx.to(x.dtype)
        if ctx.x_layout == torch.contiguous_format:
            gx = gx.contiguous()
    if handle is not None:
        handle.wait()
    if dw is not None and dw.dtype != weight.dtype:
        dw = dw.to(weight.dtype)
    if db is not None and ctx.bias_dtype is not None and db.dtype != ctx.bias_dtype:
        db = db.to(ctx.bias_dtype)
    return gx, dw, db


class UpConcatFn(torch.autograd.Function):
    """ConvTranspose3d k2s2 of x written straight into channels [0, lead) of
    ``buf``, whose channels [lead, ...) already hold the skip connection:
    torch.cat([up(x), skip], 1) of a UNet decoder (the reference's UNet,
    benches/unet_e2e.py:38) without materialising up(x) and copying it. The
    gradient of buf's first ``lead`` channels drives the transpose conv's
    backward; buf's gradient passes on whole (its skip part)."""

    @staticmethod
    def forward(ctx, x, weight, bias, buf, lead):
        desc = _tdesc(x.shape, int(weight.shape[1]), x.dtype)
        wp = _packed_weight(desc, _native.LEG_TFWD, weight)
        b = None if bias is None else bias.to(x.dtype).contiguous()
        _native.tconv_fwd_into(desc, _as_ndhwc(x), wp, b, buf)
        ctx.mark_dirty(buf)
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        ctx.bias_dtype = None if bias is None else bias.dtype
        ctx.x_layout = (torch.channels_last_3d if x.is_contiguous(memory_format=torch.channels_last_3d)
                        else torch.contiguous_format)
        ctx.lead = int(lead)
        return buf

    @staticmethod
    def backward(ctx, g):
        gx, dw, db = _tconv_backward(ctx, g[:, :ctx.lead])
        return gx, dw, db, g, None


class ConvTranspose3dWmma(nn.ConvTranspose3d):
    """k=2 s=2 p=0 drop-in; every other configuration uses nn.ConvTranspose3d."""

    def forward(self, x, output_size=None):
        in_scope = (
            self.kernel_size == (2, 2, 2) and self.stride == (2, 2, 2) and self.padding == (0, 0, 0)
            and self.output_padding == (0, 0, 0) and self.dilation == (1, 1, 1) and self.groups == 1
            and self.padding_mode == "zeros" and x.is_cuda and x.dim() == 5 and _wmma_hw()
        )
        if in_scope and output_size is not None:
            want = tuple(int(s) for s in list(output_size)[-3:])
            in_scope = want == tuple(2 * int(s) for s in x.shape[2:])
        if not in_scope:
            return super().forward(x, output_size)
        x, weight, bias = _autocast_args(x, self.weight, self.bias)
        return ConvTranspose3dWmmaFn.apply(x, weight, bias)

    def forward_into(self, x, buf, lead: int):
        """``buf`` with self(x) written into its channels [0, lead): the
        decoder concatenation torch.cat([self(x), buf[:, lead:]], 1) built in
        place. On the native path the transpose conv stores into buf directly
        (r4c_tconv_fwd_pitched); otherwise self(x) is copied there."""
        direct = (
            self.kernel_size == (2, 2, 2) and self.stride == (2, 2, 2) and self.padding == (0, 0, 0)
            and self.output_padding == (0, 0, 0) and self.dilation == (1, 1, 1) and self.groups == 1
            and self.padding_mode == "zeros" and x.is_cuda and x.dim() == 5 and _wmma_hw()
            and int(lead) == self.out_channels and buf.dim() == 5 and buf.shape[1] % 8 == 0
            and self.out_channels % 8 == 0 and self.in_channels % 8 == 0
            and tuple(buf.shape[2:]) == tuple(2 * int(v) for v in x.shape[2:])
            and buf.is_contiguous(memory_format=torch.channels_last_3d) and buf.data_ptr() % 16 == 0
        )
        if direct:
            xa, weight, bias = _autocast_args(x, self.weight, self.bias)
            direct = (xa.dtype in _HALF and buf.dtype == xa.dtype and _native.plan_kernel(
                _tdesc(xa.shape, self.out_channels, xa.dtype), _native.LEG_TFWD) == _native.KERNEL_TC)
        if not direct:
            from .bn_relu import skip_cat
            return skip_cat(self(x), buf, lead)
        return UpConcatFn.apply(xa, weight, bias, buf, int(lead))
