"""Fused BatchNorm3d + ReLU kernels (r4c_bn_*) on a B200.

Against stock BatchNorm3d + ReLU in fp32 on the same bf16/fp16-rounded
NDHWC activations: forward output (max-rel 2e-2, the output is rounded to
the activation dtype), running statistics, and the gradients dX (max-rel
2e-2), dgamma and dbeta (norm-rel 3e-2). The statistics are fp32 sums, so
they match far inside that.
"""
import pytest
import torch
import torch.nn.functional as F

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("relu", [True, False], ids=["relu", "bn"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(4, 24, 16, 32, 32), (2, 48, 8, 16, 16), (1, 192, 4, 8, 8), (3, 8, 5, 7, 9),
                                   (4, 24, 64, 128, 128)], ids=lambda s: "x".join(map(str, s)))
def test_bn_relu_matches_stock(cuda_ready, shape, dtype, relu):
    from rdna4_conv3d import _native
    from rdna4_conv3d.bn_relu import BatchNormReLU3d
    C = shape[1]
    g = torch.Generator().manual_seed(C)
    x = (torch.randn(shape, generator=g) * 2.0 + 3.0).to(dtype)        # |mean| > std: tests the pivot
    gy = torch.randn(shape, generator=g).to(dtype)
    ref = torch.nn.BatchNorm3d(C)
    with torch.no_grad():
        ref.weight.copy_(torch.rand(C, generator=g) + 0.5)
        ref.bias.copy_(torch.randn(C, generator=g) * 0.1)
    mod = BatchNormReLU3d(C, relu=relu).cuda()
    mod.load_state_dict(ref.state_dict())
    xg = x.cuda().contiguous(memory_format=torch.channels_last_3d).requires_grad_(True)
    n0 = _native.launch_count()
    y = mod(xg)
    y.backward(gy.cuda().contiguous(memory_format=torch.channels_last_3d))
    torch.cuda.synchronize()
    assert _native.launch_count() - n0 >= 6          # stats, finalize, apply, bwd sums, finalize, dX
    assert y.dtype == dtype and y.is_contiguous(memory_format=torch.channels_last_3d)

    xr = x.float().requires_grad_(True)
    yr = ref(xr)
    if relu:
        yr = F.relu(yr)
    yr.backward(gy.float())
    assert O.max_rel(y.float().cpu(), yr) <= 2e-2
    assert O.max_rel(xg.grad.float().cpu(), xr.grad) <= 2e-2
    assert O.norm_rel(mod.weight.grad.cpu(), ref.weight.grad) <= 3e-2
    assert O.norm_rel(mod.bias.grad.cpu(), ref.bias.grad) <= 3e-2
    # fp32 sums of the same inputs: far inside the stated bound
    assert O.norm_rel(mod.weight.grad.cpu(), ref.weight.grad) <= 1e-3
    assert O.norm_rel(mod.bias.grad.cpu(), ref.bias.grad) <= 1e-3
    torch.testing.assert_close(mod.running_mean.cpu(), ref.running_mean, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(mod.running_var.cpu(), ref.running_var, rtol=1e-4, atol=1e-5)
    assert int(mod.num_batches_tracked) == 1


def test_bn_relu_deterministic(cuda_ready):
    from rdna4_conv3d.bn_relu import BatchNormReLU3d
    mod = BatchNormReLU3d(48).cuda()
    x = torch.randn(2, 48, 8, 16, 16, device="cuda", dtype=torch.bfloat16).contiguous(
        memory_format=torch.channels_last_3d).requires_grad_(True)
    gy = torch.randn_like(x)
    outs = []
    for _ in range(2):
        x.grad = None
        mod.weight.grad = None
        y = mod(x)
        y.backward(gy)
        outs.append((y.detach().clone(), x.grad.clone(), mod.weight.grad.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_bn_relu_eval_and_fallbacks(cuda_ready):
    """Eval mode (running statistics) and NCDHW inputs take the stock path."""
    from rdna4_conv3d import _native
    from rdna4_conv3d.bn_relu import BatchNormReLU3d
    mod = BatchNormReLU3d(16).cuda()
    ref = torch.nn.BatchNorm3d(16).cuda()
    x = torch.randn(2, 16, 4, 6, 8, device="cuda", dtype=torch.bfloat16)
    mod.eval()
    ref.eval()
    n0 = _native.launch_count()
    torch.testing.assert_close(mod(x.contiguous(memory_format=torch.channels_last_3d)), F.relu(ref(x)))
    mod.train()
    ref.train()
    torch.testing.assert_close(mod(x), F.relu(ref(x)))           # NCDHW: stock
    assert _native.launch_count() == n0


_POOL_SHAPES = [((2, 24, 8, 16, 16), 24), ((1, 48, 4, 8, 8), 48), ((2, 8, 6, 4, 10), 0), ((4, 24, 64, 128, 128), 24)]


# ties: quantised inputs. The wide case (C/4 = 132 > 128 threads: a thread's
# channel group changes between steps) runs on random inputs only: with 32
# voxels per channel its quantised batch mean lands exactly on input values
# (27 of the 528 channels),
# and whether BatchNorm's output there is 0 or a rounding residue (which
# decides ReLU's gradient) depends on how each implementation sums the mean.
@pytest.mark.parametrize("shape,lead,quantised",
                         [(s, l, q) for s, l in _POOL_SHAPES for q in (False, True)] + [((1, 528, 2, 4, 4), 8, False)],
                         ids=[f"{i}-{q}" for i in ("24", "48", "lead0", "full") for q in ("random", "ties")] + ["wide-random"])
def test_bn_relu_pool_and_skip_buffer(cuda_ready, shape, lead, quantised):
    """forward_pool (BN + ReLU + MaxPool3d(2), skip written after `lead`
    channels of the concatenation buffer) and skip_cat against stock
    BatchNorm3d + ReLU + max_pool3d + cat, values and gradients. Quantised
    inputs put ties into the pooling windows: the argmax must follow
    max_pool3d's first-maximum rule for the gradients to agree."""
    from rdna4_conv3d.bn_relu import BatchNormReLU3d, skip_cat
    C = shape[1]
    g = torch.Generator().manual_seed(C + lead)
    x = torch.randn(shape, generator=g) * 2.0 + 0.3
    if quantised:
        x = torch.round(x * 2) / 2
    x = x.to(torch.bfloat16)
    up = torch.randn((shape[0], lead) + shape[2:], generator=g).to(torch.bfloat16)
    gcat = torch.randn((shape[0], lead + C) + shape[2:], generator=g).to(torch.bfloat16)
    gp = torch.randn((shape[0], C) + tuple(s // 2 for s in shape[2:]), generator=g).to(torch.bfloat16)
    ref = torch.nn.BatchNorm3d(C)
    mod = BatchNormReLU3d(C).cuda()
    mod.load_state_dict(ref.state_dict())
    cl = torch.channels_last_3d
    xg = x.cuda().contiguous(memory_format=cl).requires_grad_(True)
    upg = up.cuda().contiguous(memory_format=cl).requires_grad_(True)
    buf, p = mod.forward_pool(xg, lead)
    cat = skip_cat(upg, buf, lead)
    torch.autograd.backward([cat, p], [gcat.cuda().contiguous(memory_format=cl), gp.cuda().contiguous(memory_format=cl)])
    torch.cuda.synchronize()

    # the stock path on the GPU in bf16 (same rounding points as the model's stock run)
    refg = ref.cuda()
    xr = x.cuda().contiguous(memory_format=cl).requires_grad_(True)
    upr = up.cuda().contiguous(memory_format=cl).requires_grad_(True)
    yr = F.relu(refg(xr))
    pr = F.max_pool3d(yr, 2)
    catr = torch.cat([upr, yr], dim=1)
    torch.autograd.backward([catr, pr], [gcat.cuda(), gp.cuda()])
    assert p.shape == pr.shape and cat.shape == catr.shape
    assert O.max_rel(cat.float().cpu(), catr.float().cpu()) <= 2e-2
    assert O.max_rel(p.float().cpu(), pr.float().cpu()) <= 2e-2
    assert O.max_rel(xg.grad.float().cpu(), xr.grad.float().cpu()) <= 2e-2
    if lead:
        assert torch.equal(upg.grad.cpu(), upr.grad.cpu())
    # the stock path rounds the sum of the skip and pool gradients to bf16
    # before BatchNorm's backward; the fused kernels add them in fp32
    assert O.norm_rel(mod.weight.grad.cpu(), refg.weight.grad.cpu()) <= 3e-2
    assert O.norm_rel(mod.bias.grad.cpu(), refg.bias.grad.cpu()) <= 3e-2
    torch.testing.assert_close(mod.running_mean, refg.running_mean, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("amp", [False, True], ids=["bf16", "autocast-fp32-in"])
@pytest.mark.parametrize("cin,cout,pitch", [(48, 24, 48), (96, 48, 96), (64, 32, 96)])
def test_up_conv_writes_into_concat_buffer(cuda_ready, cin, cout, pitch, amp, monkeypatch):
    """ConvTranspose3dWmma.forward_into: the up-conv stores straight into the
    first channels of the decoder's concatenation buffer (pitched output);
    forward and every gradient equal the up-conv-then-copy path bit for bit."""
    import sys
    from rdna4_conv3d import ConvTranspose3dWmma
    from rdna4_conv3d.bn_relu import skip_cat
    cw = sys.modules["rdna4_conv3d.conv3d_wmma"]
    calls = []
    orig = cw.UpConcatFn.apply
    monkeypatch.setattr(cw.UpConcatFn, "apply", lambda *a: calls.append(1) or orig(*a))
    torch.manual_seed(0)
    up = ConvTranspose3dWmma(cin, cout, 2, stride=2).cuda()
    cl = torch.channels_last_3d
    x0 = torch.randn(2, cin, 4, 6, 8, device="cuda")
    skip = torch.randn(2, pitch - cout, 8, 12, 16, device="cuda").to(torch.bfloat16)
    g = torch.randn(2, pitch, 8, 12, 16, device="cuda").to(torch.bfloat16).contiguous(memory_format=cl)
    outs = []
    for direct in (True, False):
        up.zero_grad(set_to_none=True)
        x = (x0 if amp else x0.to(torch.bfloat16)).contiguous(memory_format=cl).requires_grad_(True)
        s = skip.clone().requires_grad_(True)
        head = torch.zeros(2, cout, 8, 12, 16, device="cuda", dtype=torch.bfloat16)
        buf = torch.cat([head, s], 1).contiguous(memory_format=cl)  # skip channels from a graph input
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
            y = up.forward_into(x, buf, cout) if direct else skip_cat(up(x), buf, cout)
        y.backward(g)
        outs.append((y.detach().clone(), x.grad.clone(), up.weight.grad.clone(), up.bias.grad.clone(), s.grad.clone()))
    assert len(calls) == 1                                  # the direct path ran once (first pass)
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    assert torch.equal(outs[0][0][:, cout:], skip)          # the skip channels are untouched



@pytest.mark.parametrize("cin,cout,shape,direct", [
    (128, 64, (4, 16, 32, 32), True),    # tcgen05 plan with per-thread stores
    (832, 16, (1, 2, 4, 4), False),      # 13 K boxes: no tcgen05 plan
], ids=["128x64", "832x16"])
def test_up_conv_into_buffer_plans(cuda_ready, monkeypatch, cin, cout, shape, direct):
    """The up-conv writes into the buffer when the transpose conv has a
    tcgen05 plan and falls back to up-conv-then-copy otherwise; either way
    the result equals the copy path."""
    import sys
    from rdna4_conv3d import ConvTranspose3dWmma
    from rdna4_conv3d.bn_relu import skip_cat
    cw = sys.modules["rdna4_conv3d.conv3d_wmma"]
    calls = []
    orig = cw.UpConcatFn.apply
    monkeypatch.setattr(cw.UpConcatFn, "apply", lambda *a: calls.append(1) or orig(*a))
    torch.manual_seed(0)
    up = ConvTranspose3dWmma(cin, cout, 2, stride=2).cuda()
    cl = torch.channels_last_3d
    n, d, h, w = shape
    x = torch.randn(n, cin, d, h, w, device="cuda").to(torch.bfloat16).contiguous(memory_format=cl)
    buf = torch.randn(n, 2 * cout, 2 * d, 2 * h, 2 * w, device="cuda").to(torch.bfloat16).contiguous(memory_format=cl)
    with torch.no_grad():
        a = up.forward_into(x, buf.clone(), cout)
        b = skip_cat(up(x), buf.clone(), cout)
    assert calls == ([1] if direct else [])
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("shape,lead,pitch", [
    ((4, 24, 8, 16, 16), 0, 48),     # the up-conv part of a UNet concatenation
    ((4, 24, 8, 16, 16), 24, 48),    # the skip part
    ((1, 8, 3, 5, 7), 16, 32),       # odd extents, one vector per voxel
    ((2, 96, 2, 4, 6), 96, 192),
], ids=["lead", "skip", "odd", "wide"])
def test_channel_slice_copy(cuda_ready, shape, lead, pitch, dtype):
    """r4c_channel_slice_copy: a channel slice of an NDHWC buffer copied dense,
    bit-identical to PyTorch's copy of the same view."""
    from rdna4_conv3d import _native
    n, C, d, h, w = shape
    torch.manual_seed(0)
    buf = torch.randn(n, pitch, d, h, w, device="cuda").to(dtype).contiguous(memory_format=torch.channels_last_3d)
    view = buf[:, lead:lead + C]
    out = _native.channel_slice_dense(view)
    assert out is not None and out.is_contiguous(memory_format=torch.channels_last_3d)
    assert torch.equal(out, view.contiguous(memory_format=torch.channels_last_3d))


def test_channel_slice_copy_declines_other_views(cuda_ready):
    """Views that are not a channel slice of an NDHWC buffer (NCDHW, a
    channel count that is not a multiple of 8, fp32) are left to PyTorch."""
    from rdna4_conv3d import _native
    cl = torch.channels_last_3d
    a = torch.randn(2, 16, 4, 4, 4, device="cuda", dtype=torch.bfloat16)
    assert _native.channel_slice_dense(a[:, :8]) is None
    b = torch.randn(2, 16, 4, 4, 4, device="cuda", dtype=torch.bfloat16).contiguous(memory_format=cl)
    assert _native.channel_slice_dense(b[:, :12]) is None
    c = torch.randn(2, 16, 4, 4, 4, device="cuda").contiguous(memory_format=cl)
    assert _native.channel_slice_dense(c[:, :8]) is None


@pytest.mark.parametrize("quantised", [False, True], ids=["random", "ties"])
def test_pool_backward_with_forward_argmax(cuda_ready, quantised):
    """The pool backward fed the forward's argmax gives bit-identical dx,
    dgamma, dbeta to the backward that recomputes the argmax from x."""
    from rdna4_conv3d import _native
    cl = torch.channels_last_3d
    n, C, d, h, w, lead = 2, 24, 8, 12, 16, 24
    g = torch.Generator().manual_seed(7)
    x = torch.randn(n, C, d, h, w, generator=g) * 2.0 + 0.3
    if quantised:
        x = torch.round(x * 2) / 2
    x = x.to(torch.bfloat16).cuda().contiguous(memory_format=cl)
    mi = torch.stack([x.float().mean(dim=(0, 2, 3, 4)), 1.0 / (x.float().var(dim=(0, 2, 3, 4)) + 1e-5).sqrt()])
    af = torch.stack([torch.rand(C, generator=g) + 0.5, torch.randn(C, generator=g) * 0.1]).cuda()
    mi, af = mi.contiguous(), af.contiguous()
    buf, p, am = _native.bn_relu_pool_forward(x, mi, af, lead)
    assert am is not None
    gbuf = torch.randn(n, lead + C, d, h, w, generator=g).to(torch.bfloat16).cuda().contiguous(memory_format=cl)
    gp = torch.randn(n, C, d // 2, h // 2, w // 2, generator=g).to(torch.bfloat16).cuda().contiguous(memory_format=cl)
    cnt = float(n * d * h * w)
    a = _native.bn_relu_pool_backward(gbuf, lead, gp, x, mi, af, cnt, True, None, argmax=am)
    b = _native.bn_relu_pool_backward(gbuf, lead, gp, x, mi, af, cnt, True, None, argmax=None)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    # channels [0, lead) of the buffer are zero until an up-conv writes them
    assert torch.count_nonzero(buf[:, :lead]) == 0
