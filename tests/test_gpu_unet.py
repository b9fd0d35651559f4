"""UNet3D training parity on a B200.

The reference's headline parity claim is the loss trajectory of its UNet
under AMP with Adam: max |loss_wmma - loss_stock| over 40 steps, 3-4e-4 on
its hardware (README.md:66 of the reference). Here: the full UNet3D base 24
(24/48/96/192 channels, 4 levels) on a [4, 1, 64, 128, 128] N(0,1) input with
uniform random labels in {0..3}, cross-entropy, AMP bf16, Adam lr 1e-3, seed
0, run once on stock PyTorch (cuDNN) and once with every Conv3d /
ConvTranspose3d on this package's kernels, from the same initial weights.
North-star bound, absolute: |delta loss| <= 1e-3.

That bound sits below this setup's own noise floor over 40 steps: stock
PyTorch against itself with 1% of the input elements moved by one bf16 ulp
drifts apart by ~1.6e-3 by step 40 (random labels, Adam at lr 1e-3: small
gradient differences flip Adam's per-parameter steps). So the test holds
the north-star bound over the first 20 steps, where that floor is ~3e-4, and
over all 40 steps asserts that our run stays within twice the drift of the
perturbed stock run measured in the same test (and within 1e-3 whenever the
floor is below half of it).
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

LOSS_TOL = 1e-3


def _train(net, x, tgt, steps, loss_fn=F.cross_entropy):
    opt = torch.optim.Adam(net.parameters(), lr=1e-3)
    hist = []
    for _ in range(steps):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = loss_fn(net(x), tgt)
        loss.backward()
        opt.step()
        hist.append(loss.detach())
    return [float(v) for v in hist]


def test_unet3d_base24_amp_loss_parity(cuda_ready):
    from rdna4_conv3d import _native
    from rdna4_conv3d.losses import cross_entropy
    from rdna4_conv3d.unet3d import unet3d
    dev = torch.device("cuda")
    torch.manual_seed(0)
    stock = unet3d(24, wmma=False, device=dev)
    state = {k: v.clone() for k, v in stock.state_dict().items()}
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(4, 1, 64, 128, 128, device=dev, generator=g).contiguous(memory_format=torch.channels_last_3d)
    tgt = torch.randint(0, 4, (4, 64, 128, 128), device=dev, generator=g)
    ref = _train(stock, x, tgt, 40)
    # the noise floor: the same stock run on an input 1 bf16 ulp away in 1% of its elements
    xb = x.to(torch.bfloat16).float()
    flip = torch.rand(x.shape, device=dev, generator=g) < 0.01
    xp = torch.where(flip, xb * (1 + 2.0 ** -7), xb).contiguous(memory_format=torch.channels_last_3d)
    pert = unet3d(24, wmma=False, device=dev)
    pert.load_state_dict(state)
    floor = [abs(a - b) for a, b in zip(ref, _train(pert, xp, tgt, 40))]
    ours = unet3d(24, wmma=True, device=dev)
    ours.load_state_dict(state)
    n0 = _native.launch_count()
    got = _train(ours, x, tgt, 40, cross_entropy)   # the whole step on the library: convs, BN, loss
    assert _native.launch_count() - n0 > 40 * 50, "the UNet did not run on the native kernels"
    assert _native.device_error() == 0
    diffs = [abs(a - b) for a, b in zip(ref, got)]
    print("per-step |loss_ours - loss_stock|:", [f"{d:.2e}" for d in diffs])
    print("per-step |loss_stock_perturbed - loss_stock|:", [f"{d:.2e}" for d in floor])
    assert max(diffs[:20]) <= LOSS_TOL, (max(diffs[:20]), diffs[:20])
    assert max(diffs) <= max(LOSS_TOL, 2.0 * max(floor)), (max(diffs), max(floor))
    assert ref[-1] < ref[0]          # the run trains at all


def test_unet3d_channels_and_shapes(cuda_ready):
    """Every conv of the model is served by the native path (no F.conv3d
    fallback inside), and the output keeps the NDHWC layout."""
    from rdna4_conv3d import Conv3dWmma, ConvTranspose3dWmma
    from rdna4_conv3d.conv3d_wmma import conv3d_kernels
    from rdna4_conv3d.unet3d import unet3d
    net = unet3d(24, wmma=True, device="cuda")
    convs = [m for m in net.modules() if isinstance(m, Conv3dWmma)]
    tconvs = [m for m in net.modules() if isinstance(m, ConvTranspose3dWmma)]
    assert len(convs) == 15 and len(tconvs) == 3
    x = torch.randn(1, 1, 16, 32, 32, device="cuda").contiguous(memory_format=torch.channels_last_3d)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = net(x)
    assert y.shape == (1, 4, 16, 32, 32) and y.dtype == torch.bfloat16
    assert y.is_contiguous(memory_format=torch.channels_last_3d)
    fams = conv3d_kernels((4, 48, 64, 128, 128), 24, 3, 1)
    assert set(fams.values()) == {"tcgen05"}
