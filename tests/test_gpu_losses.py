"""Cross-entropy over NDHWC logits (r4c_ce_*) against F.cross_entropy.

The stock loss is computed in fp32 from the same bf16/fp16 logits (what
autocast does); the loss must agree to fp32 rounding and the logits gradient
to one rounding of the logits' dtype.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

LOSS_TOL = 1e-5   # relative, fp32 vs fp32 (the library sums in double)
GRAD_TOL = 1e-2   # max|g - ref| / max|ref|, one bf16 rounding


def _logits(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    z = (3 * torch.randn(shape, device="cuda", generator=g)).to(dtype)
    return z.contiguous(memory_format=torch.channels_last_3d)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(4, 4, 64, 128, 128), (2, 4, 3, 5, 7), (1, 16, 4, 4, 4), (2, 3, 2, 3, 4)],
                         ids=["unet", "small", "c16", "c3"])
def test_ce_matches_stock(cuda_ready, shape, dtype):
    from rdna4_conv3d.losses import cross_entropy
    from rdna4_conv3d import _native
    n, c, d, h, w = shape
    z = _logits(shape, dtype, 1).requires_grad_(True)
    g = torch.Generator(device="cuda").manual_seed(2)
    t = torch.randint(0, c, (n, d, h, w), device="cuda", generator=g)
    t[..., 0] = -100                                     # ignored voxels
    n0 = _native.launch_count()
    loss = cross_entropy(z, t)
    loss.backward()
    assert _native.launch_count() - n0 == 3, "the loss did not run on the native kernels"
    zr = z.detach().float().requires_grad_(True)
    ref = F.cross_entropy(zr, t)
    ref.backward()
    assert loss.dtype == torch.float32 and z.grad.dtype == dtype
    assert z.grad.is_contiguous(memory_format=torch.channels_last_3d)
    assert abs(float(loss.detach()) - float(ref.detach())) <= LOSS_TOL * abs(float(ref.detach()))
    # the stock gradient reaches fp16/bf16 logits through autocast's cast:
    # compare with it rounded the same way (fp16 gradients of a mean over
    # millions of voxels sit in the subnormal range, spacing 2^-24)
    gr = zr.grad.to(dtype).float()
    err = float((z.grad.float() - gr).abs().max())
    assert err <= GRAD_TOL * float(gr.abs().max()) + (2.0 ** -24 if dtype == torch.float16 else 0.0)
    assert float(z.grad[..., 0].abs().max()) == 0.0      # ignored voxels get no gradient
    assert _native.device_error() == 0


def test_ce_deterministic_and_scaled(cuda_ready):
    from rdna4_conv3d.losses import cross_entropy
    z = _logits((2, 4, 8, 16, 16), torch.bfloat16, 3).requires_grad_(True)
    t = torch.randint(0, 4, (2, 8, 16, 16), device="cuda")
    a = cross_entropy(z, t)
    b = cross_entropy(z, t)
    assert float(a) == float(b)                          # fixed summation order
    (2.5 * a).backward()                                 # upstream gradient read from device memory
    g1 = z.grad.clone()
    z.grad = None
    cross_entropy(z, t).backward()
    assert torch.allclose(g1.float(), 2.5 * z.grad.float(), rtol=1e-2, atol=1e-6)


def test_ce_falls_back_for_other_layouts(cuda_ready):
    from rdna4_conv3d import _native
    from rdna4_conv3d.losses import cross_entropy
    z = torch.randn(2, 4, 3, 5, 7, device="cuda")        # fp32, NCDHW: the stock path
    t = torch.randint(0, 4, (2, 3, 5, 7), device="cuda")
    n0 = _native.launch_count()
    assert torch.allclose(cross_entropy(z, t), F.cross_entropy(z, t))
    assert _native.launch_count() == n0
