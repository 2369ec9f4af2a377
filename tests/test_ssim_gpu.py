"""Fused SSIM (libcvhrf) against the CPU restatement (oracle/ssim_oracle.py) and the
reference's own fusedssim kernels (oracle/_ref)."""
import pytest
import torch

from oracle import ssim_oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(3, 64, 80), (3, 100, 75), (3, 256, 256)]


def rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _imgs(shape, seed, cuda):
    g = torch.Generator().manual_seed(seed)
    a = torch.rand(shape, generator=g)
    b = (a + 0.2 * torch.randn(shape, generator=g)).clamp(0, 1)
    return a.to(cuda), b.to(cuda)


@pytest.mark.parametrize("shape", SHAPES)
def test_map_and_gradient_vs_oracle(cuda, shape):
    from complex_valued_holographic_radiance_fields_b200.ssim import C1, C2, FusedSSIMMap
    a, b = _imgs(shape, 1, cuda)
    g = torch.randn(shape, generator=torch.Generator().manual_seed(2)).to(cuda)
    x = a.clone().requires_grad_(True)
    m = FusedSSIMMap.apply(C1, C2, x, b)
    m.backward(g)
    om, og = O.ssim_map_and_grad(a, b, g)
    assert rel(m, om) < 1e-5
    assert rel(x.grad, og) < 1e-4


@pytest.mark.parametrize("shape", SHAPES)
def test_fast_ssim_mean_and_gradient_vs_oracle(cuda, shape):
    from complex_valued_holographic_radiance_fields_b200.ssim import fast_ssim
    a, b = _imgs(shape, 3, cuda)
    x = a.clone().requires_grad_(True)
    s = fast_ssim(x, b)
    (s * 0.7).backward()
    om, og = O.ssim_map_and_grad(a, b, torch.full(shape, 0.7 / a.numel()))
    assert abs(s.item() - om.mean().item()) <= 1e-6 * abs(om.mean().item())
    assert rel(x.grad, og) < 1e-4


@pytest.mark.parametrize("shape", SHAPES)
def test_reference_fusedssim_pins_the_oracle(cuda, ref, shape):
    a, b = _imgs(shape, 5, cuda)
    m = ref.cov3d().fusedssim(0.01 ** 2, 0.03 ** 2, a, b)
    assert rel(m, O.ssim_map(a.cpu(), b.cpu())) < 1e-5


def test_reference_backward_interior(cuda, ref):
    """The reference backward (fusedssim_backwardCUDA) drops the terms of pixels in its
    blocks' 5-pixel halos (their dL/dmap is read as 0, conv.cu:1082-1084), so it is
    compared with the oracle only at pixels at least 5 away from its 22-pixel block seams."""
    shape = (3, 96, 120)
    a, b = _imgs(shape, 7, cuda)
    g = torch.randn(shape, generator=torch.Generator().manual_seed(8)).to(cuda)
    rg = ref.cov3d().fusedssim_backward(0.01 ** 2, 0.03 ** 2, a, b, g)
    _, og = O.ssim_map_and_grad(a, b, g)
    ys = torch.arange(shape[1])
    xs = torch.arange(shape[2])
    iy = ((ys % 22) >= 5) & ((ys % 22) < 17)
    ix = ((xs % 22) >= 5) & ((xs % 22) < 17)
    mask = iy[:, None] & ix[None, :]
    sel = lambda t: t.detach().cpu()[:, mask]  # noqa: E731
    assert rel(sel(rg), sel(og)) < 1e-4
