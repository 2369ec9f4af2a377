"""Fused L2 intensity loss (libcvhrf) against the torch expression of the training step."""
import pytest
import torch

from complex_valued_holographic_radiance_fields_b200.loss import intensity_l2_loss

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(3, 800, 800), (1, 5, 7), (2, 33, 31), (1,)])
def test_loss_and_grad_match_torch(cuda, shape):
    g = torch.Generator(device=cuda).manual_seed(3)
    holo = torch.randn(shape, dtype=torch.complex64, device=cuda, generator=g)
    target = torch.rand(shape, dtype=torch.float32, device=cuda, generator=g)
    for _ in range(2):  # the completion counter resets itself between calls
        a = holo.clone().requires_grad_(True)
        la = intensity_l2_loss(a, target)
        la.backward(torch.tensor(0.75, device=cuda))
        b = holo.clone().requires_grad_(True)
        lb = ((b.real.square() + b.imag.square() - target) ** 2).mean()
        lb.backward(torch.tensor(0.75, device=cuda))
        assert abs(la.item() - lb.item()) <= 1e-6 * abs(lb.item())
        err = (a.grad - b.grad).abs().pow(2).sum().sqrt() / b.grad.abs().pow(2).sum().sqrt()
        assert err.item() < 1e-6


def test_loss_is_deterministic(cuda):
    g = torch.Generator(device=cuda).manual_seed(4)
    holo = torch.randn(3, 400, 400, dtype=torch.complex64, device=cuda, generator=g)
    target = torch.rand(3, 400, 400, dtype=torch.float32, device=cuda, generator=g)
    vals = {intensity_l2_loss(holo, target).item() for _ in range(5)}
    assert len(vals) == 1
