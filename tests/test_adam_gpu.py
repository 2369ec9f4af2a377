"""GPU parity of the fused sparse Adam against the reference adamUpdate kernel.

Bar: Adam-updated parameters within 1e-5 after one step on
identical gradients (the reference kernel is fed the same gradients).
"""
import pytest
import torch

from complex_valued_holographic_radiance_fields_b200 import optimizer as OPT

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _mk(N, D, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(N, D, generator=g).cuda() for _ in range(2)] + [torch.rand(N, D, generator=g).cuda() * 1e-2]


@pytest.mark.parametrize("N,D,V", [(1000, 3, 400), (300000, 4, 250000), (5000, 1, 5000), (10, 3, 0)])
def test_sparse_adam_update_vs_reference(cuda, ref, N, D, V):
    p, g, v0 = _mk(N, D, N + D)
    m0 = torch.randn(N, D, device="cuda") * 0.1
    vis = torch.randperm(N, device="cuda")[:V].sort().values
    gc = g[vis].unsqueeze(0).contiguous()
    mine = [t.clone().unsqueeze(0) for t in (p, m0, v0)]
    theirs = [t.clone().unsqueeze(0) for t in (p, m0, v0)]
    for step in range(3):
        OPT.sparse_adam_update(mine[0], gc, mine[1], mine[2], vis, 1e-3, 0.9, 0.999, 1e-15)
        if V > 0:
            ref.ref_adam_update(theirs[0], gc, theirs[1], theirs[2], vis, 1e-3, 0.9, 0.999, 1e-15)
    for a, b in zip(mine, theirs):
        assert (a - b).abs().max().item() <= TOL


def test_sparse_gaussian_adam_step(cuda, ref):
    """SparseGaussianAdam.step (optimizer.py:180-265): 2-D groups sparse, 1-D group dense."""
    N, V = 20000, 12000
    torch.manual_seed(0)
    shapes = {"means": (N, 3), "scales": (N, 3), "quats": (N, 4), "colours": (N, 3), "phase": (N, 3),
              "opac": (N,), "planes": (N, 3)}
    ps = {k: torch.randn(*s, device="cuda").requires_grad_(True) for k, s in shapes.items()}
    grads = {k: torch.randn(*s, device="cuda") for k, s in shapes.items()}
    vis = torch.randperm(N, device="cuda")[:V].sort().values
    opt = OPT.SparseGaussianAdam([{"params": [p], "lr": 1e-3} for p in ps.values()], lr=1e-3, eps=1e-15)
    expected = {}
    for k, p in ps.items():
        p.grad = grads[k].clone()
        e = p.detach().clone()
        m = torch.zeros_like(e)
        v = torch.zeros_like(e)
        if e.dim() == 1:
            m.mul_(0.9).add_(grads[k], alpha=0.1)
            v.mul_(0.999).addcmul_(grads[k], grads[k], value=0.001)
            e.addcdiv_(m, v.sqrt().add_(1e-15), value=-1e-3)
        else:
            ref.ref_adam_update(e.unsqueeze(0), grads[k][vis].unsqueeze(0).contiguous(), m.unsqueeze(0),
                                v.unsqueeze(0), vis, 1e-3, 0.9, 0.999, 1e-15)
        expected[k] = e
    opt.step(vis)
    for k, p in ps.items():
        assert (p.detach() - expected[k]).abs().max().item() <= TOL, k
