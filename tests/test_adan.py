"""Adan: the CPU restatement (oracle) against the reference's own golden vectors, and
libcvhrf's fused kernel (GPU) against the same vectors."""
import glob
import os

import numpy as np
import pytest

from oracle.adan_oracle import AdanOracle

GOLD = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "adan_*.npz")))


def _case(path):
    z = np.load(path)
    wd, mgn, no_prox, eps, b1, b2, b3, lr0, lr1 = z["config"]
    steps = int(z["steps"])
    kw = dict(betas=(b1, b2, b3), eps=eps, weight_decay=wd, max_grad_norm=mgn, no_prox=bool(no_prox))
    return z, [lr0, lr1], steps, kw


def _rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


@pytest.mark.parametrize("path", GOLD)
def test_oracle_matches_reference_adan(path):
    z, lrs, steps, kw = _case(path)
    o = AdanOracle([z["init_0"], z["init_1"]], lrs, **kw)
    for j in range(steps):
        o.step([z["grads_0"][j], z["grads_1"][j]])
    for k in range(2):
        assert _rel(o.p[k], z[f"param_{k}"]) < 1e-6
        assert _rel(o.m[k], z[f"exp_avg_{k}"]) < 1e-6
        assert _rel(o.v[k], z[f"exp_avg_sq_{k}"]) < 1e-6
        assert _rel(o.diff[k], z[f"exp_avg_diff_{k}"]) < 1e-6
        assert _rel(o.npg[k], z[f"neg_pre_grad_{k}"]) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("path", GOLD)
def test_fused_adan_matches_reference(cuda, path):
    import torch
    from complex_valued_holographic_radiance_fields_b200.optimizer import Adan
    z, lrs, steps, kw = _case(path)
    params = [torch.nn.Parameter(torch.from_numpy(z[f"init_{k}"]).to(cuda)) for k in range(2)]
    opt = Adan([{"params": [p], "lr": lr} for p, lr in zip(params, lrs)], lr=0.0, **kw)
    for j in range(steps):
        for k, p in enumerate(params):
            p.grad = torch.from_numpy(z[f"grads_{k}"][j]).to(cuda)
        opt.step()
    for k, p in enumerate(params):
        st = opt.state[p]
        assert _rel(p.detach().cpu().numpy(), z[f"param_{k}"]) < 1e-5
        assert _rel(st["exp_avg"].cpu().numpy(), z[f"exp_avg_{k}"]) < 1e-5
        assert _rel(st["exp_avg_sq"].cpu().numpy(), z[f"exp_avg_sq_{k}"]) < 1e-5
        assert _rel(st["exp_avg_diff"].cpu().numpy(), z[f"exp_avg_diff_{k}"]) < 1e-5
        assert _rel(st["neg_pre_grad"].cpu().numpy(), z[f"neg_pre_grad_{k}"]) < 1e-5


@pytest.mark.gpu
def test_trainer_with_adan_steps(cuda):
    import torch
    from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer
    tr = HoloTrainer(N=20000, W=128, H=128, K=3, device=cuda, seed=4, optimizer="adan")
    before = {k: v.detach().clone() for k, v in tr.params.items()}
    losses = [tr.step().item() for _ in range(3)]
    assert all(np.isfinite(losses))
    assert all(not torch.equal(before[k], tr.params[k]) for k in before)
