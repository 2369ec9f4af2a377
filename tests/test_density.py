"""Adaptive density control and opacity regularisation: the CPU restatement (oracle)
against the reference's own golden vectors (tests/golden/density_*.npz, made by running
model.py's two methods), and libcvhrf's kernels (GPU) against the same vectors and
against the oracle at larger sizes.

Bars: row selection and order, copied rows and gradients bit-exact; the computed values
(clone means and opacities, split children's means) within 1e-5 relative L2."""
import glob
import os

import numpy as np
import pytest

from oracle import density_oracle as D

GOLD = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "density_*.npz")))
COMPUTED = ("means", "pre_act_opacities")


def _rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


def _load(path):
    z = np.load(path)
    th = [float(x) for x in z["thresholds"]]
    p = {k: z[f"in_{k}"] for k in D.PARAMS}
    g = {k: (z[f"in_grad_{k}"] if f"in_grad_{k}" in z.files else None) for k in D.PARAMS}
    kw = dict(grad_threshold=th[0], opacity_threshold=th[1], small_scale_threshold=th[2],
              large_scale_threshold=th[3], split_factor=th[4], clone_offset_factor=th[5])
    return z, p, g, kw, th[6]


def _compare(out_p, out_g, z_or_dict, get):
    for k in D.PARAMS:
        a, b = out_p[k], get(z_or_dict, "out_", k)
        assert a.shape == b.shape, (k, a.shape, b.shape)
        if k in COMPUTED:
            assert _rel(a, b) <= 1e-5, k
        else:
            assert np.array_equal(a, b), k
        assert np.array_equal(out_g[k], get(z_or_dict, "out_grad_", k)), k


def test_golden_fixtures_present():
    assert len(GOLD) == 3


@pytest.mark.parametrize("path", GOLD)
def test_oracle_matches_reference_density_control(path):
    z, p, g, kw, amount = _load(path)
    op, og, counts = D.density_control(p, g, z["noise"], **kw)
    _compare(op, og, z, lambda zz, pre, k: zz[f"{pre}{k}"])
    assert op["means"].shape[0] == counts[0] + counts[1] + 2 * counts[2]
    reg, affected = D.opacity_regularization(z["out_pre_act_opacities"], amount)
    assert _rel(reg, z["reg_pre_act_opacities"]) <= 1e-6
    assert affected == int(z["reg_affected"])


def test_oracle_all_categories_exercised():
    seen = np.zeros(3, bool)
    for path in GOLD:
        z, p, g, kw, _ = _load(path)
        _, _, counts = D.density_control(p, g, z["noise"], **kw)
        seen |= np.array([counts[1] > 0, counts[2] > 0, counts[3] > 0])
    assert seen.all()


# ---------------------------------------------------------------- GPU ----------
def _to_cuda(p, g, cuda):
    import torch
    params = {}
    for k in D.PARAMS:
        t = torch.from_numpy(np.ascontiguousarray(p[k])).to(cuda).requires_grad_(True)
        t.grad = None if g[k] is None else torch.from_numpy(np.ascontiguousarray(g[k])).to(cuda)
        params[k] = t
    return params


def _np(params):
    return ({k: v.detach().cpu().numpy() for k, v in params.items()},
            {k: v.grad.cpu().numpy() for k, v in params.items()})


@pytest.mark.gpu
@pytest.mark.parametrize("path", GOLD)
def test_gpu_density_control_matches_reference(cuda, path):
    import torch
    from complex_valued_holographic_radiance_fields_b200 import density
    z, p, g, kw, amount = _load(path)
    new, counts = density.density_control(_to_cuda(p, g, cuda), noise=torch.from_numpy(z["noise"]).to(cuda), **kw)
    op, og = _np(new)
    _compare(op, og, z, lambda zz, pre, k: zz[f"{pre}{k}"])
    assert counts["split"] == z["noise"].shape[0]
    assert all(v.is_leaf and v.requires_grad for v in new.values())
    affected = density.opacity_regularization(new, amount)
    assert affected == int(z["reg_affected"])
    assert _rel(new["pre_act_opacities"].detach().cpu().numpy(), z["reg_pre_act_opacities"]) <= 1e-6


def _random_set(N, K, C, seed):
    rng = np.random.default_rng(seed)
    f = np.float32
    p = {"means": rng.uniform(-1, 1, (N, 3)).astype(f), "pre_act_quats": rng.standard_normal((N, 4)).astype(f),
         "pre_act_scales": (rng.standard_normal((N, 3)) - 3.8).astype(f), "colours": rng.random((N, C)).astype(f),
         "pre_act_phase": (rng.random((N, C)) * 6.28).astype(f),
         "pre_act_opacities": (rng.standard_normal(N) * 3.5).astype(f),
         "pre_act_plane_assignment": (rng.standard_normal((N, K)) * 10).astype(f)}
    g = {k: (rng.standard_normal(v.shape) * 1e-4).astype(f) for k, v in p.items()}
    g["means"] = (rng.standard_normal((N, 3)) * 10.0 ** rng.uniform(-8, -3, (N, 1))).astype(f)
    return p, g


@pytest.mark.gpu
@pytest.mark.parametrize("N,K,C,seed", [(300_000, 3, 3, 0), (65_537, 5, 1, 1)])
def test_gpu_density_control_matches_oracle_large(cuda, N, K, C, seed):
    import torch
    from complex_valued_holographic_radiance_fields_b200 import density
    p, g = _random_set(N, K, C, seed)
    torch.manual_seed(seed)
    new, counts = density.density_control(_to_cuda(p, g, cuda))
    # the same draw the product made: randn(n_split, 3) from the same seed
    torch.manual_seed(seed)
    noise = torch.randn((counts["split"], 3), device=cuda).cpu().numpy()
    op, og, oc = D.density_control(p, g, noise)
    assert (counts["kept"], counts["cloned"], counts["split"], counts["pruned"]) == oc
    assert min(oc[1:]) > 0
    _compare(*_np(new), {"p": op, "g": og}, lambda d, pre, k: d["g" if pre == "out_grad_" else "p"][k])


@pytest.mark.gpu
def test_gpu_density_control_edges(cuda):
    import torch
    from complex_valued_holographic_radiance_fields_b200 import density
    # empty set
    p, g = _random_set(0, 3, 3, 0)
    new, counts = density.density_control(_to_cuda(p, g, cuda))
    assert counts == {"kept": 0, "cloned": 0, "split": 0, "pruned": 0}
    assert new["means"].shape == (0, 3) and new["pre_act_plane_assignment"].shape == (0, 3)
    # everything pruned
    p, g = _random_set(1000, 3, 3, 1)
    p["pre_act_opacities"][:] = -20.0
    new, counts = density.density_control(_to_cuda(p, g, cuda))
    assert counts["pruned"] == 1000 and new["means"].shape[0] == 0
    # absent plane-logit gradient reads as zeros; zero-gradient clones stay in place
    p, g = _random_set(5000, 3, 3, 2)
    g["means"][:100] = 0.0
    g["pre_act_plane_assignment"] = None
    new, counts = density.density_control(_to_cuda(p, g, cuda), grad_threshold=0.0, small_scale_threshold=1.0,
                                          large_scale_threshold=1e9)
    op, og, oc = D.density_control(p, g, np.zeros((0, 3), np.float32), grad_threshold=0.0,
                                   small_scale_threshold=1.0, large_scale_threshold=1e9)
    assert counts["cloned"] == oc[1] > 100
    _compare(*_np(new), {"p": op, "g": og}, lambda d, pre, k: d["g" if pre == "out_grad_" else "p"][k])
    assert not new["pre_act_plane_assignment"].grad.any()
    # a missing required gradient is an error, as in the reference
    params = _to_cuda(*_random_set(10, 3, 3, 3), cuda)
    params["colours"].grad = None
    with pytest.raises(ValueError):
        density.density_control(params)


@pytest.mark.gpu
def test_trainer_densify_then_step(cuda):
    import torch
    from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer
    t = HoloTrainer(N=30000, W=128, H=128, K=3, device=cuda, seed=5)
    for _ in range(2):
        t.step()
    n0 = t.params["means"].shape[0]
    counts = t.densify(grad_threshold=1e-7, small_scale_threshold=0.012, large_scale_threshold=0.012)
    n1 = t.params["means"].shape[0]
    assert n1 == counts["kept"] + counts["cloned"] + 2 * counts["split"] != n0
    loss = t.step()
    assert torch.isfinite(loss)
    t.capture(headroom=1.5, warmup=1)
    assert torch.isfinite(t.replay())
