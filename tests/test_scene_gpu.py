"""GPU: the fused caller glue (cvhrf_scene_prepare/backward) equals the torch restatement
of Scene.render (model.py:1365-1402) on the rows it keeps, forward and backward."""
import math

import pytest
import torch

from complex_valued_holographic_radiance_fields_b200 import scene as SC

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,K,C", [(5000, 3, 3), (3000, 5, 1)])
@pytest.mark.parametrize("view", [0, 1])
def test_fused_glue_matches_torch(cuda, N, K, C, view):
    cam = SC.PinholeCamera(128, 96) if view == 0 else SC.look_at_camera(128, 96, 0.7, 0.3, radius=2.5)
    cam.near = 3.5 if view == 0 else 1.0   # some rows fall outside (near, far)
    base = SC.make_gaussians(N, K=K, C=C, seed=4, device="cuda")
    base["pre_act_phase"] = base["pre_act_phase"] * 3 - 8   # negative and > 2 pi phases
    pa = {k: v.clone().requires_grad_(True) for k, v in base.items()}
    pb = {k: v.clone().requires_grad_(True) for k, v in base.items()}
    ka, ia = SC.render_inputs(pa, cam)
    kb, ib = SC.render_inputs_fused(pb, cam)
    n = ia.numel()
    assert n < N and torch.equal(ia, ib[:n])
    names = ["cam_means_3D", "z_vals", "quats", "scales", "colours", "phase", "opacities", "plane_probs"]
    for k in names:
        assert torch.allclose(ka[k], kb[k][:n], rtol=1e-6, atol=1e-6), k
    assert bool((kb["z_vals"][n:] <= cam.near).all() | (kb["z_vals"][n:] >= cam.far).all())
    g = torch.Generator().manual_seed(1)
    ws = {k: torch.randn(kb[k].shape, generator=g).cuda() for k in names if k != "z_vals"}
    la = sum((ka[k] * ws[k][:n]).sum() for k in ws)
    lb = sum((kb[k][:n] * ws[k][:n]).sum() for k in ws)
    la.backward()
    lb.backward()
    for k in pa:
        # the straight-through gradient is softmax(x / 0.001) with logits ~1e4: one ulp of a
        # scaled logit moves exp() by ~1e-3 relative, so it is compared at 1e-3
        rtol = 1e-3 if k == "pre_act_plane_assignment" else 1e-4
        assert torch.allclose(pa[k].grad, pb[k].grad, rtol=rtol, atol=1e-5), k
