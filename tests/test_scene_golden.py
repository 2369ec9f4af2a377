"""The caller glue of the hot path (Scene.render up to splat_tile_cuda, model.py:1365-1402,
with apply_activations :595-608 and the straight-through estimator :41-64) against golden
vectors produced by executing the reference's own code (tests/golden/make_scene_golden.py).

Bars: the kept rows and their depth sequence bit-exact (rows of exactly equal depth,
whose order the unstable torch.sort leaves open, compared as sets); every rasterizer input within 1e-6
(relative and absolute); parameter gradients within 1e-4 (1e-3 for the straight-through
gradient, softmax(x / 0.001) of logits ~1e4, where one ulp of a scaled logit moves exp()
by ~1e-3 relative).

CPU: `scene.render_inputs`, the torch statement of the glue.  GPU: `render_inputs_fused`
(cvhrf_scene_prepare / cvhrf_scene_backward), whose first rows are the kept ones in
depth order and whose remaining rows are culled.
"""
import glob
import os

import numpy as np
import pytest
import torch

from complex_valued_holographic_radiance_fields_b200 import scene as SC

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "scene_*.npz")))
PARAMS = ("means", "pre_act_quats", "pre_act_scales", "colours", "pre_act_phase", "pre_act_opacities",
          "pre_act_plane_assignment")
OUTS = ("cam_means_3D", "z_vals", "quats", "scales", "colours", "phase", "opacities", "plane_probs")


def _camera(z):
    N, K, C, W, H = (int(v) for v in z["config"])
    cam = SC.PinholeCamera(W, H, R=torch.from_numpy(z["R"]), T=torch.from_numpy(z["T"]))
    cam.near = float(z["near"])
    return cam


def _tie_order(z, idx):
    """Positions sorted by (depth, row): the depth sort leaves the order of equal depths
    to the sort implementation (torch.sort is not stable), so rows of equal depth are
    compared as sets."""
    return np.lexsort((idx, z))


def _check(z, kw, idxs, params, n_kept_rows_first):
    n = z["idxs"].shape[0]
    got_idx = idxs[:n].long().cpu().numpy() if n_kept_rows_first else idxs.long().cpu().numpy()
    got_z = kw["z_vals"][:n].detach().cpu().numpy()
    assert np.array_equal(got_z, z["out_z_vals"])           # the depth sequence, bit-exact
    mine, theirs = _tie_order(got_z, got_idx), _tie_order(z["out_z_vals"], z["idxs"])
    assert np.array_equal(got_idx[mine], z["idxs"][theirs])  # the kept rows, ties as sets
    for k in OUTS:
        a = kw[k][:n].detach().cpu().numpy()[mine]
        b = z[f"out_{k}"][theirs]
        assert np.allclose(a, b, rtol=1e-6, atol=1e-6), (k, float(np.abs(a - b).max()))
    assert np.allclose(kw["view_matrix"].detach().cpu().numpy(), z["view_matrix"])
    assert np.allclose([kw["fx"], kw["fy"], kw["px"], kw["py"]], z["intrinsics"], rtol=1e-6)
    # the golden weights follow the reference's row order; permute them onto this order
    perm = np.empty(n, np.int64)
    perm[mine] = theirs
    perm_t = torch.from_numpy(perm)
    loss = sum((kw[k][:n] * torch.from_numpy(z[f"w_{k}"])[perm_t].to(kw[k].device)).sum()
               for k in OUTS if k != "z_vals")
    loss.backward()
    for k in PARAMS:
        g = params[k].grad.cpu().numpy()
        rtol = 1e-3 if k == "pre_act_plane_assignment" else 1e-4
        assert np.allclose(g, z[f"grad_{k}"], rtol=rtol, atol=1e-5), (k, float(np.abs(g - z[f"grad_{k}"]).max()))


@pytest.mark.parametrize("path", GOLDEN, ids=os.path.basename)
def test_render_inputs_vs_reference_golden(path):
    z = np.load(path)
    params = {k: torch.from_numpy(z[f"in_{k}"]).clone().requires_grad_(True) for k in PARAMS}
    kw, idxs = SC.render_inputs(params, _camera(z))
    _check(z, kw, idxs, params, False)


@pytest.mark.gpu
@pytest.mark.parametrize("path", GOLDEN, ids=os.path.basename)
def test_fused_glue_vs_reference_golden(cuda, path):
    z = np.load(path)
    params = {k: torch.from_numpy(z[f"in_{k}"]).to(cuda).requires_grad_(True) for k in PARAMS}
    kw, idxs = SC.render_inputs_fused(params, _camera(z))
    n = z["idxs"].shape[0]
    # rows past the kept ones are outside (near, far)
    zz = kw["z_vals"][n:]
    assert bool(((zz <= float(z["near"])) | (zz >= 1000.0)).all())
    _check(z, kw, idxs, params, True)
