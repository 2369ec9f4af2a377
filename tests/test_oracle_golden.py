"""CPU: the oracle restatements reproduce the reference kernels' golden outputs.

Golden vectors were produced by the reference's own CUDA kernels
(tests/golden/make_golden.py on a B200).  Integer outputs must match exactly;
floating-point outputs within 1e-4 relative L2 (the oracle is scalar C / float64
numpy, the reference fp32 CUDA with atomics).
"""
import glob
import os

import numpy as np
import pytest

from oracle import asm_oracle as AO
from oracle import raster_oracle as RO

GOLD = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-4


def rel(a, b):
    return float(np.linalg.norm((np.asarray(a) - np.asarray(b)).ravel()) / max(np.linalg.norm(np.asarray(b).ravel()), 1e-30))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "asm_*.npz"))))
def test_asm_oracle_vs_reference_golden(path):
    d = np.load(path)
    S, H, W, wl, pitch, dist, ap = d["params"]
    S, H, W = int(S), int(H), int(W)
    out = AO.propagate(d["field"], wl, pitch, dist, S, ap)
    assert rel(out, d["out"]) < TOL
    gf = AO.propagate_adjoint(d["grad_out"], wl, pitch, dist, S, (H, W), ap)
    assert rel(gf, d["grad_field"]) < TOL


def _raster_inputs(d):
    inp = dict(cam_means=d["in_cam_means"], z_vals=d["in_z_vals"], quats=d["in_quats"], scales=d["in_scales"],
               colours=d["in_colours"], phase=d["in_phase"], opacities=d["in_opacities"],
               plane_probs=d["in_plane_probs"], view=d["view"])
    fx, fy, px, py, W, H, near, far = d["camera"]
    return inp, (int(W), int(H), fx, fy, px, py, near, far)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "raster_*.npz"))))
def test_raster_oracle_vs_reference_golden(path):
    d = np.load(path)
    inp, cam = _raster_inputs(d)
    f = RO.forward(inp, *cam)
    assert np.array_equal(f["point_list"], d["point_list"])
    assert np.array_equal(f["ranges"], d["ranges"])
    assert np.array_equal(f["n_contrib"], d["n_contrib"])
    assert np.array_equal(f["visible"], d["visible"])
    assert rel(f["final_Ts"], d["final_Ts"]) < TOL
    assert rel(f["field"], d["field"]) < TOL
    g = RO.backward(inp, *cam, d["grad_out"], f)
    for k in ("cam_means", "quats", "scales", "colours", "phase", "opacities", "plane_probs"):
        assert rel(g[k], d["grad_" + k]) < TOL, k


def test_goldens_present():
    assert len(glob.glob(os.path.join(GOLD, "asm_*.npz"))) >= 4
    assert len(glob.glob(os.path.join(GOLD, "raster_*.npz"))) >= 3
