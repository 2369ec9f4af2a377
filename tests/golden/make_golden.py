"""Generate golden vectors by running the REFERENCE's own kernels (oracle/_ref).

Run on a GPU box after ``python oracle/build_ref.py`` (the built modules travel
with the repo):  ``python tests/golden/make_golden.py [asm|raster|all]``.
Writes small ``.npz`` fixtures next to this script; the CPU tests pin the
oracle restatements against them.  Inputs are seeded synthetic data with the
distributions of BASELINE.json configs 1-3 at reduced sizes.
"""
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import ref_harness as R  # noqa: E402

# (S, H, W, wavelength, pitch, distance, aperture) — padded grid 2S, field H x W
ASM_CASES = [
    (32, 32, 32, 532e-9, 8e-6, 2e-3, -1.0),
    (40, 30, 40, 639e-9, 8e-6, -2e-3, 32.0),
    (48, 48, 36, 473e-9, 3.74e-6, -4e-3, 48.0),
    (64, 64, 64, 532e-9, 8e-6, 0.0, -1.0),
]

# (N, W, H, K, C, seed)
RASTER_CASES = [
    (300, 64, 48, 3, 3, 0),
    (800, 96, 64, 2, 1, 1),
    (1500, 128, 96, 3, 3, 2),
]


def rand_field(H, W, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.rand(H, W, generator=g)
    ph = torch.rand(H, W, generator=g) * 2 * math.pi
    return torch.polar(a, ph).to(torch.complex64)


def make_asm():
    for i, (S, H, W, wl, pitch, d, ap) in enumerate(ASM_CASES):
        f = rand_field(H, W, 100 + i)
        g = rand_field(S, S, 200 + i)
        x = f.cuda().requires_grad_(True)
        y = R.RefBandlimitedPropagationFunction.apply(x, wl, pitch, d, [S, S], ap)
        y.backward(g.cuda())
        np.savez_compressed(os.path.join(HERE, f"asm_{i}.npz"), field=f.numpy(), grad_out=g.numpy(),
                            out=y.detach().cpu().numpy(), grad_field=x.grad.cpu().numpy(),
                            params=np.array([S, H, W, wl, pitch, d, ap], np.float64))
        print("asm", i, "written")


def make_raster():
    from complex_valued_holographic_radiance_fields_b200 import scene as SC
    for i, (N, W, H, K, C, seed) in enumerate(RASTER_CASES):
        cam = SC.PinholeCamera(W, H)
        params = SC.make_gaussians(N, K=K, C=C, seed=seed, device="cuda")
        kw, _ = SC.render_inputs(params, cam)
        args = [a.detach().clone() if torch.is_tensor(a) else a for a in SC.splat_args(kw)]
        diff = [0, 2, 3, 4, 5, 6, 7]
        for j in diff:
            args[j].requires_grad_(True)
        args[12] = R.view_buffer(kw["view_matrix"])
        out, vis = R.RefSplatTileCuda.apply(*args)
        T, nc, pl, rg, _ = R.get_rasterizer_info()
        g = torch.Generator().manual_seed(50 + i)
        gout = torch.complex(torch.randn(out.shape, generator=g), torch.randn(out.shape, generator=g)).cuda()
        out.backward(gout)
        names = ["cam_means", "z_vals", "quats", "scales", "colours", "phase", "opacities", "plane_probs"]
        d = {f"in_{n}": args[j].detach().cpu().numpy() for j, n in enumerate(names)}
        d.update({f"grad_{names[j]}": args[j].grad.cpu().numpy() for j in diff})
        d.update(field=out.detach().cpu().numpy(), visible=vis.cpu().numpy(), final_Ts=T.cpu().numpy(),
                 n_contrib=nc.cpu().numpy(), point_list=pl.cpu().numpy(), ranges=rg.cpu().numpy(),
                 grad_out=gout.cpu().numpy(),
                 camera=np.array([kw["fx"], kw["fy"], kw["px"], kw["py"], W, H, kw["near_plane"], kw["far_plane"]]),
                 view=kw["view_matrix"].cpu().numpy())
        np.savez_compressed(os.path.join(HERE, f"raster_{i}.npz"), **d)
        print("raster", i, "written")


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    if what in ("asm", "all"):
        make_asm()
    if what in ("raster", "all"):
        make_raster()
