"""GPU parity of the tile rasterizer against the reference's own kernels (oracle/_ref).

Bars: tile/sort indices (point_list, ranges) and n_contrib
bit-exact; complex fields and final transmittance within 1e-4 relative L2 (fp32).
Gradients: the reference accumulates them with float atomics in nondeterministic
order, so they are compared at GRAD_TOL relative L2.
"""
import pytest
import torch

from complex_valued_holographic_radiance_fields_b200 import rasterizer as RZ
from complex_valued_holographic_radiance_fields_b200 import scene as SC

pytestmark = pytest.mark.gpu
TOL = 1e-4
GRAD_TOL = 1e-3


def rel(a, b):
    a = a.detach().double() if not a.is_complex() else a.detach().to(torch.complex128)
    b = b.detach().double() if not b.is_complex() else b.detach().to(torch.complex128)
    return float((a - b).abs().pow(2).sum().sqrt() / b.abs().pow(2).sum().sqrt().clamp_min(1e-30))


def inputs(N, W, H, K=3, C=3, seed=0, camera=None):
    cam = camera or SC.PinholeCamera(W, H)
    params = SC.make_gaussians(N, K=K, C=C, seed=seed, device="cuda")
    kw, _ = SC.render_inputs(params, cam)
    return {k: (v.detach() if torch.is_tensor(v) else v) for k, v in kw.items()}


def run_ref(ref, kw):
    args = list(SC.splat_args(kw))
    args[12] = ref.view_buffer(kw["view_matrix"])
    out, vis = ref.RefSplatTileCuda.apply(*args)
    return out, vis


CASES = [
    dict(N=2000, W=128, H=96, K=3, C=3),
    dict(N=20000, W=256, H=256, K=3, C=3),
    dict(N=5000, W=160, H=128, K=1, C=1),
    dict(N=5000, W=144, H=112, K=5, C=3),
    dict(N=4000, W=128, H=128, K=8, C=1),
    dict(N=100000, W=800, H=800, K=3, C=3),   # config 2
]
# C = 2 is not compared with the reference: it dispatches renderTileKernel<MAX_CHANNELS=3>
# for two channels (forward_splat.cu:380-402), whose third-channel store (:263-268) lands
# in the next plane's first channel and, for the last plane, past the end of the output.
# C = 2 is covered against the oracle below.


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"N{c['N']}_{c['W']}x{c['H']}_K{c['K']}_C{c['C']}")
def test_forward_vs_reference(cuda, ref, case):
    kw = inputs(case["N"], case["W"], case["H"], case["K"], case["C"])
    field, info = RZ.rasterize_forward(*SC.splat_args(kw))
    rfield, rvis = run_ref(ref, kw)
    rT, rnc, rpl, rrg, _ = ref.get_rasterizer_info()
    assert torch.equal(info["visible"], rvis)
    assert info["num_pairs"] == rpl.numel()
    assert torch.equal(info["point_list"][:info["num_pairs"]], rpl)
    assert torch.equal(info["ranges"], rrg)
    nc_mis = int((info["n_contrib"] != rnc).sum())
    assert nc_mis == 0, f"n_contrib mismatches: {nc_mis}"
    assert rel(info["final_Ts"], rT) < TOL
    assert rel(field, rfield) < TOL


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"N{c['N']}_{c['W']}x{c['H']}_K{c['K']}_C{c['C']}")
def test_backward_vs_reference(cuda, ref, case):
    kw = inputs(case["N"], case["W"], case["H"], case["K"], case["C"], seed=1)
    g = torch.Generator().manual_seed(5)
    K, C, H, W = case["K"], case["C"], case["H"], case["W"]
    gout = torch.complex(torch.randn(K, C, H, W, generator=g), torch.randn(K, C, H, W, generator=g)).cuda()
    diff_idx = [0, 2, 3, 4, 5, 6, 7]

    def grads(fn, mk):
        args = list(SC.splat_args(kw))
        leaves = []
        for i in diff_idx:
            args[i] = args[i].clone().requires_grad_(True)
            leaves.append(args[i])
        if mk is not None:
            args[12] = mk(args[12])
        out, _ = fn(*args)
        out.backward(gout)
        return [l.grad for l in leaves]

    mine = grads(RZ.SplatTileCuda.apply, None)
    theirs = grads(ref.RefSplatTileCuda.apply, ref.view_buffer)
    names = ["cam_means", "quats", "scales", "colours", "phase", "opacities", "plane_probs"]
    errs = {n: rel(a, b) for n, a, b in zip(names, mine, theirs)}
    assert all(e < GRAD_TOL for e in errs.values()), errs


ORACLE_CASES = [
    dict(N=1500, W=100, H=75, K=3, C=3),     # edge tiles in both directions
    dict(N=800, W=64, H=48, K=2, C=1),
    dict(N=3000, W=200, H=136, K=4, C=2),
]


@pytest.mark.parametrize("case", ORACLE_CASES, ids=lambda c: f"N{c['N']}_{c['W']}x{c['H']}_K{c['K']}_C{c['C']}")
def test_forward_backward_vs_oracle(cuda, case):
    """libcvhrf vs the scalar-C restatement (oracle/raster_oracle.c), incl. edge tiles."""
    import numpy as np
    from oracle import raster_oracle as RO
    kw = inputs(case["N"], case["W"], case["H"], case["K"], case["C"], seed=3)
    field, info = RZ.rasterize_forward(*SC.splat_args(kw))
    inp = dict(cam_means=kw["cam_means_3D"], z_vals=kw["z_vals"], quats=kw["quats"], scales=kw["scales"],
               colours=kw["colours"], phase=kw["phase"], opacities=kw["opacities"], plane_probs=kw["plane_probs"],
               view=kw["view_matrix"])
    inp = {k: v.cpu().numpy() for k, v in inp.items()}
    cam = (case["W"], case["H"], kw["fx"], kw["fy"], kw["px"], kw["py"], kw["near_plane"], kw["far_plane"])
    f = RO.forward(inp, *cam)
    assert np.array_equal(info["point_list"][:info["num_pairs"]].cpu().numpy(), f["point_list"])
    assert np.array_equal(info["ranges"].cpu().numpy(), f["ranges"])
    assert np.array_equal(info["visible"].cpu().numpy(), f["visible"])
    assert int((info["n_contrib"].cpu().numpy() != f["n_contrib"]).sum()) == 0
    assert rel(info["final_Ts"].cpu(), torch.from_numpy(f["final_Ts"])) < TOL
    assert rel(field.cpu(), torch.from_numpy(f["field"].astype(np.complex64))) < TOL
    g = torch.Generator().manual_seed(9)
    gout = torch.complex(torch.randn(field.shape, generator=g), torch.randn(field.shape, generator=g))
    mine = RZ.rasterize_backward(gout.cuda(), kw["cam_means_3D"], kw["z_vals"], kw["quats"], kw["scales"],
                                 kw["colours"], kw["phase"], kw["opacities"], kw["plane_probs"], kw["view_matrix"],
                                 info)
    og = RO.backward(inp, *cam, gout.numpy(), f)
    names = ["cam_means", "z_vals", "quats", "scales", "colours", "phase", "opacities", "plane_probs"]
    for n, a in zip(names, mine):
        if n == "z_vals":
            assert float(a.abs().max()) == 0.0
            continue
        assert rel(a.cpu(), torch.from_numpy(og[n])) < TOL, n
