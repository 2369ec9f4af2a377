"""Golden vectors for the caller glue of the hot path from the REFERENCE's own Python code.

Runs in the build container (it reads the reference source, which is not on the GPU
box): ``python tests/golden/make_scene_golden.py <reference root>``.  model.py cannot be
imported here (it needs odak, imageio, pytorch3d and the CUDA extensions), so these are
taken from the file's syntax tree unmodified and executed on CPU:

  * ``Scene.render`` (model.py:1365-1402): depth values, near/far filter, depth sort,
    gathers, activations;
  * ``Scene.compute_depth_values`` (model.py:1105-1113) and
    ``Scene.get_idxs_to_filter_and_sort`` (model.py:1123-1127);
  * ``Scene.splat`` up to its ``splat_tile_cuda`` call (model.py:1130-1192): camera
    intrinsics, view matrix and the camera-space means;
  * ``Gaussians.apply_activations`` (model.py:595-608) with ``STEFunction`` and
    ``StraightThroughEstimator`` (model.py:41-64).

``splat_tile_cuda`` is replaced by a recorder that stores its keyword arguments and
stops the render.  Third-party pieces are restated:
  * pytorch3d 0.7 ``PerspectiveCameras`` as a stand-in holding R (1, 3, 3), T (1, 3),
    focal_length and principal_point, whose ``get_world_to_view_transform()
    .transform_points(X)`` is pytorch3d's homogeneous row-vector product
    [X, 1] @ [[R, 0], [T, 1]] divided by the w column;
  * ``odak.pi`` (odak 0.2.6) as the double-precision pi.
The backward is taken through the same executed code: a seeded weighted sum of every
recorded output is back-propagated to the seven parameter tensors.  Writes
scene_<i>.npz next to this script.
"""
import ast
import math
import os
import sys
import types

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
PARAMS = ("means", "pre_act_quats", "pre_act_scales", "colours", "pre_act_phase", "pre_act_opacities",
          "pre_act_plane_assignment")
OUTS = ("cam_means_3D", "z_vals", "quats", "scales", "colours", "phase", "opacities", "plane_probs")

# (N, K, C, W, H, camera, near, seed): camera "eye" = R = I, T = (0, 0, 4); otherwise
# (azimuth, elevation, radius) of a look-at camera
CASES = [
    (3000, 3, 3, 128, 96, "eye", 1.0, 0),
    (2500, 5, 1, 96, 96, (0.7, 0.3, 2.5), 1.0, 1),
    (4000, 3, 3, 160, 120, "eye", 3.5, 2),          # the near plane cuts the scene
    (2000, 7, 3, 112, 84, (2.4, -0.35, 4.0), 1.0, 3),
]


class _StopRender(Exception):
    pass


def _look_at(azimuth, elevation, radius):
    ce, se, ca, sa = math.cos(elevation), math.sin(elevation), math.cos(azimuth), math.sin(azimuth)
    eye = torch.tensor([radius * ce * sa, radius * se, -radius * ce * ca], dtype=torch.float64)
    fwd = -eye / eye.norm()
    up = torch.tensor([0.0, 1.0, 0.0], dtype=torch.float64)
    right = torch.linalg.cross(up, fwd)
    right = right / right.norm()
    up2 = torch.linalg.cross(fwd, right)
    R = torch.stack([right, up2, fwd], dim=1)
    T = -(eye @ R)
    return R.float(), T.float()


class _WorldToView:
    def __init__(self, R, T):
        M = torch.zeros(4, 4, dtype=R.dtype)
        M[:3, :3] = R
        M[3, :3] = T
        M[3, 3] = 1.0
        self.M = M

    def transform_points(self, X):
        Xh = torch.cat([X, torch.ones_like(X[:, :1])], dim=1)
        Y = Xh @ self.M
        return Y[:, :3] / Y[:, 3:]


class _Camera:
    """Stand-in for one pytorch3d PerspectiveCameras (screen-space focal length and principal point)."""

    def __init__(self, R, T, fx, fy, px, py):
        self.R = R[None]
        self.T = T[None]
        self.focal_length = torch.tensor([[fx, fy]], dtype=torch.float32)
        self.principal_point = torch.tensor([[px, py]], dtype=torch.float32)

    def get_world_to_view_transform(self):
        return _WorldToView(self.R[0], self.T[0])


def load_code(root):
    path = os.path.join(root, "model.py")
    tree = ast.parse(open(path).read(), path)
    classes = {n.name: n for n in tree.body if isinstance(n, ast.ClassDef)}
    gauss = next(n for n in classes["Gaussians"].body if isinstance(n, ast.FunctionDef)
                 and n.name == "apply_activations")
    gauss.decorator_list = []
    scene_fns = [n for n in classes["Scene"].body if isinstance(n, ast.FunctionDef)
                 and n.name in ("render", "compute_depth_values", "get_idxs_to_filter_and_sort", "splat")]
    assert len(scene_fns) == 4
    mod = ast.Module(body=[classes["STEFunction"], classes["StraightThroughEstimator"], gauss] + scene_fns,
                     type_ignores=[])
    recorded = {}

    def splat_tile_cuda(**kw):
        recorded.clear()
        recorded.update(kw)
        raise _StopRender()

    class _Event:
        def __init__(self, *a, **k):
            pass

        def record(self, *a, **k):
            pass

    class TorchProxy(types.ModuleType):
        def __getattr__(self, name):
            return getattr(torch, name)

    tp = TorchProxy("torch")
    tp.cuda = types.SimpleNamespace(Event=_Event, synchronize=lambda *a: None)
    ns = {"torch": tp, "math": math, "F": F, "odak": types.SimpleNamespace(pi=math.pi), "Tuple": tuple,
          "PerspectiveCameras": object, "USE_SPLAT_TILE_CUDA": True, "splat_tile_cuda": splat_tile_cuda,
          "print": lambda *a, **k: None}
    exec(compile(mod, path, "exec"), ns)
    return ns, recorded


def make_params(N, K, C, seed):
    g = torch.Generator().manual_seed(seed)
    return {
        "means": torch.rand(N, 3, generator=g) * 2 - 1,
        "pre_act_quats": torch.randn(N, 4, generator=g),
        "pre_act_scales": torch.randn(N, 3, generator=g) * 0.5 - 4.5,
        "colours": torch.sigmoid(torch.randn(N, C, generator=g)),
        # negative and > 2 pi phases exercise the mod
        "pre_act_phase": torch.rand(N, C, generator=g) * 6 * math.pi - 8.0,
        "pre_act_opacities": torch.randn(N, generator=g),
        "pre_act_plane_assignment": torch.randn(N, K, generator=g) * 10.0,
    }


def main(root):
    ns, recorded = load_code(root)
    for ci, (N, K, C, W, H, cam, near, seed) in enumerate(CASES):
        p = make_params(N, K, C, seed)
        if cam == "eye":
            R, T = torch.eye(3), torch.tensor([0.0, 0.0, 4.0])
        else:
            R, T = _look_at(*cam)
        fov = 0.69
        fx = (W / 2.0) / math.tan(fov / 2.0)
        camera = _Camera(R, T, fx, fx, W / 2.0, H / 2.0)
        leaves = {k: torch.nn.Parameter(v.clone()) for k, v in p.items()}
        gaussians = types.SimpleNamespace(NEAR_PLANE=near, FAR_PLANE=1000.0, apply_activations=ns["apply_activations"],
                                          **leaves)
        scene = types.SimpleNamespace(gaussians=gaussians, wavelengths=torch.tensor([639e-9, 532e-9, 473e-9][:C]))
        for name in ("render", "compute_depth_values", "get_idxs_to_filter_and_sort", "splat"):
            setattr(scene, name, types.MethodType(ns[name], scene))
        try:
            scene.render(camera, img_size=(W, H))
            raise RuntimeError("splat_tile_cuda was not reached")
        except _StopRender:
            pass
        out = {k: recorded[k] for k in OUTS}
        # the rows kept, in depth order: recover them from the recorded means
        z = (p["means"] @ R + T)[:, 2]
        keep = torch.where((camera.get_world_to_view_transform().transform_points(p["means"])[:, 2] > near)
                           & (camera.get_world_to_view_transform().transform_points(p["means"])[:, 2] < 1000.0))[0]
        zs, order = torch.sort(z[keep])
        idxs = keep[order[zs >= 0]]
        assert torch.equal(out["z_vals"].detach(), z[idxs])
        g = torch.Generator().manual_seed(1000 + seed)
        weights = {k: torch.randn(out[k].shape, generator=g) for k in OUTS if k != "z_vals"}
        loss = sum((out[k] * weights[k]).sum() for k in weights)
        loss.backward()
        d = {"config": np.array([N, K, C, W, H], np.int64), "near": np.array(near, np.float64),
             "R": R.numpy(), "T": T.numpy(), "fx": np.array(fx), "idxs": idxs.numpy()}
        for k in PARAMS:
            d[f"in_{k}"] = p[k].numpy()
            d[f"grad_{k}"] = leaves[k].grad.numpy()
        for k in OUTS:
            d[f"out_{k}"] = out[k].detach().numpy()
            if k in weights:
                d[f"w_{k}"] = weights[k].numpy()
        d["view_matrix"] = recorded["view_matrix"].detach().numpy()
        d["intrinsics"] = np.array([float(recorded[k]) for k in ("fx", "fy", "px", "py")], np.float64)
        np.savez_compressed(os.path.join(HERE, f"scene_{ci}.npz"), **d)
        print(f"scene_{ci}: N={N} -> {idxs.numel()} rows kept")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CVHRF_REFERENCE_ROOT", "."))
