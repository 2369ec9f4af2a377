"""Golden vectors for density control from the REFERENCE's own Python code.

Runs in the build container (it reads the reference source, which is not on the GPU
box): ``python tests/golden/make_density_golden.py <reference root>``.  model.py cannot
be imported here (it needs odak, imageio, pytorch3d and the CUDA extensions), so the
two methods ``Gaussians.density_control`` (model.py:626-1047) and
``Gaussians.opacity_regularization`` (model.py:1049-1077) are taken from the file's
syntax tree unmodified and executed on CPU against a small stand-in ``self`` holding
the seven parameters with their gradients.  Their one third-party call,
``pytorch3d.transforms.quaternion_to_matrix`` (pytorch3d 0.7, real part first), is given
by the standard unit-quaternion rotation formula below; ``torch.randn_like`` is wrapped
so the split noise it draws is recorded.  Writes density_<i>.npz next to this script.
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

# (N, K, C, grad_threshold, opacity_threshold, small, large, split_factor, clone_offset,
#  plane-logit grads present, regularisation amount, seed)
CASES = [
    (1200, 3, 3, 5e-6, 1e-3, 0.01, 0.05, 2.0, 0.05, True, 1e-3, 0),
    (800, 4, 3, 0.0, 1e-3, 0.02, 0.03, 1.6, 0.01, False, 2e-3, 1),   # threshold 0: zero-gradient clones
    (501, 3, 1, 2e-5, 5e-2, 0.01, 0.05, 2.0, 0.05, True, 1e-3, 2),
]


def quaternion_to_matrix(q):
    r, i, j, k = torch.unbind(q, -1)
    two_s = 2.0 / (q * q).sum(-1)
    m = torch.stack((1 - two_s * (j * j + k * k), two_s * (i * j - k * r), two_s * (i * k + j * r),
                     two_s * (i * j + k * r), 1 - two_s * (i * i + k * k), two_s * (j * k - i * r),
                     two_s * (i * k - j * r), two_s * (j * k + i * r), 1 - two_s * (i * i + j * j)), -1)
    return m.reshape(q.shape[:-1] + (3, 3))


def load_methods(root):
    path = os.path.join(root, "model.py")
    tree = ast.parse(open(path).read(), path)
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "Gaussians")
    fns = [n for n in cls.body if isinstance(n, ast.FunctionDef)
           and n.name in ("density_control", "opacity_regularization")]
    assert len(fns) == 2
    mod = ast.Module(body=fns, type_ignores=[])
    draws = []

    class TorchProxy(types.ModuleType):
        def __getattr__(self, name):
            return getattr(torch, name)

    tp = TorchProxy("torch")

    def randn_like(x, *a, **k):
        out = torch.randn_like(x, *a, **k)
        draws.append(out.clone())
        return out

    tp.randn_like = randn_like
    p3d = types.SimpleNamespace(transforms=types.SimpleNamespace(quaternion_to_matrix=quaternion_to_matrix))
    ns = {"torch": tp, "math": math, "F": F, "pytorch3d": p3d, "sys": sys, "print": lambda *a, **k: None}
    exec(compile(mod, path, "exec"), ns)
    return ns["density_control"], ns["opacity_regularization"], draws


def make_inputs(N, K, C, seed, with_opt_grads):
    g = torch.Generator().manual_seed(seed)
    p = {
        "means": torch.rand(N, 3, generator=g) * 2 - 1,
        "pre_act_quats": torch.randn(N, 4, generator=g),
        "pre_act_scales": torch.randn(N, 3, generator=g) - 3.8,
        "colours": torch.rand(N, C, generator=g),
        "pre_act_phase": torch.rand(N, C, generator=g) * 2 * math.pi,
        "pre_act_opacities": torch.randn(N, generator=g) * 3.5,
        "pre_act_plane_assignment": torch.randn(N, K, generator=g) * 10,
    }
    gr = {k: torch.randn(v.shape, generator=g) * 1e-4 for k, v in p.items()}
    # gradient magnitudes spread over 1e-8 .. 1e-3; some rows exactly zero
    mag = 10.0 ** (torch.rand(N, 1, generator=g) * 5 - 8)
    gm = torch.randn(N, 3, generator=g)
    gr["means"] = gm / gm.norm(dim=1, keepdim=True) * mag
    gr["means"][::97] = 0.0
    if not with_opt_grads:
        gr["pre_act_plane_assignment"] = None  # the one gradient the reference allows to be absent
    return p, gr


def main(root):
    density_control, opacity_regularization, draws = load_methods(root)
    for ci, (N, K, C, gt, ot, sm, lg, sf, co, og, amount, seed) in enumerate(CASES):
        p, gr = make_inputs(N, K, C, seed, og)
        obj = types.SimpleNamespace(device="cpu", num_planes=K, is_isotropic=False)
        for k in PARAMS:
            t = torch.nn.Parameter(p[k].clone())
            t.grad = None if gr[k] is None else gr[k].clone()
            setattr(obj, k, t)
        draws.clear()
        torch.manual_seed(100 + seed)
        density_control(obj, grad_threshold=gt, opacity_threshold=ot, small_scale_threshold=sm,
                        large_scale_threshold=lg, split_factor=sf, clone_offset_factor=co)
        assert len(draws) <= 1
        noise = draws[0].numpy() if draws else np.zeros((0, 3), np.float32)
        d = {"config": np.array([N, K, C], np.int64),
             "thresholds": np.array([gt, ot, sm, lg, sf, co, amount], np.float64),
             "opt_grads": np.array(int(og)), "noise": noise}
        for k in PARAMS:
            d[f"in_{k}"] = p[k].numpy()
            if gr[k] is not None:
                d[f"in_grad_{k}"] = gr[k].numpy()
            d[f"out_{k}"] = getattr(obj, k).detach().numpy()
            d[f"out_grad_{k}"] = getattr(obj, k).grad.numpy()
        affected = opacity_regularization(obj, decrease_amount=amount)
        d["reg_pre_act_opacities"] = obj.pre_act_opacities.detach().numpy()
        d["reg_affected"] = np.array(affected)
        np.savez_compressed(os.path.join(HERE, f"density_{ci}.npz"), **d)
        print(f"density_{ci}: N={N} -> {d['out_means'].shape[0]} rows, {noise.shape[0]} split, affected {affected}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CVHRF_REFERENCE_ROOT", "."))
