"""Golden vectors for Adan from the REFERENCE's own Python implementation.

Runs in the build container (it reads the reference source, which is not on the GPU
box): ``python tests/golden/make_adan_golden.py <reference root>``.  utils/optimizer.py
is executed unmodified except for its one import of the CUDA extension
(``from cuda_prop.cov3d_cuda.python_import import sparse_adam_update``, used only by
SparseGaussianAdam), which is replaced by a stub because that import builds the
extension.  Adan then runs on CPU through both of its torch paths (foreach and single
tensor).  Writes adan_<i>.npz next to this script.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (lr per group, betas, eps, weight_decay, max_grad_norm, no_prox, foreach, steps, sizes, seed)
CASES = [
    ((1e-3, 5e-3), (0.98, 0.92, 0.99), 1e-8, 0.0, 0.0, False, True, 4, (1000, 333), 0),
    ((2e-3, 2e-3), (0.98, 0.92, 0.99), 1e-8, 0.02, 1.0, False, False, 4, (517, 64), 1),
    ((1e-3, 2.5e-2), (0.9, 0.95, 0.999), 1e-15, 0.02, 0.0, True, True, 5, (300, 1200), 2),
    ((5e-3, 1e-3), (0.98, 0.92, 0.99), 1e-8, 0.0, 0.5, True, False, 3, (2048, 7), 3),
]


def load_reference_adan(root):
    path = os.path.join(root, "utils", "optimizer.py")
    src = open(path).read()
    stub_line = "from cuda_prop.cov3d_cuda.python_import import sparse_adam_update"
    assert stub_line in src
    src = src.replace(stub_line, "sparse_adam_update = None  # stub: the CUDA extension is not built here")
    ns = {"__name__": "reference_optimizer", "__file__": path}
    exec(compile(src, path, "exec"), ns)
    return ns["Adan"]


def main(root):
    Adan = load_reference_adan(root)
    for i, (lrs, betas, eps, wd, mgn, no_prox, foreach, steps, sizes, seed) in enumerate(CASES):
        g = torch.Generator().manual_seed(seed)
        init = [torch.randn(n, generator=g) for n in sizes]
        grads = [[torch.randn(n, generator=g) * (0.1 + j) for n in sizes] for j in range(steps)]
        params = [torch.nn.Parameter(x.clone()) for x in init]
        opt = Adan([{"params": [p], "lr": lr} for p, lr in zip(params, lrs)], lr=0.0, betas=betas, eps=eps,
                   weight_decay=wd, max_grad_norm=mgn, no_prox=no_prox, foreach=foreach)
        for j in range(steps):
            for p, gr in zip(params, grads[j]):
                p.grad = gr.clone()
            opt.step()
        d = {"config": np.array([wd, mgn, float(no_prox), eps] + list(betas) + list(lrs), np.float64),
             "steps": np.array(steps)}
        for k, p in enumerate(params):
            st = opt.state[p]
            d[f"init_{k}"] = init[k].numpy()
            d[f"grads_{k}"] = np.stack([grads[j][k].numpy() for j in range(steps)])
            d[f"param_{k}"] = p.detach().numpy()
            for name in ("exp_avg", "exp_avg_sq", "exp_avg_diff", "neg_pre_grad"):
                d[f"{name}_{k}"] = st[name].numpy()
        np.savez_compressed(os.path.join(HERE, f"adan_{i}.npz"), **d)
        print("adan", i, "written")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
