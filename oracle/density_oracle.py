"""CPU restatement of the reference's adaptive density control and opacity
regularisation (test infrastructure only: the checker of libcvhrf's
cvhrf_density_classify / cvhrf_density_apply / cvhrf_opacity_regularization, never part
of the product path).

Follows model.py:
  * the masks :655-672 (grad_mag = |grad means|, avg_scale = mean exp(scales),
    keep = sigmoid(opacity) >= opacity_threshold, clone / split = keep & large gradient &
    small / large scale; clone and split rows are taken only from kept rows, :729, :808);
  * clones :749-786 (opacity 1 - sqrt(1 - o) mapped back through log(c / (1 - c + 1e-6)
    + 1e-6), means offset by clone_offset_factor * grad / max(|grad|, 1e-8), gradients
    copied; an absent plane-logit gradient reads as zeros);
  * splits :868-930 (scales - log(split_factor), children at means +/- R(q / |q|)
    (noise * mean exp(scales) * 0.5), R the real-first unit-quaternion rotation matrix,
    everything else copied, gradients halved);
  * the output order :932-975, [kept | clones | split children 1 | split children 2];
  * opacity_regularization :1063-1071.
float32 numpy arithmetic.  Pinned to tests/golden/density_*.npz, produced by the
reference's own two methods (tests/golden/make_density_golden.py).
"""
import math

import numpy as np

f32 = np.float32
PARAMS = ("means", "pre_act_quats", "pre_act_scales", "colours", "pre_act_phase", "pre_act_opacities",
          "pre_act_plane_assignment")


def _sigmoid(x):
    return (f32(1) / (f32(1) + np.exp(-x))).astype(f32)


def classify(p, g, grad_threshold, opacity_threshold, small, large):
    """Boolean masks (keep, clone, split) of model.py:655-672 restricted to kept rows."""
    gm = g["means"].astype(f32)
    gmag = np.sqrt((gm * gm).sum(1, dtype=f32)).astype(f32)
    avg = (np.exp(p["pre_act_scales"].astype(f32)).sum(1, dtype=f32) / f32(3)).astype(f32)
    keep = ~(_sigmoid(p["pre_act_opacities"].astype(f32)) < f32(opacity_threshold))
    large_grad = gmag >= f32(grad_threshold)
    clone = keep & large_grad & (avg < f32(small))
    split = keep & large_grad & (avg > f32(large))
    return keep, clone, split, gmag, avg


def quat_to_rot(q):
    q = q / np.maximum(np.sqrt((q * q).sum(1, keepdims=True, dtype=f32)), f32(1e-12))
    r, i, j, k = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    ts = f32(2) / (q * q).sum(1, dtype=f32)
    R = np.stack([1 - ts * (j * j + k * k), ts * (i * j - k * r), ts * (i * k + j * r),
                  ts * (i * j + k * r), 1 - ts * (i * i + k * k), ts * (j * k - i * r),
                  ts * (i * k - j * r), ts * (j * k + i * r), 1 - ts * (i * i + j * j)], 1)
    return R.reshape(-1, 3, 3).astype(f32)


def density_control(p, g, noise, grad_threshold=5e-6, opacity_threshold=1e-3, small_scale_threshold=0.01,
                    large_scale_threshold=0.05, split_factor=2.0, clone_offset_factor=0.05):
    """p, g: dicts of float32 arrays keyed by PARAMS (g[k] None = absent gradient).
    noise: (n_split, 3) standard-normal draws.  Returns (new params, new grads, counts)."""
    N = p["means"].shape[0]
    g = {k: (np.zeros_like(p[k]) if g.get(k) is None else g[k].astype(f32)) for k in PARAMS}
    keep, clone, split, gmag, avg = classify(p, g, grad_threshold, opacity_threshold, small_scale_threshold,
                                             large_scale_threshold)
    ki, ci, si = np.nonzero(keep)[0], np.nonzero(clone)[0], np.nonzero(split)[0]
    assert noise.shape == (len(si), 3)
    newp = {k: [p[k][ki], p[k][ci].copy(), p[k][si].copy(), p[k][si].copy()] for k in PARAMS}
    newg = {k: [g[k][ki], g[k][ci], g[k][si] * f32(0.5), g[k][si] * f32(0.5)] for k in PARAMS}
    # clones
    o = _sigmoid(p["pre_act_opacities"][ci])
    c = (f32(1) - np.sqrt(f32(1) - o)).astype(f32)
    eps = f32(1e-6)
    newp["pre_act_opacities"][1] = np.log(c / (f32(1) - c + eps) + eps).astype(f32)
    nrm = np.maximum(gmag[ci], f32(1e-8))[:, None]
    newp["means"][1] = (p["means"][ci] + f32(clone_offset_factor) * g["means"][ci] / nrm).astype(f32)
    # splits
    R = quat_to_rot(p["pre_act_quats"][si].astype(f32))
    n = noise.astype(f32) * (avg[si] * f32(0.5))[:, None]
    d = np.einsum("nij,nj->ni", R, n).astype(f32)
    newp["means"][2] = (p["means"][si] + d).astype(f32)
    newp["means"][3] = (p["means"][si] - d).astype(f32)
    down = (p["pre_act_scales"][si] - f32(math.log(split_factor))).astype(f32)
    newp["pre_act_scales"][2] = down
    newp["pre_act_scales"][3] = down.copy()
    outp = {k: np.concatenate(v, 0) for k, v in newp.items()}
    outg = {k: np.concatenate(v, 0) for k, v in newg.items()}
    counts = (len(ki), len(ci), len(si), N - len(ki))
    return outp, outg, counts


def opacity_regularization(pre_opac, amount=1e-3):
    """model.py:1063-1071: returns (new pre-activation opacities, affected count)."""
    x = pre_opac.astype(f32)
    o = _sigmoid(x)
    den = np.maximum(o * (f32(1) - o), f32(1e-6))
    return (x - f32(amount) / den).astype(f32), int((o > f32(amount)).sum())
