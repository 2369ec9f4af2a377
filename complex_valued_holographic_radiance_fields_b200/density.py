"""Adaptive density control and opacity regularisation on the device.

``density_control(params, ...)`` is Gaussians.density_control (model.py:626-1047) and
``opacity_regularization(params, amount)`` is Gaussians.opacity_regularization
(model.py:1049-1077), over the same seven parameter tensors (``params`` as the
training loop holds them: leaf tensors keyed by the model's attribute names, with
``.grad`` from the last backward).  Classification, the compaction scan and the row
writes are libcvhrf kernels; the host reads the four row counts once to size the new
tensors.  The split noise is drawn with ``torch.randn_like(means_split)`` exactly as the
reference draws it, so a seeded generator gives the reference's children.

Like the reference, the returned tensors are new leaves with ``.grad`` set to the
inherited gradients; optimizer state for them starts fresh (the reference's
setup_optimizer carries state over only between tensors of equal shape,
utils/optimizer.py:67-101).
"""
import ctypes
import math

import torch

from . import _lib

PARAMS = ("means", "pre_act_quats", "pre_act_scales", "colours", "pre_act_phase", "pre_act_opacities",
          "pre_act_plane_assignment")
_FIELDS = dict(zip(PARAMS, ("means", "pre_quats", "pre_scales", "colours", "pre_phase", "pre_opac", "pre_planes")))


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return None if t is None else t.data_ptr()


def _set(values, grads, N, K, C):
    s = _lib.GaussianSet(N=N, K=K, C=C)
    for k in PARAMS:
        setattr(s, _FIELDS[k], _ptr(values[k]))
        setattr(s, "grad_" + _FIELDS[k], _ptr(grads[k]))
    return s


def _checked(params):
    means = params["means"]
    if not means.is_cuda:
        raise ValueError("density_control runs on CUDA tensors")
    N = means.shape[0]
    K = params["pre_act_plane_assignment"].shape[1]
    C = params["colours"].shape[1]
    shapes = {"means": (N, 3), "pre_act_quats": (N, 4), "pre_act_scales": (N, 3), "colours": (N, C),
              "pre_act_phase": (N, C), "pre_act_opacities": (N,), "pre_act_plane_assignment": (N, K)}
    vals, grads = {}, {}
    for k in PARAMS:
        t = params[k]
        if tuple(t.shape) != shapes[k] or t.dtype != torch.float32 or t.device != means.device:
            raise ValueError(f"{k}: expected float32 {shapes[k]} on {means.device}, got {t.dtype} {tuple(t.shape)}")
        vals[k] = t.detach().contiguous()
        g = t.grad
        if g is None and k != "pre_act_plane_assignment":
            # the reference indexes every other .grad unconditionally (model.py:706-711)
            raise ValueError(f"{k}.grad is None: call backward() first")
        grads[k] = None if g is None else g.contiguous()
    return vals, grads, N, K, C


@torch.no_grad()
def density_control(params, grad_threshold=0.000005, opacity_threshold=0.001, small_scale_threshold=0.01,
                    large_scale_threshold=0.05, split_factor=2.0, clone_offset_factor=0.05, noise=None):
    """Clone / split / prune (model.py:626-1047).  Returns (new params dict, counts) where
    counts = dict(kept, cloned, split, pruned) and the new tensors are leaves requiring grad
    with .grad holding the inherited gradients; rows are [kept | clones | split children 1 |
    split children 2].  ``noise`` (n_split x 3, optional) replaces the standard-normal
    draw, e.g. to replay a recorded one."""
    vals, grads, N, K, C = _checked(params)
    dev = vals["means"].device
    L = _lib.lib()
    st = _stream(dev)
    dp = _lib.DensityParams(grad_threshold, opacity_threshold, small_scale_threshold, large_scale_threshold,
                            split_factor, clone_offset_factor)
    src = _set(vals, grads, N, K, C)
    nbytes = L.cvhrf_density_workspace_bytes(N)
    if N > 0 and nbytes == 0:
        raise ValueError(f"density_control: N = {N} is too large")
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    counts = torch.empty(4, dtype=torch.int32, device=dev)
    _lib.check(L.cvhrf_density_classify(ctypes.byref(src), ctypes.byref(dp), _ptr(ws), nbytes, _ptr(counts), st),
               "cvhrf_density_classify")
    kept, cloned, n_split, pruned = (int(x) for x in counts.cpu())
    n_out = kept + cloned + 2 * n_split
    # the reference's draw: torch.randn_like(means_split), means_split = means[split_idx]
    if noise is None:
        noise = torch.randn((n_split, 3), dtype=torch.float32, device=dev)
    elif tuple(noise.shape) != (n_split, 3):
        raise ValueError(f"noise must be ({n_split}, 3), got {tuple(noise.shape)}")
    noise = noise.to(device=dev, dtype=torch.float32).contiguous()
    noise_arg = noise if n_split > 0 else torch.zeros(3, dtype=torch.float32, device=dev)
    out_v = {k: torch.empty((n_out,) + tuple(vals[k].shape[1:]), dtype=torch.float32, device=dev) for k in PARAMS}
    out_g = {k: torch.empty_like(out_v[k]) for k in PARAMS}
    dst = _set(out_v, out_g, n_out, K, C)
    _lib.check(L.cvhrf_density_apply(ctypes.byref(src), ctypes.byref(dp), _ptr(noise_arg), _ptr(ws), nbytes,
                                     ctypes.byref(dst), st), "cvhrf_density_apply")
    new = {}
    for k in PARAMS:
        t = out_v[k].requires_grad_(True)
        t.grad = out_g[k]
        new[k] = t
    return new, {"kept": kept, "cloned": cloned, "split": n_split, "pruned": pruned}


@torch.no_grad()
def opacity_regularization(params, decrease_amount=0.001):
    """model.py:1049-1077, in place on params["pre_act_opacities"]; returns the number of
    rows whose opacity exceeded decrease_amount."""
    t = params["pre_act_opacities"]
    if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError("pre_act_opacities must be a contiguous float32 CUDA tensor")
    affected = torch.empty(1, dtype=torch.int32, device=t.device)
    _lib.check(_lib.lib().cvhrf_opacity_regularization(t.data_ptr(), t.numel(), float(decrease_amount),
                                                       _ptr(affected), _stream(t.device)),
               "cvhrf_opacity_regularization")
    return int(affected.item())
