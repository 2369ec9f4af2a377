"""The caller of the hot path: seeded synthetic scenes and the ``Scene.render`` glue.

The reference's datasets are not available, so scenes are drawn from the
distributions the benchmark configs name (seeded, on the CPU, then moved to the
device so every implementation sees identical bits):

* means U[-1, 1]^3, log-scales N(-4.5, 0.5), quaternions normalize(N(0, 1)^4),
  opacity logits N(0, 1), colours sigmoid(N(0, 1)), phase U[0, 2 pi), plane logits
  10 N(0, 1) (model.py:138-169 ``_load_random``);
* a pinhole camera R = I, T = (0, 0, 4), fov 0.69 rad (fx = fy = (W/2) / tan(0.345)),
  principal point at the image centre, near 1, far 1000 (model.py:80-81).

``render_inputs`` restates ``Scene.render`` (model.py:1365-1402): camera transform
X @ R + T, near/far filter, depth sort, gather, activations
(``apply_activations`` model.py:595-608 with the straight-through one-hot of
model.py:41-56).  It stays PyTorch: it is glue around the kernels, not the hot path.
"""
import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class PinholeCamera:
    W: int
    H: int
    fov: float = 0.69
    R: torch.Tensor = None
    T: torch.Tensor = None
    near: float = 1.0
    far: float = 1000.0

    def __post_init__(self):
        if self.R is None:
            self.R = torch.eye(3)
        if self.T is None:
            self.T = torch.tensor([0.0, 0.0, 4.0])

    def on(self, device):
        """(R, T) as contiguous float32 tensors on `device`, copied once and cached (a
        per-step host-to-device copy from pageable memory would synchronise the GPU)."""
        dev = torch.device(device)
        cache = self.__dict__.setdefault("_dev_cache", {})
        key = (str(dev), self.R.data_ptr(), self.T.data_ptr())
        if key not in cache:
            cache.clear()
            cache[key] = (self.R.to(dev, torch.float32).contiguous(), self.T.to(dev, torch.float32).contiguous())
        return cache[key]

    @property
    def fx(self):
        return (self.W / 2.0) / math.tan(self.fov / 2.0)

    @property
    def fy(self):
        return self.fx

    @property
    def px(self):
        return self.W / 2.0

    @property
    def py(self):
        return self.H / 2.0


def look_at_camera(W, H, azimuth, elevation, radius=4.0, fov=0.69):
    """World-to-view (R, T) for a camera on a sphere looking at the origin, in the
    row-vector convention X_cam = X_world @ R + T used by the model."""
    ce, se, ca, sa = math.cos(elevation), math.sin(elevation), math.cos(azimuth), math.sin(azimuth)
    eye = torch.tensor([radius * ce * sa, radius * se, -radius * ce * ca])
    fwd = -eye / eye.norm()
    up = torch.tensor([0.0, 1.0, 0.0])
    right = torch.linalg.cross(up, fwd)
    right = right / right.norm()
    up2 = torch.linalg.cross(fwd, right)
    Rm = torch.stack([right, up2, fwd], dim=1)      # columns: camera axes in world coords
    T = -(eye @ Rm)
    return PinholeCamera(W, H, fov, Rm.float(), T.float())


def make_gaussians(N, K=3, C=3, seed=0, device="cuda", frustum=None):
    """Pre-activation Gaussian parameters (dict of float32 tensors on `device`)."""
    g = torch.Generator().manual_seed(seed)
    if frustum is None:
        means = torch.rand(N, 3, generator=g) * 2 - 1
        log_scales = torch.randn(N, 3, generator=g) * 0.5 - 4.5
    else:  # (depth_min, depth_max, half_tan_x, half_tan_y, log_scale_mean, log_scale_std, cam_T_z)
        dmin, dmax, htx, hty, lm, ls, tz = frustum
        d = torch.rand(N, generator=g) * (dmax - dmin) + dmin
        x = (torch.rand(N, generator=g) * 2 - 1) * htx * d
        y = (torch.rand(N, generator=g) * 2 - 1) * hty * d
        means = torch.stack([x, y, d - tz], 1)
        log_scales = torch.randn(N, 3, generator=g) * ls + lm
    p = dict(
        means=means,
        pre_act_scales=log_scales,
        pre_act_quats=torch.randn(N, 4, generator=g),
        pre_act_opacities=torch.randn(N, generator=g),
        colours=torch.sigmoid(torch.randn(N, C, generator=g)),
        pre_act_phase=torch.rand(N, C, generator=g) * 2 * math.pi,
        pre_act_plane_assignment=torch.randn(N, K, generator=g) * 10.0,
    )
    return {k: v.float().to(device).contiguous() for k, v in p.items()}


class _STE(torch.autograd.Function):
    """model.py:41-56: one-hot forward, softmax(x / 0.001) backward."""

    @staticmethod
    def forward(ctx, x, temperature=0.001):
        ctx.save_for_backward(x)
        ctx.t = temperature
        return F.one_hot(torch.argmax(x, dim=1), num_classes=x.size(1)).float()

    @staticmethod
    def backward(ctx, g):
        x, = ctx.saved_tensors
        return g * F.softmax(x / ctx.t, dim=1), None


def apply_activations(pre_act_quats, pre_act_scales, pre_act_phase, pre_act_opacities, pre_act_plane_assignment):
    """model.py:595-608."""
    scales = torch.exp(pre_act_scales)
    quats = F.normalize(pre_act_quats)
    phase = pre_act_phase % (2.0 * math.pi)
    opacities = torch.sigmoid(pre_act_opacities)
    plane_probs = _STE.apply(pre_act_plane_assignment)
    return quats, scales, phase, opacities, plane_probs


def render_inputs(params, camera):
    """Scene.render up to the splat call (model.py:1365-1402).

    Returns (kwargs for splat_tile_cuda, idxs) where idxs maps the filtered,
    depth-sorted subset back to rows of `params`.
    """
    dev = params["means"].device
    R, T = camera.on(dev)
    cam_all = params["means"] @ R + T
    z_all = cam_all[:, 2]
    valid = torch.where((z_all > camera.near) & (z_all < camera.far))[0]
    zs, order = torch.sort(z_all[valid])
    idxs = valid[order[zs >= 0]]
    quats, scales, phase, opacities, plane_probs = apply_activations(
        params["pre_act_quats"][idxs], params["pre_act_scales"][idxs], params["pre_act_phase"][idxs],
        params["pre_act_opacities"][idxs], params["pre_act_plane_assignment"][idxs])
    cam_means = params["means"][idxs] @ R + T
    kw = dict(cam_means_3D=cam_means, z_vals=cam_means[:, 2].contiguous(), quats=quats, scales=scales,
              colours=params["colours"][idxs], phase=phase, opacities=opacities, plane_probs=plane_probs,
              fx=camera.fx, fy=camera.fy, px=camera.px, py=camera.py, view_matrix=R,
              img_size=(camera.W, camera.H), near_plane=camera.near, far_plane=camera.far)
    return kw, idxs


def splat_args(kw):
    """Positional argument tuple of splat_tile_cuda / SplatTileCuda.apply from `render_inputs` kwargs."""
    return (kw["cam_means_3D"], kw["z_vals"], kw["quats"], kw["scales"], kw["colours"], kw["phase"],
            kw["opacities"], kw["plane_probs"], kw["fx"], kw["fy"], kw["px"], kw["py"], kw["view_matrix"],
            kw["img_size"], kw["near_plane"], kw["far_plane"])


_PARAM_ORDER = ("means", "pre_act_quats", "pre_act_scales", "colours", "pre_act_phase", "pre_act_opacities",
                "pre_act_plane_assignment")


class FusedRenderInputs(torch.autograd.Function):
    """`render_inputs` as two libcvhrf kernels (cvhrf_scene_prepare / cvhrf_scene_backward).

    Returns the rasterizer inputs for ALL rows in depth order (rows outside near/far sort
    last and are culled by the rasterizer) plus `order`, the parameter row of each.
    """

    @staticmethod
    def forward(ctx, means, pq, ps, col, pph, pop, ppl, R, T, near, far, owned_planes=0xFFFFFFFF):
        import ctypes
        from . import _lib
        dev = means.device
        ins = [t.contiguous() for t in (means, pq, ps, col, pph, pop, ppl)]
        N, C, K = means.shape[0], col.shape[1], ppl.shape[1]
        G = _lib.Gaussians(N, K, C, *[t.data_ptr() for t in ins])
        R = R.to(dev, torch.float32).contiguous()
        T = T.to(dev, torch.float32).contiguous()
        L = _lib.lib()
        ws = torch.empty(max(1, L.cvhrf_scene_workspace_bytes(N)), dtype=torch.uint8, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        order = torch.empty(N, dtype=torch.int32, device=dev)
        outs = [torch.empty(N, 3, **f32), torch.empty(N, **f32), torch.empty(N, 4, **f32), torch.empty(N, 3, **f32),
                torch.empty(N, C, **f32), torch.empty(N, C, **f32), torch.empty(N, **f32), torch.empty(N, K, **f32)]
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        from .profiling import timed
        with timed("scene_prepare"):
            rc = L.cvhrf_scene_prepare_owned(ctypes.byref(G), R.data_ptr(), T.data_ptr(), float(near), float(far),
                                             int(owned_planes) & 0xFFFFFFFF, ws.data_ptr(), ws.numel(),
                                             order.data_ptr(), *[o.data_ptr() for o in outs], st)
        _lib.check(rc, "cvhrf_scene_prepare_owned")
        ctx.save_for_backward(*ins, R, order)
        ctx.mark_non_differentiable(order, outs[1])
        return (*outs, order)

    @staticmethod
    def backward(ctx, g_cam, g_z, g_q, g_s, g_col, g_ph, g_op, g_pl, g_order):
        import ctypes
        from . import _lib
        *ins, R, order = ctx.saved_tensors
        N, C, K = ins[0].shape[0], ins[3].shape[1], ins[6].shape[1]
        dev = ins[0].device
        G = _lib.Gaussians(N, K, C, *[t.data_ptr() for t in ins])

        def g(t, shape):
            return torch.zeros(shape, dtype=torch.float32, device=dev) if t is None else t.contiguous()
        gs = [g(g_cam, (N, 3)), g(g_q, (N, 4)), g(g_s, (N, 3)), g(g_col, (N, C)), g(g_ph, (N, C)), g(g_op, (N,)),
              g(g_pl, (N, K))]
        # all parameter gradients live in ONE flat buffer (views), so a data-parallel
        # exchange can all-reduce them in place without a concatenating copy
        flat = torch.empty(sum(t.numel() for t in ins), dtype=torch.float32, device=dev)
        d, off = [], 0
        for t in ins:
            d.append(flat[off:off + t.numel()].view_as(t))
            off += t.numel()
        FusedRenderInputs.last_grad_buffer = flat
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        from .profiling import timed
        with timed("scene_backward"):
            rc = _lib.lib().cvhrf_scene_backward(ctypes.byref(G), R.data_ptr(), order.data_ptr(),
                                                 *[t.data_ptr() for t in gs], *[t.data_ptr() for t in d], st)
        _lib.check(rc, "cvhrf_scene_backward")
        return (*d, None, None, None, None, None)


def render_inputs_fused(params, camera, owned_planes=0xFFFFFFFF):
    """Same contract as `render_inputs`, through the fused kernels (all rows, culled by depth).
    `owned_planes` (bit p = plane p) additionally culls the rows whose one-hot plane is not
    owned (plane-parallel training)."""
    R, T = camera.on(params["means"].device)
    outs = FusedRenderInputs.apply(*[params[k] for k in _PARAM_ORDER], R, T, camera.near, camera.far, owned_planes)
    cam, z, q, s, col, ph, op, pl, order = outs
    kw = dict(cam_means_3D=cam, z_vals=z, quats=q, scales=s, colours=col, phase=ph, opacities=op, plane_probs=pl,
              fx=camera.fx, fy=camera.fy, px=camera.px, py=camera.py,
              view_matrix=R,
              img_size=(camera.W, camera.H), near_plane=camera.near, far_plane=camera.far)
    return kw, order.long()


# ---- checkpoint format (model.py:610-624 save_gaussians) ------------------------------

CHECKPOINT_KEYS = ("pre_act_quats", "means", "pre_act_scales", "colours", "pre_act_phase", "pre_act_opacities",
                   "pre_act_plane_assignment")


def save_gaussians(params, path):
    """The reference's Gaussian checkpoint: torch.save of a dict of the seven pre-activation
    parameter tensors, moved to the CPU (model.py:610-624; same keys, same layout)."""
    torch.save({k: params[k].detach().cpu() for k in CHECKPOINT_KEYS}, path)


def load_gaussians(path, device="cuda", requires_grad=True):
    """Load a checkpoint written by save_gaussians (or by the reference's save_gaussians)
    as contiguous float32 tensors on `device`."""
    state = torch.load(path, map_location="cpu")
    missing = [k for k in CHECKPOINT_KEYS if k not in state]
    if missing:
        raise KeyError(f"checkpoint lacks {missing}")
    return {k: state[k].to(device=device, dtype=torch.float32).contiguous().requires_grad_(requires_grad)
            for k in CHECKPOINT_KEYS}
