"""Complex-field tile rasterizer (the ``cov3d_cuda`` operator surface).

Mirrors ``cuda_prop/cov3d_cuda/python_import.py``:

* ``SplatTileCuda.apply(cam_means_3D, z_vals, quats, scales, colours, phase, opacities,
  plane_probs, fx, fy, px, py, view_matrix, img_size, near_plane, far_plane,
  tile_size=(16, 16))`` (python_import.py:283-342) returns ``(field, visible_indices)``
  with ``field`` complex64 (K, C, H, W); backward returns 8 gradients + 9 ``None``.
* ``splat_tile_cuda(...)`` (python_import.py:421-447), same arguments.

State the backward needs (per-Gaussian geometry, the sorted pair list, ranges,
final transmittance, last-contributor index) lives on ``ctx``, not on a process-wide
singleton, so several forwards may precede their backwards.  ``forward_info`` keeps
the reference tuple ``(final_Ts, n_contrib, point_list, ranges, visible_indices)``.
"""
import ctypes

import torch

from . import _lib
from .profiling import timed

_F32 = torch.float32
# (tile, Gaussian) pair count of the most recent forward (diagnostics / benchmarking)
last_num_pairs = 0


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None and t.numel() > 0 else ctypes.c_void_p(0)


def _f(v):
    return float(v.item()) if torch.is_tensor(v) else float(v)


def _prep(t, name, shape_tail=None):
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (libcvhrf has no CPU path)")
    if t.dtype != _F32:
        raise TypeError(f"{name} must be float32, got {t.dtype}")
    return t.contiguous()


def _scene(cam, z, q, s, col, ph, op, pp, view, W, H, fx, fy, px, py, near, far):
    N = cam.shape[0]
    sc = _lib.RasterScene()
    sc.N, sc.K, sc.C, sc.W, sc.H = N, pp.shape[1], col.shape[1], int(W), int(H)
    sc.fx, sc.fy, sc.px, sc.py, sc.near_plane, sc.far_plane = fx, fy, px, py, near, far
    for name, t in (("cam_means", cam), ("z_vals", z), ("quats", q), ("scales", s), ("colours", col),
                    ("phase", ph), ("opacities", op), ("plane_probs", pp), ("view_matrix", view)):
        setattr(sc, name, t.data_ptr() if t.numel() > 0 else 0)
    return sc


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def rasterize_forward(cam, z, q, s, col, ph, op, pp, fx, fy, px, py, view, img_size, near, far,
                      pairs_capacity=None):
    """Run the forward; returns (field, info) where info holds everything the backward needs.

    With `pairs_capacity` the call makes no host round trip (CUDA-graph capturable): buffers
    are sized for that many (tile, Gaussian) pairs, visibility comes back as a uint8 mask,
    and info["overflow"] (device int32) becomes 1 if the scene needed more pairs."""
    dev = cam.device
    cam, z, q, s = (_prep(cam, "cam_means_3D"), _prep(z, "z_vals"), _prep(q, "quats"), _prep(s, "scales"))
    col, ph, op, pp = (_prep(col, "colours"), _prep(ph, "phase"), _prep(op, "opacities"), _prep(pp, "plane_probs"))
    view = _prep(view.reshape(3, 3), "view_matrix")
    if s.dim() != 2 or s.shape[1] != 3:
        raise ValueError("scales must be (N, 3)")
    W, H = (int(img_size[0]), int(img_size[1]))
    N, K, C = cam.shape[0], pp.shape[1], col.shape[1]
    if C > 3 or K > 8:
        raise ValueError(f"C <= 3 and K <= 8 required (got C={C}, K={K})")
    fx, fy, px, py, near, far = (_f(v) for v in (fx, fy, px, py, near, far))
    sc = _scene(cam, z, q, s, col, ph, op, pp, view, W, H, fx, fy, px, py, near, far)
    L = _lib.lib()
    st = _stream(dev)
    gbytes = L.cvhrf_raster_geometry_workspace_bytes(N, K, C)
    geom = torch.empty(gbytes, dtype=torch.uint8, device=dev)
    counts = torch.empty(2, dtype=torch.int32, device=dev)
    with timed("raster_geometry"):
        _lib.check(L.cvhrf_raster_forward_geometry(ctypes.byref(sc), _p(geom), gbytes, _p(counts), st),
                   "cvhrf_raster_forward_geometry")
    if pairs_capacity is not None:
        return _render_capacity(sc, geom, gbytes, counts, int(pairs_capacity), N, K, C, W, H, dev, st,
                                (fx, fy, px, py, near, far))
    num_pairs, num_visible = (int(v) for v in counts.cpu().tolist())  # one host sync (the reference has four)
    global last_num_pairs
    last_num_pairs = num_pairs
    bbytes = L.cvhrf_raster_binning_workspace_bytes(N, num_pairs, W, H)
    binws = torch.empty(bbytes, dtype=torch.uint8, device=dev)
    T = ((W + 15) // 16) * ((H + 15) // 16)
    field = torch.empty((K, C, H, W), dtype=torch.complex64, device=dev)
    final_Ts = torch.empty((K, H, W), dtype=_F32, device=dev)
    n_contrib = torch.empty((K, H, W), dtype=torch.int32, device=dev)
    point_list = torch.zeros(max(num_pairs, 1), dtype=torch.int32, device=dev)
    ranges = torch.empty((T, 2), dtype=torch.int32, device=dev)
    vis = torch.empty(num_visible if num_pairs > 0 else 0, dtype=torch.int64, device=dev)
    with timed("raster_render"):
        _lib.check(L.cvhrf_raster_forward_render(ctypes.byref(sc), _p(geom), gbytes, num_pairs, vis.numel(), _p(binws),
                                                 bbytes, _p(field), _p(final_Ts), _p(n_contrib), _p(point_list),
                                                 _p(ranges), _p(vis), st), "cvhrf_raster_forward_render")
    info = dict(geom=geom, gbytes=gbytes, binws=binws, bbytes=bbytes, num_pairs=num_pairs, final_Ts=final_Ts,
                n_contrib=n_contrib, point_list=point_list, ranges=ranges, visible=vis, img=(W, H),
                cam=(fx, fy, px, py, near, far))
    return field, info


last_counts = None


def _render_capacity(sc, geom, gbytes, counts, cap, N, K, C, W, H, dev, st, camp):
    global last_counts
    L = _lib.lib()
    cap = max(cap, 1)
    bbytes = L.cvhrf_raster_binning_workspace_bytes(N, cap, W, H)
    binws = torch.empty(bbytes, dtype=torch.uint8, device=dev)
    T = ((W + 15) // 16) * ((H + 15) // 16)
    field = torch.empty((K, C, H, W), dtype=torch.complex64, device=dev)
    final_Ts = torch.empty((K, H, W), dtype=_F32, device=dev)
    n_contrib = torch.empty((K, H, W), dtype=torch.int32, device=dev)
    point_list = torch.empty(cap, dtype=torch.int32, device=dev)
    ranges = torch.empty((T, 2), dtype=torch.int32, device=dev)
    vis = torch.empty(max(N, 1), dtype=torch.uint8, device=dev)[:N]
    overflow = torch.zeros(1, dtype=torch.int32, device=dev)
    with timed("raster_render"):
        _lib.check(L.cvhrf_raster_forward_render_capacity(ctypes.byref(sc), _p(geom), gbytes, _p(counts), cap,
                                                          _p(binws), bbytes, _p(field), _p(final_Ts), _p(n_contrib),
                                                          _p(point_list), _p(ranges), _p(vis), _p(overflow), st),
                   "cvhrf_raster_forward_render_capacity")
    last_counts = counts
    info = dict(geom=geom, gbytes=gbytes, binws=binws, bbytes=bbytes, num_pairs=cap, final_Ts=final_Ts,
                n_contrib=n_contrib, point_list=point_list, ranges=ranges, visible=vis, img=(W, H), cam=camp,
                counts=counts, overflow=overflow)
    return field, info


def rasterize_backward(grad_field, cam, z, q, s, col, ph, op, pp, view, info):
    dev = cam.device
    cam, z, q, s, col, ph, op, pp = (t.contiguous() for t in (cam, z, q, s, col, ph, op, pp))
    view = view.reshape(3, 3).contiguous()
    g = grad_field.contiguous()
    if g.dtype != torch.complex64:
        g = g.to(torch.complex64)
    W, H = info["img"]
    fx, fy, px, py, near, far = info["cam"]
    N, K, C = cam.shape[0], pp.shape[1], col.shape[1]
    sc = _scene(cam, z, q, s, col, ph, op, pp, view, W, H, fx, fy, px, py, near, far)
    L = _lib.lib()
    npairs = info["num_pairs"]
    rbytes = L.cvhrf_raster_backward_workspace_bytes(npairs, K, C)
    rws = torch.empty(rbytes, dtype=torch.uint8, device=dev)
    gcam = torch.empty((N, 3), dtype=_F32, device=dev)
    gz = torch.empty((N,), dtype=_F32, device=dev)
    gq = torch.empty((N, 4), dtype=_F32, device=dev)
    gs = torch.empty((N, 3), dtype=_F32, device=dev)
    gcol = torch.empty((N, C), dtype=_F32, device=dev)
    gph = torch.empty((N, C), dtype=_F32, device=dev)
    gop = torch.empty((N,), dtype=_F32, device=dev)
    gpp = torch.empty((N, K), dtype=_F32, device=dev)
    with timed("raster_backward"):
        _lib.check(L.cvhrf_raster_backward(ctypes.byref(sc), _p(info["geom"]), info["gbytes"], _p(info["binws"]),
                                           info["bbytes"], npairs, _p(g), _p(info["final_Ts"]),
                                           _p(info["n_contrib"]), _p(info["point_list"]), _p(info["ranges"]), _p(rws),
                                           rbytes, _p(gcam), _p(gz), _p(gq), _p(gs), _p(gcol), _p(gph), _p(gop),
                                           _p(gpp), _stream(dev)),
                   "cvhrf_raster_backward")
    return gcam, gz, gq, gs, gcol, gph, gop, gpp


class SplatTileCuda(torch.autograd.Function):
    """python_import.py:283-342 — same argument order and return tuple."""

    @staticmethod
    def forward(ctx, cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                fx, fy, px, py, view_matrix, img_size, near_plane, far_plane, tile_size=(16, 16)):
        field, info = rasterize_forward(cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                                        fx, fy, px, py, view_matrix, img_size, near_plane, far_plane)
        ctx.save_for_backward(cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                              view_matrix)
        ctx.info = info
        ctx.forward_info = (info["final_Ts"], info["n_contrib"], info["point_list"], info["ranges"], info["visible"])
        ctx.mark_non_differentiable(info["visible"])
        return field, info["visible"]

    @staticmethod
    def backward(ctx, grad_output, grad_visible_indices=None):
        cam, z, q, s, col, ph, op, pp, view = ctx.saved_tensors
        grads = rasterize_backward(grad_output, cam, z, q, s, col, ph, op, pp, view, ctx.info)
        return grads + (None,) * 9


class SplatTileCudaCapacity(torch.autograd.Function):
    """SplatTileCuda without host synchronisation (CUDA-graph capturable).

    Extra last argument `pairs_capacity`; returns (field, visible_mask) where visible_mask
    is uint8 per Gaussian.  The tensor `ctx`-independent overflow flag of the latest call
    is `rasterizer.last_overflow` (device int32, 1 = capacity exceeded, outputs invalid)."""

    @staticmethod
    def forward(ctx, cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                fx, fy, px, py, view_matrix, img_size, near_plane, far_plane, pairs_capacity):
        global last_overflow
        field, info = rasterize_forward(cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                                        fx, fy, px, py, view_matrix, img_size, near_plane, far_plane,
                                        pairs_capacity=pairs_capacity)
        ctx.save_for_backward(cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                              view_matrix)
        ctx.info = info
        last_overflow = info["overflow"]
        ctx.mark_non_differentiable(info["visible"])
        return field, info["visible"]

    @staticmethod
    def backward(ctx, grad_output, grad_visible=None):
        cam, z, q, s, col, ph, op, pp, view = ctx.saved_tensors
        grads = rasterize_backward(grad_output, cam, z, q, s, col, ph, op, pp, view, ctx.info)
        return grads + (None,) * 9


last_overflow = None


def splat_tile_cuda(cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                    fx, fy, px, py, view_matrix, img_size, near_plane, far_plane, tile_size=(16, 16)):
    """python_import.py:421-447.  `tile_size` is accepted and ignored (tiles are 16 x 16, as in the reference)."""
    return SplatTileCuda.apply(cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                               fx, fy, px, py, view_matrix, img_size, near_plane, far_plane, tile_size)
