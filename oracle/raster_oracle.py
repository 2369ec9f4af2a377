"""ctypes wrapper of oracle/raster_oracle.c (TEST INFRASTRUCTURE ONLY).

Builds ``oracle/_build/libraster_oracle.so`` with the committed Makefile on first use.
All arrays are numpy float32 / int32, contiguous, on the host.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "_build", "libraster_oracle.so")
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(SO) or os.path.getmtime(SO) < os.path.getmtime(os.path.join(HERE, "raster_oracle.c")):
            build()
        _lib = ctypes.CDLL(SO)
        _lib.ora_raster_forward.restype = ctypes.c_int
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def forward(inp, W, H, fx, fy, px, py, near, far):
    """inp: dict of cam_means, z_vals, quats, scales, colours, phase, opacities, plane_probs, view."""
    a = {k: _f32(v) for k, v in inp.items()}
    N, K, C = a["cam_means"].shape[0], a["plane_probs"].shape[1], a["colours"].shape[1]
    T = ((W + 15) // 16) * ((H + 15) // 16)
    field = np.zeros((K, C, H, W, 2), np.float32)
    final_T = np.zeros((K, H, W), np.float32)
    nc = np.zeros((K, H, W), np.int32)
    ranges = np.zeros((T, 2), np.int32)
    vis = np.zeros(N, np.uint8)
    means = np.zeros((N, 2), np.float32)
    cov = np.zeros((N, 4), np.float32)
    cap = max(64, 8 * N)
    L = lib()
    while True:
        pl = np.zeros(cap, np.int32)
        args = [ctypes.c_int(v) for v in (N, K, C, W, H)] + [ctypes.c_float(v) for v in (fx, fy, px, py, near, far)]
        args += [_ptr(a[k]) for k in ("cam_means", "z_vals", "quats", "scales", "colours", "phase", "opacities",
                                     "plane_probs", "view")]
        args += [_ptr(field), _ptr(final_T), _ptr(nc), _ptr(pl), ctypes.c_int(cap), _ptr(ranges), _ptr(vis),
                 _ptr(means), _ptr(cov)]
        n = L.ora_raster_forward(*args)
        if n >= 0:
            break
        cap = -n
    return dict(field=field[..., 0] + 1j * field[..., 1], final_Ts=final_T, n_contrib=nc, point_list=pl[:n],
                ranges=ranges, visible=np.nonzero(vis)[0].astype(np.int64), means2d=means, cov2d=cov)


def backward(inp, W, H, fx, fy, px, py, near, far, grad_field, fwd):
    a = {k: _f32(v) for k, v in inp.items()}
    N, K, C = a["cam_means"].shape[0], a["plane_probs"].shape[1], a["colours"].shape[1]
    gf = np.ascontiguousarray(np.stack([np.real(grad_field), np.imag(grad_field)], -1).astype(np.float32))
    out = dict(cam_means=np.zeros((N, 3), np.float32), z_vals=np.zeros(N, np.float32),
               quats=np.zeros((N, 4), np.float32), scales=np.zeros((N, 3), np.float32),
               colours=np.zeros((N, C), np.float32), phase=np.zeros((N, C), np.float32),
               opacities=np.zeros(N, np.float32), plane_probs=np.zeros((N, K), np.float32))
    pl = np.ascontiguousarray(fwd["point_list"].astype(np.int32))
    if pl.size == 0:
        pl = np.zeros(1, np.int32)
    args = [ctypes.c_int(v) for v in (N, K, C, W, H)] + [ctypes.c_float(v) for v in (fx, fy, px, py, near, far)]
    args += [_ptr(a[k]) for k in ("cam_means", "z_vals", "quats", "scales", "colours", "phase", "opacities",
                                 "plane_probs", "view")]
    args += [_ptr(gf), _ptr(np.ascontiguousarray(fwd["final_Ts"], np.float32)),
             _ptr(np.ascontiguousarray(fwd["n_contrib"], np.int32)), _ptr(pl),
             _ptr(np.ascontiguousarray(fwd["ranges"], np.int32))]
    args += [_ptr(out[k]) for k in ("cam_means", "z_vals", "quats", "scales", "colours", "phase", "opacities",
                                   "plane_probs")]
    lib().ora_raster_backward(*args)
    return out
