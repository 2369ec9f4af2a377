"""The training step of BASELINE config 3 on the host CPU (TEST INFRASTRUCTURE ONLY).

Used by bench.py as the CPU baseline and as the ``--impl reference`` arm.  Every
piece is the reference's CPU-capable algorithm:
  * rasterizer forward/backward: oracle/raster_oracle.c (scalar C restatement of the
    reference CUDA rasterizer, OpenMP over tiles);
  * propagation: the reference's own pure-torch path
    (cuda_prop/python_function.py:35-78 ``bandlimited_angular_spectrum_propagation``,
    odak's zero_pad / crop_center / circular_binary_mask restated), run with
    torch.fft on the CPU and differentiated by torch autograd;
  * loss and glue: train.py / model.py restated in torch (as on the GPU path);
  * sparse Adam: conv.cu:1200-1228 restated in torch.
"""
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from oracle import raster_oracle as RO  # noqa: E402


def circular_mask(n, radius):
    """Aperture of the reference CUDA kernel (bandlimited_propagation_cuda.cu:74-80), shifted space."""
    if radius <= 0:
        return torch.ones(n, n)
    off = n / 2.0 - 0.5
    i = torch.arange(n, dtype=torch.float32) - off
    return ((i[None, :] ** 2 + i[:, None] ** 2) < radius * radius).float()


def torch_asm(field, wavelength, pixel_pitch, distance, size, aperture_size=-1.0):
    """python_function.py:35-78 (pure torch)."""
    P = 2 * size
    H, W = field.shape
    pad = torch.zeros(P, P, dtype=field.dtype)
    oy, ox = (P - H) // 2, (P - W) // 2
    pad = torch.nn.functional.pad(field, (ox, P - W - ox, oy, P - H - oy))
    ap = circular_mask(P, aperture_size)
    F = torch.fft.fftshift(torch.fft.fft2(pad))
    fx = torch.fft.fftshift(torch.fft.fftfreq(P, d=pixel_pitch))
    FX, FY = torch.meshgrid(fx, fx, indexing="ij")
    x = torch.tensor(pixel_pitch * float(P))
    d = torch.tensor(distance)
    wl = torch.tensor(wavelength)
    fmax = 1 / torch.sqrt((2 * d * (1 / x)) ** 2 + 1) / wl
    bl = (torch.abs(FX) < fmax) & (torch.abs(FY) < fmax)
    k = 2 * torch.pi / wl
    kz = torch.sqrt(k ** 2 - (2 * torch.pi * FX) ** 2 - (2 * torch.pi * FY) ** 2)
    kz = torch.where(torch.isnan(kz), 0, kz)
    Hf = torch.exp(1j * d * kz) * bl
    y = torch.fft.ifft2(torch.fft.ifftshift(F * Hf * ap))
    s0 = (P - size) // 2
    return y[s0:s0 + size, s0:s0 + size]


class _CpuSplat(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cam, z, q, s, col, ph, op, pp, meta):
        inp = dict(cam_means=cam, z_vals=z, quats=q, scales=s, colours=col, phase=ph, opacities=op, plane_probs=pp,
                   view=meta["view"])
        inp = {k: v.detach().numpy() for k, v in inp.items()}
        f = RO.forward(inp, *meta["cam"])
        ctx.inp, ctx.meta, ctx.fwd = inp, meta, f
        meta["visible"] = torch.from_numpy(f["visible"])
        return torch.from_numpy(f["field"].astype(np.complex64))

    @staticmethod
    def backward(ctx, g):
        out = RO.backward(ctx.inp, *ctx.meta["cam"], g.numpy(), ctx.fwd)
        names = ["cam_means", "z_vals", "quats", "scales", "colours", "phase", "opacities", "plane_probs"]
        return tuple(torch.from_numpy(out[n]) for n in names) + (None,)


class CpuHoloStep:
    """Config-3 training iteration on the CPU, same scene and optics as HoloTrainer."""

    def __init__(self, N=300000, W=800, H=800, K=3, pitch=8e-6, lr=1e-3, eps=1e-15, seed=0):
        from complex_valued_holographic_radiance_fields_b200 import scene as SC
        from complex_valued_holographic_radiance_fields_b200.train_step import WAVELENGTHS, plane_distances
        self.SC = SC
        self.W, self.H, self.K, self.S = W, H, K, max(W, H)
        self.pitch, self.lr, self.eps = pitch, lr, eps
        self.wl = WAVELENGTHS
        d = plane_distances(K)
        self.dist = [float(-d[p]) for p in range(K)]
        self.camera = SC.PinholeCamera(W, H)
        self.params = {k: v.requires_grad_(True) for k, v in SC.make_gaussians(N, K=K, seed=seed, device="cpu").items()}
        self.state = {k: (torch.zeros_like(v), torch.zeros_like(v)) for k, v in self.params.items()}
        g = torch.Generator().manual_seed(1)
        self.target = torch.rand(3, self.S, self.S, generator=g)

    def step(self):
        SC = self.SC
        for p in self.params.values():
            p.grad = None
        kw, idxs = SC.render_inputs(self.params, self.camera)
        meta = dict(cam=(self.W, self.H, kw["fx"], kw["fy"], kw["px"], kw["py"], kw["near_plane"], kw["far_plane"]),
                    view=kw["view_matrix"])
        a = SC.splat_args(kw)
        field = _CpuSplat.apply(a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7], meta)
        holo = 0
        for p in range(self.K):
            holo = holo + torch.stack([torch_asm(field[p, c], self.wl[c], self.pitch, self.dist[p], self.S, self.S)
                                       for c in range(len(self.wl))])
        loss = ((holo.abs() ** 2 - self.target) ** 2).mean()
        loss.backward()
        vis = idxs[meta["visible"]]
        with torch.no_grad():
            for k, prm in self.params.items():
                m, v = self.state[k]
                rows = torch.arange(prm.shape[0]) if prm.dim() == 1 else vis
                g = prm.grad[rows]
                m[rows] = 0.9 * m[rows] + (1.0 - 0.9) * g
                v[rows] = 0.999 * v[rows] + (1.0 - 0.999) * g * g
                prm[rows] += -self.lr * m[rows] / (v[rows].sqrt() + self.eps)
        return float(loss.detach())


def num_threads():
    return int(RO.lib().ora_num_threads())
