"""Golden vectors for the reconstruction / multiplane-loss path from the REFERENCE's own
Python code.

Runs in the build container (it reads the reference source, which is not on the GPU
box): ``python tests/golden/make_recon_golden.py <reference root>``.  utils/propagator.py
is executed unmodified except for its two odak import lines, which are replaced by a stub
module: odak 0.2.6 is not installed, so its helpers (get_propagation_kernel for the
band-limited angular spectrum, custom, generate_complex_field, calculate_amplitude /
phase, zero_pad, crop_center, circular_binary_mask, generate_2d_gaussian) come from this
package's restatement (reconstruction.py) and from the short definitions below.  These
vectors therefore pin the reference's own propagator / multiplane_loss_odak code and the
train.py:280-300 loss loop around it, not odak itself.  The propagation runs on CPU
(torch.fft).  With the identity laser powers of train.py:878 every frame holds one
channel, so the reconstructions are stored summed over frames (depths x channels).
Writes recon_<i>.npz next to this script.
"""
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from complex_valued_holographic_radiance_fields_b200 import reconstruction as R  # noqa: E402

# (S, H, W, K, volume_depth, d_val, aperture_size, blur_ratio, target_blur_size, seed)
CASES = [
    (64, 64, 64, 3, 4e-3, -2e-3, 64, 8, 20, 0),
    (64, 48, 56, 2, 2e-3, 1e-3, 50, 1, 6, 1),
]
WAVELENGTHS = [639e-9, 532e-9, 473e-9]
PITCH = 8e-6


def zero_pad(field, size=None, method="center"):
    orig = field.shape
    while field.dim() < 4:
        field = field.unsqueeze(0)
    res = [field.shape[0], field.shape[1], 2 * field.shape[-2], 2 * field.shape[-1]] if size is None else \
        [field.shape[0], field.shape[1], size[0], size[1]]
    out = torch.zeros(res, dtype=field.dtype)
    y0, x0 = res[-2] // 2 - field.shape[-2] // 2, res[-1] // 2 - field.shape[-1] // 2
    out[:, :, y0:y0 + field.shape[-2], x0:x0 + field.shape[-1]] = field
    return out.view(out.shape[-2:]) if len(orig) == 2 else out.view(*orig[:-2], *out.shape[-2:])


def crop_center(field, size=None):
    orig = field.shape
    f = field
    while f.dim() < 4:
        f = f.unsqueeze(0)
    if size is None:
        qx, qy = f.shape[-2] // 4, f.shape[-1] // 4
        c = f[:, :, qx:qx + f.shape[-2] // 2, qy:qy + f.shape[-1] // 2]
    else:
        cx, cy, hx, hy = f.shape[-2] // 2, f.shape[-1] // 2, size[0] // 2, size[1] // 2
        c = f[:, :, cx - hx:cx + hx, cy - hy:cy + hy]
    return c.reshape(c.shape[-2:]) if len(orig) == 2 else c.reshape(*orig[:-2], *c.shape[-2:])


def custom(field, kernel, zero_padding=False, aperture=1.0):
    H = kernel * aperture
    U1 = torch.fft.fftshift(torch.fft.fft2(torch.fft.fftshift(field))) * aperture
    U2 = H * U1
    return torch.fft.ifftshift(torch.fft.ifft2(torch.fft.ifftshift(U2)))


def get_propagation_kernel(nu, nv, dx, wavelength, distance, device, propagation_type, samples=None, scale=1):
    assert propagation_type == "Bandlimited Angular Spectrum"
    return R.band_limited_angular_spectrum_kernel(nu, nv, dx, wavelength, float(distance), "cpu")


def odak_stub():
    wave = types.SimpleNamespace(
        get_propagation_kernel=get_propagation_kernel, custom=custom,
        wavenumber=lambda wl: 2 * np.pi / wl,
        generate_complex_field=lambda a, p: a * torch.cos(p) + 1j * a * torch.sin(p),
        calculate_amplitude=torch.abs, calculate_phase=torch.angle)
    tools = types.SimpleNamespace(zero_pad=zero_pad, crop_center=crop_center,
                                  circular_binary_mask=R.circular_binary_mask,
                                  generate_2d_gaussian=lambda kernel_length=[21, 21], nsigma=[3, 3], mu=[0, 0],
                                  normalize=False: R.generate_2d_gaussian(kernel_length, nsigma, mu, normalize))
    return wave, tools


def load_reference(root):
    path = os.path.join(root, "utils", "propagator.py")
    src = open(path).read()
    l1 = "from odak.learn.wave import get_propagation_kernel, custom\n"
    l2 = "from odak.learn.wave import wavenumber, generate_complex_field, calculate_amplitude, calculate_phase\n"
    l3 = "from odak.learn.tools import zero_pad, crop_center, circular_binary_mask, generate_2d_gaussian\n"
    for l in (l1, l2, l3):
        assert l in src, l
        src = src.replace(l, "")
    wave, tools = odak_stub()
    ns = {"__name__": "reference_propagator", "__file__": path}
    for k in ("get_propagation_kernel", "custom", "wavenumber", "generate_complex_field", "calculate_amplitude",
              "calculate_phase"):
        ns[k] = getattr(wave, k)
    for k in ("zero_pad", "crop_center", "circular_binary_mask", "generate_2d_gaussian"):
        ns[k] = getattr(tools, k)
    exec(compile(src, path, "exec"), ns)
    return ns["propagator"], ns["multiplane_loss_odak"]


def main(root):
    Prop, MLoss = load_reference(root)
    for ci, (S, H, W, K, vd, dval, ap, blur, bsize, seed) in enumerate(CASES):
        g = torch.Generator().manual_seed(seed)
        holo0 = torch.complex(torch.randn(3, S, S, generator=g), torch.randn(3, S, S, generator=g)) * 0.3
        image = torch.rand(3, H, W, generator=g)
        depth = torch.rand(1, H, W, generator=g)
        prop = Prop(resolution=[S, S], wavelengths=WAVELENGTHS, pixel_pitch=PITCH, number_of_frames=3,
                    number_of_depth_layers=K, volume_depth=vd, image_location_offset=dval,
                    propagation_type="Bandlimited Angular Spectrum", propagator_type="forward",
                    laser_channel_power=torch.eye(3), aperture_size=ap, aperture=None, method="conventional",
                    device="cpu")
        lf = MLoss(target_image=image, target_depth=depth, target_blur_size=bsize, number_of_planes=K,
                   blur_ratio=blur, weights=[1.0, 1.0, 1.0, 0.0], scheme="defocus", reduction="mean",
                   split_ratio=1.0, device="cpu")
        targets, masks, qdepth = lf.get_targets()
        # train.py:280-300 (the SSIM term excluded: pytorch_msssim is absent)
        holo = holo0.clone().requires_grad_(True)
        phase_map = torch.angle(holo) % (2 * np.pi)
        amplitude = torch.abs(holo)
        phase_map = phase_map - phase_map.mean()
        recon_sum = prop.reconstruct(phase_map, amplitude=amplitude, no_grad=False)
        recon = torch.sum(recon_sum, dim=0)
        loss = 0.0
        for idx, (ri, t) in enumerate(zip(recon, targets)):
            pred = crop_center(ri, size=(H, W))
            pred = torch.clamp(pred, min=0.0, max=1.0)
            loss = loss + lf(pred, t, idx)
        loss.backward()
        cplx = prop.reconstruct(phase_map.detach(), amplitude=amplitude.detach(), no_grad=True, get_complex=True)
        # identity laser powers: frame f lights channel f only, every other entry is zero
        eye = torch.eye(3).view(3, 1, 3, 1, 1)
        assert torch.all(recon_sum.detach() * (1 - eye) == 0) and torch.all(cplx * (1 - eye) == 0)
        np.savez_compressed(
            os.path.join(HERE, f"recon_{ci}.npz"),
            config=np.array([S, H, W, K, vd, dval, ap, blur, bsize], np.float64),
            wavelengths=np.array(WAVELENGTHS), pitch=np.array(PITCH),
            holo=holo0.numpy(), image=image.numpy(), depth=depth.numpy(),
            targets=targets.numpy(), masks=masks.numpy().astype(np.uint8),
            recon=recon_sum.detach().sum(0).numpy(), recon_complex=cplx.sum(0).numpy(),
            loss=np.array(float(loss.detach())), grad_holo=holo.grad.numpy())
        print(f"recon_{ci}: S={S} K={K} loss {float(loss.detach()):.6f} |grad| {holo.grad.abs().max():.3e}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CVHRF_REFERENCE_ROOT", "."))
