"""CPU restatement of the reconstruction / multiplane-loss path (test infrastructure
only: the checker of libcvhrf's transfer-table upload, fused reconstruction and
cvhrf_multiplane_loss, never part of the product path).

Follows:
  * utils/propagator.py:548-636 (_reconstruct_impl) with train.py:878's identity laser
    powers: channel c of the frame-summed reconstruction at depth d is
    |crop(IFFT2(H_{d,c} A FFT2(pad(amplitude_c exp(i phase_c)))))|^2;
  * odak 0.2.6's band-limited angular-spectrum kernel and circular aperture (absent here;
    restated from the published algorithm, float32 like odak);
  * train.py:293-300 and multiplane_loss_odak.__call__ (utils/propagator.py:138-169): per
    plane crop_center, clamp to [0, 1], w0 MSE + w1 masked MSE + w2 target-weighted MSE;
  * pytorch_msssim's SSIM (absent here; 11-tap Gaussian window sigma 1.5, valid
    filtering, C1 = 0.01^2, C2 = 0.03^2) for GaussianLoss (utils/data_utils.py:124-157).
numpy; FFTs in complex128.  Pinned to tests/golden/recon_*.npz (the reference's own
propagator / multiplane_loss_odak code and train.py's loss loop, run with odak's helpers
restated, tests/golden/make_recon_golden.py): the reference's own code is pinned, odak
and pytorch_msssim are not.
"""
import numpy as np

f32 = np.float32


def blasm_kernel(n, dx, wavelength, distance):
    """Centred n x n band-limited angular-spectrum transfer function (odak's grid)."""
    x = dx * float(n)
    f = np.linspace(-1 / (2 * dx) + 0.5 / (2 * x), 1 / (2 * dx) - 0.5 / (2 * x), n).astype(f32)
    FY, FX = np.meshgrid(f, f, indexing="ij")
    hh = f32(2 * np.pi) * np.sqrt(f32(1 / wavelength ** 2) - (FX * FX + FY * FY))
    d = f32(distance)
    h_exp = (hh * d).astype(f32)
    fmax = f32(1 / np.sqrt((2 * d * (1 / x)) ** 2 + 1) / wavelength)
    filt = ((np.abs(FX) < fmax) & (np.abs(FY) < fmax)).astype(f32)
    return filt * np.cos(h_exp) + 1j * filt * np.sin(h_exp)


def circular_mask(p, r):
    g = np.linspace(-p / 2.0, p / 2.0, p).astype(f32)
    X, Y = np.meshgrid(g, g, indexing="ij")
    return (np.sqrt(X * X + Y * Y) < r).astype(f32)


def propagate(field, H):
    """crop_S(IFFT2(ifftshift(H) FFT2(pad_2S(field)))) for an S x S field, H centred 2S x 2S."""
    S = field.shape[-1]
    P = 2 * S
    pad = np.zeros((P, P), np.complex128)
    o = P // 2 - S // 2
    pad[o:o + S, o:o + S] = field
    out = np.fft.ifft2(np.fft.ifftshift(H) * np.fft.fft2(pad))
    q = P // 4
    return out[q:q + S, q:q + S]


def plane_fields(holo, wavelengths, distances, pitch, aperture_size):
    """K x C x S x S fields of the reconstruction of holo (C x S x S complex): each channel
    propagated to each depth with the odak kernel times the circular aperture."""
    C, S, _ = holo.shape
    A = circular_mask(2 * S, aperture_size)
    out = np.zeros((len(distances), C, S, S), np.complex128)
    for p, d in enumerate(distances):
        for c in range(C):
            out[p, c] = propagate(holo[c], blasm_kernel(2 * S, pitch, wavelengths[c], d) * A)
    return out


def hologram_from_field(holo):
    """train.py:280-283 and _reconstruct_impl: amplitude |h| and phase (angle(h) mod 2 pi)
    minus its mean, recombined."""
    phase = np.mod(np.angle(holo), 2 * np.pi)
    phase = phase - phase.mean()
    return np.abs(holo) * np.exp(1j * phase)


def crop_center(x, H, W):
    S = x.shape[-1]
    return x[..., S // 2 - H // 2:S // 2 + H // 2, S // 2 - W // 2:S // 2 + W // 2]


def multiplane_loss(intensity, targets, masks, weights=(1.0, 1.0, 1.0)):
    """Sum over planes of w0 MSE(x, t) + w1 MSE(x m, t m) + w2 MSE(x t, t t), x the clamped
    centred crop of the plane intensities (K x C x S x S)."""
    K, C, H, W = targets.shape
    x = np.clip(crop_center(intensity, H, W), 0.0, 1.0)
    t, m = targets.astype(np.float64), masks.astype(np.float64)
    loss = 0.0
    for p in range(K):
        loss += weights[0] * np.mean((x[p] - t[p]) ** 2)
        loss += weights[1] * np.mean((x[p] * m[p] - t[p] * m[p]) ** 2)
        loss += weights[2] * np.mean((x[p] * t[p] - t[p] * t[p]) ** 2)
    return loss, x


def _gauss_1d(size=11, sigma=1.5):
    c = np.arange(size, dtype=np.float64) - size // 2
    g = np.exp(-(c ** 2) / (2 * sigma ** 2))
    return g / g.sum()


def _valid_filter(img, g):
    n = len(g)
    H, W = img.shape
    t = sum(g[k] * img[:, k:W - n + 1 + k] for k in range(n))
    return sum(g[k] * t[k:H - n + 1 + k, :] for k in range(n))


def ssim_msssim(x, y, c1=0.01 ** 2, c2=0.03 ** 2):
    """pytorch_msssim SSIM(data_range=1, size_average=True) of C x H x W images."""
    g = _gauss_1d()
    vals = []
    for a, b in zip(x.astype(np.float64), y.astype(np.float64)):
        mu1, mu2 = _valid_filter(a, g), _valid_filter(b, g)
        s11 = _valid_filter(a * a, g) - mu1 * mu1
        s22 = _valid_filter(b * b, g) - mu2 * mu2
        s12 = _valid_filter(a * b, g) - mu1 * mu2
        cs = (2 * s12 + c2) / (s11 + s22 + c2)
        vals.append((((2 * mu1 * mu2 + c1) / (mu1 * mu1 + mu2 * mu2 + c1)) * cs).mean())
    return float(np.mean(vals))
