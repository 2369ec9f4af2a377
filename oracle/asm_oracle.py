"""CPU restatement of the band-limited angular-spectrum propagation (numpy).

TEST INFRASTRUCTURE ONLY — the checker for libcvhrf's fused FFT propagation.

Follows the CUDA path of the reference:
  * cuda_prop/python_function.py:109-163 (forward): zero_pad to [2S, 2S] (odak
    zero_pad: centred, left pad = (P - n) // 2), fft2, fftshift, transfer kernel,
    ifftshift, ifft2, crop_center to [S, S] (start = (P - S) // 2);
  * cuda_prop/python_function.py:165-218 (backward): same with the grad padded from
    [S, S] and cropped to the input size, and the conjugate transfer function;
  * cuda_prop/cuda/bandlimited_propagation_cuda.cu:29-86 / 88-147 (transfer x
    aperture) with host constants from :149-170 — k = float(2 pi / lambda) in double,
    kz^2 in double then stored to float32, kz = sqrt in float32, phase = d * kz in
    float32; FX/FY are fftshift(fftfreq(P, d=pitch)) in float32
    (python_function.py:137-142), i.e. float32(i) * float32(1 / (P * pitch)).

The FFTs run in complex128 (numpy.fft), so the oracle is more accurate than
both the reference (cuFFT fp32) and libcvhrf; parity is judged at 1e-4 relative L2.
Pinned against the reference kernels' own outputs: tests/golden/asm_*.npz.
"""
import numpy as np


def fftfreq32(n, d):
    """torch.fft.fftfreq(n, d) bit pattern: float32(i) * float32(1/(n*d))."""
    i = np.concatenate([np.arange(0, (n + 1) // 2), np.arange(-(n // 2), 0)]).astype(np.float32)
    return (i * np.float32(1.0 / (n * d))).astype(np.float32)


def transfer_shifted(P, wavelength, pitch, distance, aperture=-1.0):
    """Transfer x aperture on the fftshifted P x P grid (bandlimited_propagation_cuda.cu:44-85)."""
    wl = np.float32(wavelength)
    d = np.float32(distance)
    k = np.float32(2.0 * np.pi / np.float64(wl))
    x_size = np.float32(np.float32(pitch) * np.float32(P))
    a = np.float32(np.float32(2.0) * d * np.float32(np.float32(1.0) / x_size))
    fmax = np.float32(np.float32(1.0) / np.sqrt(np.float32(a * a + np.float32(1.0))) / wl)
    f = np.fft.fftshift(fftfreq32(P, pitch))
    FX = f[:, None].astype(np.float32)          # rows  (meshgrid 'ij')
    FY = f[None, :].astype(np.float32)          # cols
    within = (np.abs(FX) < fmax) & (np.abs(FY) < fmax)
    kk = np.float64(np.float32(k * k))
    kz2 = (kk - (2 * np.pi * FX.astype(np.float64)) ** 2 - (2 * np.pi * FY.astype(np.float64)) ** 2).astype(np.float32)
    ok = (kz2 > 0) & within
    kz = np.sqrt(np.where(ok, kz2, np.float32(0))).astype(np.float32)
    phase = (d * kz).astype(np.float32).astype(np.float64)
    T = np.where(ok, np.cos(phase) + 1j * np.sin(phase), 0.0)
    if aperture > 0:
        off = np.float32(P / 2.0 - 0.5)
        idx = np.arange(P, dtype=np.float32)
        x = (idx[None, :] - off).astype(np.float32)   # column index
        y = (idx[:, None] - off).astype(np.float32)   # row index
        m = (x * x + y * y) < np.float32(aperture) * np.float32(aperture)
        T = T * m
    return T


def zero_pad(x, P):
    H, W = x.shape
    out = np.zeros((P, P), dtype=np.complex128)
    oy, ox = (P - H) // 2, (P - W) // 2
    out[oy:oy + H, ox:ox + W] = x
    return out


def crop_center(x, H, W):
    P = x.shape[0]
    oy, ox = (P - H) // 2, (P - W) // 2
    return x[oy:oy + H, ox:ox + W]


def propagate(field, wavelength, pitch, distance, S, aperture=-1.0, out_hw=None):
    """crop(ifft2(ifftshift(T * fftshift(fft2(pad(field)))))) in complex128 -> complex64."""
    P = 2 * S
    F = np.fft.fftshift(np.fft.fft2(zero_pad(np.asarray(field, np.complex128), P)))
    F = F * transfer_shifted(P, wavelength, pitch, distance, aperture)
    y = np.fft.ifft2(np.fft.ifftshift(F))
    Ho, Wo = (S, S) if out_hw is None else out_hw
    return crop_center(y, Ho, Wo).astype(np.complex64)


def propagate_adjoint(grad, wavelength, pitch, distance, S, in_hw, aperture=-1.0):
    """Backward of propagate (python_function.py:165-218): conj transfer == distance -> -distance."""
    return propagate(grad, wavelength, pitch, -np.float32(distance), S, aperture, out_hw=in_hw)


def propagate_planes(fields, wavelengths, distances, pitch, S, aperture=-1.0):
    """model.py:1251-1272: holo[c] = sum_p propagate(fields[p, c], lambda_c, distances[p])."""
    K, C, H, W = fields.shape
    out = np.zeros((C, S, S), np.complex128)
    for p in range(K):
        for c in range(C):
            out[c] += propagate(fields[p, c], wavelengths[c], pitch, distances[p], S, aperture)
    return out.astype(np.complex64)


def rel_l2(a, b):
    a = np.asarray(a, np.complex128)
    b = np.asarray(b, np.complex128)
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))
