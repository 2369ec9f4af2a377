"""SLM -> plane reconstruction and the multiplane training loss (train.py:280-304).

CPU: the oracle (oracle/recon_oracle.py) and the product's target construction
(MultiplaneLoss) against golden vectors from the reference's own propagator /
multiplane_loss_odak code (tests/golden/recon_*.npz).  GPU: the fused reconstruction and
loss kernels against the same vectors, against torch fp32 compositions of the same
operations, and against the oracle.

Tolerances.  The transfer function's phase d kz is about 4e4 rad and odak holds it in
float32 (steps of 4e-3 rad), so two float32 evaluations of the kernel (numpy against
torch) agree to about 1e-3 relative: the oracle's reconstructions are held to 1e-3, its
loss to 1e-5.  The GPU path given the same kernels as the golden run is held to 1e-4
(fields, loss) and 1e-3 (the hologram gradient, which passes through angle() and abs()).
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import recon_oracle as O

GOLD = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "recon_*.npz")))


def _rel(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(np.asarray(b).ravel()), 1e-30))


def _case(path):
    z = np.load(path)
    S, H, W, K, vd, dval, ap, blur, bsize = z["config"]
    cfg = dict(S=int(S), H=int(H), W=int(W), K=int(K), vd=float(vd), dval=float(dval), ap=float(ap),
               blur=float(blur), bsize=int(bsize))
    dist = (torch.linspace(-cfg["vd"] / 2.0, cfg["vd"] / 2.0, cfg["K"]) + cfg["dval"]).tolist()
    return z, cfg, dist


def test_golden_fixtures_present():
    assert len(GOLD) == 2


@pytest.mark.parametrize("path", GOLD)
def test_oracle_matches_reference_reconstruction_and_loss(path):
    z, cfg, dist = _case(path)
    f = O.plane_fields(O.hologram_from_field(z["holo"]), z["wavelengths"], dist, float(z["pitch"]), cfg["ap"])
    inten = np.abs(f) ** 2
    assert _rel(inten, z["recon"]) <= 1e-3
    assert _rel(f, z["recon_complex"]) <= 1e-3
    loss, _ = O.multiplane_loss(inten, z["targets"], z["masks"])
    assert abs(loss - float(z["loss"])) <= 1e-5 * abs(float(z["loss"]))


@pytest.mark.parametrize("path", GOLD)
def test_multiplane_targets_match_reference(path):
    from complex_valued_holographic_radiance_fields_b200.reconstruction import MultiplaneLoss
    z, cfg, _ = _case(path)
    lf = MultiplaneLoss(torch.from_numpy(z["image"]), torch.from_numpy(z["depth"]), target_blur_size=cfg["bsize"],
                        number_of_planes=cfg["K"], blur_ratio=cfg["blur"], weights=[1.0, 1.0, 1.0, 0.0],
                        scheme="defocus", reduction="mean", split_ratio=1.0, device="cpu")
    t, m, _ = lf.get_targets()
    assert np.array_equal(m.numpy().astype(np.uint8), z["masks"])
    assert np.allclose(t.numpy(), z["targets"], rtol=1e-6, atol=1e-7)


# ---------------------------------------------------------------- GPU ----------
def _propagator(cfg, dist, cuda, kernels_on_cpu=True):
    from complex_valued_holographic_radiance_fields_b200 import reconstruction as R
    p = R.Propagator(resolution=[cfg["S"], cfg["S"]], wavelengths=[639e-9, 532e-9, 473e-9], pixel_pitch=8e-6,
                     number_of_frames=3, number_of_depth_layers=cfg["K"], volume_depth=cfg["vd"],
                     image_location_offset=cfg["dval"], propagator_type="forward",
                     laser_channel_power=torch.eye(3), aperture_size=cfg["ap"], device=cuda)
    if kernels_on_cpu:
        P = 2 * cfg["S"]
        ks = torch.stack([torch.stack([R.band_limited_angular_spectrum_kernel(P, P, 8e-6, wl, d, "cpu")
                                       for wl in (639e-9, 532e-9, 473e-9)]) for d in dist])
        p.set_kernels(ks)
    return p


@pytest.mark.gpu
@pytest.mark.parametrize("path", GOLD)
def test_gpu_reconstruct_matches_reference(cuda, path):
    z, cfg, dist = _case(path)
    p = _propagator(cfg, dist, cuda)
    holo = torch.from_numpy(z["holo"]).to(cuda)
    phase = torch.remainder(torch.angle(holo), 2 * np.pi)
    phase = phase - phase.mean()
    amp = torch.abs(holo)
    r = p.reconstruct(phase, amplitude=amp)
    assert r.shape == (3, cfg["K"], 3, cfg["S"], cfg["S"])
    assert _rel(r.sum(0).cpu().numpy(), z["recon"]) <= 1e-4
    c = p.reconstruct(phase, amplitude=amp, get_complex=True)
    assert _rel(c.sum(0).cpu().numpy(), z["recon_complex"]) <= 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("path", GOLD)
def test_gpu_training_loss_matches_reference(cuda, path):
    from complex_valued_holographic_radiance_fields_b200 import reconstruction as R
    z, cfg, dist = _case(path)
    p = _propagator(cfg, dist, cuda)
    holo = torch.from_numpy(z["holo"]).to(cuda).requires_grad_(True)
    t = torch.from_numpy(z["targets"]).to(cuda)
    m = torch.from_numpy(z["masks"].astype(np.float32)).to(cuda)
    loss = R.hologram_training_loss(p, holo, t, m, ssim=False)
    loss.backward()
    assert abs(float(loss) - float(z["loss"])) <= 1e-4 * float(z["loss"])
    assert _rel(holo.grad.cpu().numpy(), z["grad_holo"]) <= 1e-3


def _torch_ssim_valid(x, y):
    """pytorch_msssim's SSIM restated with torch conv2d (valid filtering), fp32."""
    c = torch.arange(11, dtype=torch.float32, device=x.device) - 5
    g = torch.exp(-(c ** 2) / (2 * 1.5 ** 2))
    g = g / g.sum()
    C = x.shape[0]

    def filt(a):
        a = a.unsqueeze(0)
        a = torch.nn.functional.conv2d(a, g.view(1, 1, 1, 11).expand(C, 1, 1, 11), groups=C)
        return torch.nn.functional.conv2d(a, g.view(1, 1, 11, 1).expand(C, 1, 11, 1), groups=C)[0]

    mu1, mu2 = filt(x), filt(y)
    s11, s22, s12 = filt(x * x) - mu1 ** 2, filt(y * y) - mu2 ** 2, filt(x * y) - mu1 * mu2
    cs = (2 * s12 + 0.03 ** 2) / (s11 + s22 + 0.03 ** 2)
    return (((2 * mu1 * mu2 + 0.01 ** 2) / (mu1 ** 2 + mu2 ** 2 + 0.01 ** 2)) * cs).mean()


@pytest.mark.gpu
@pytest.mark.parametrize("K,C,S,H,W,scale", [(3, 3, 64, 64, 64, (1.0, 1.0, 1.0)), (2, 3, 128, 96, 112, (1.0, 2.0, 0.5)),
                                            (3, 1, 256, 200, 256, (1.5,))])
def test_gpu_fused_loss_matches_torch(cuda, K, C, S, H, W, scale):
    from complex_valued_holographic_radiance_fields_b200 import reconstruction as R
    g = torch.Generator(device=cuda).manual_seed(K * 100 + S)
    f = (torch.randn(K, C, S, S, 2, generator=g, device=cuda) * 0.6)
    f = torch.view_as_complex(f).contiguous()
    t = torch.rand(K, C, H, W, generator=g, device=cuda)
    m = (torch.rand(K, C, H, W, generator=g, device=cuda) > 0.5).float()
    w = (1.0, 0.7, 1.3)
    a = f.clone().requires_grad_(True)
    la = R.reconstruction_loss(a, t, m, w, scale, ssim=True)
    la.backward()
    b = f.clone().requires_grad_(True)
    sc = torch.tensor(scale, device=cuda).view(1, C, 1, 1)
    inten = sc * (b.real ** 2 + b.imag ** 2)
    oy, ox = S // 2 - H // 2, S // 2 - W // 2
    x = torch.clamp(inten[:, :, oy:oy + H, ox:ox + W], 0.0, 1.0)
    mse = torch.nn.functional.mse_loss
    lb = 0.0
    for p in range(K):
        lb = lb + w[0] * mse(x[p], t[p]) + w[1] * mse(x[p] * m[p], t[p] * m[p]) + w[2] * mse(x[p] * t[p], t[p] * t[p])
        lb = lb + 0.025 * (1 - _torch_ssim_valid(x[p], t[p])) * 0.2
    lb.backward()
    assert abs(float(la) - float(lb)) <= 1e-5 * abs(float(lb))
    assert _rel(a.grad.cpu().numpy(), b.grad.cpu().numpy()) <= 1e-4


@pytest.mark.gpu
def test_gpu_msssim_matches_oracle(cuda):
    from complex_valued_holographic_radiance_fields_b200.reconstruction import msssim_ssim
    g = torch.Generator().manual_seed(4)
    x = torch.rand(3, 70, 90, generator=g)
    y = (x + 0.1 * torch.randn(3, 70, 90, generator=g)).clamp(0, 1)
    s = float(msssim_ssim(x.to(cuda), y.to(cuda)))
    assert abs(s - O.ssim_msssim(x.numpy(), y.numpy())) <= 1e-5


@pytest.mark.gpu
def test_gpu_reconstruct_general_powers_matches_torch(cuda):
    """A non-diagonal laser power matrix (every frame lights every channel, method
    'multi-color'): each frame propagated with its own phase, checked against torch.fft."""
    from complex_valued_holographic_radiance_fields_b200 import reconstruction as R
    S, K = 64, 2
    p = R.Propagator(resolution=[S, S], wavelengths=[639e-9, 532e-9, 473e-9], number_of_frames=3,
                     number_of_depth_layers=K, volume_depth=2e-3, image_location_offset=1e-3,
                     propagator_type="back and forth", laser_channel_power=torch.rand(3, 3) + 0.2,
                     method="multi-color", aperture_size=40, device=cuda)
    assert not p.diagonal_power()
    g = torch.Generator().manual_seed(2)
    phase = (torch.rand(3, S, S, generator=g) * 6.28).to(cuda)
    amp = torch.rand(3, S, S, generator=g).to(cuda)
    r = p.reconstruct(phase, amplitude=amp)
    p.table()
    H = p.kernels * p.aperture                                  # K x C x 2S x 2S centred
    power = p.get_laser_powers().to(cuda)
    ref = torch.zeros_like(r)
    for f in range(3):
        for c in range(3):
            u = torch.zeros(2 * S, 2 * S, dtype=torch.complex64, device=cuda)
            u[S // 2:S // 2 + S, S // 2:S // 2 + S] = power[f, c] * amp[c] * torch.exp(1j * phase[f])
            for d in range(K):
                o = torch.fft.ifft2(torch.fft.ifftshift(H[d, c]) * torch.fft.fft2(u))
                ref[f, d, c] = o[S // 2:S // 2 + S, S // 2:S // 2 + S].abs() ** 2
    assert _rel(r.cpu().numpy(), ref.cpu().numpy()) <= 1e-4


@pytest.mark.gpu
def test_trainer_multiplane_graph_matches_eager(cuda):
    """The training step with the multiplane reconstruction loss: finite, and the CUDA-graph
    iteration equal to the eager one bit for bit."""
    from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer
    kw = dict(N=20000, W=128, H=128, K=3, device=cuda, seed=5, loss="multiplane")
    a, b = HoloTrainer(**kw), HoloTrainer(**kw)
    assert a.target.shape == (2, 3, 3, 128, 128)
    b.capture(headroom=1.5, warmup=2)
    for _ in range(3):
        a.step()
    for _ in range(3):
        la, lb = a.step(), b.replay()
        torch.cuda.synchronize()
        assert torch.isfinite(la)
        assert torch.equal(la, lb)
    assert not b.graph_overflowed()
    for k in a.params:
        assert torch.equal(a.params[k], b.params[k]), k


@pytest.mark.gpu
@pytest.mark.parametrize("C,S,scale", [(3, 64, (1.0, 1.0, 1.0)), (3, 200, (1.0, 0.8, 1.2)), (1, 128, (0.5,))])
def test_gpu_hologram_field_matches_torch(cuda, C, S, scale):
    """The fused hologram -> SLM field step against train.py:280-283's torch ops (with
    exact zeros in the hologram, where both give a zero gradient)."""
    from complex_valued_holographic_radiance_fields_b200.reconstruction import HologramFieldFunction
    g = torch.Generator(device=cuda).manual_seed(C * 7 + S)
    h = torch.view_as_complex(torch.randn(C, S, S, 2, generator=g, device=cuda)).contiguous()
    h[0, :3, :5] = 0
    up = torch.view_as_complex(torch.randn(C, S, S, 2, generator=g, device=cuda)).contiguous()
    a = h.clone().requires_grad_(True)
    fa = HologramFieldFunction.apply(a, list(scale))
    fa.backward(up)
    b = h.clone().requires_grad_(True)
    phase = torch.remainder(torch.angle(b), 2 * np.pi)
    phase = phase - phase.mean()
    sc = torch.tensor(scale, device=cuda).view(C, 1, 1)
    fb = torch.polar(torch.abs(b), phase * sc)
    fb.backward(up)
    assert _rel(fa.detach().cpu().numpy(), fb.detach().cpu().numpy()) <= 1e-5
    gb = torch.nan_to_num(b.grad)
    assert _rel(a.grad.cpu().numpy(), gb.cpu().numpy()) <= 1e-4
