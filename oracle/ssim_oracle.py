"""CPU restatement of the reference's fused SSIM (test infrastructure only).

Follows cov3d_cuda/conv.cu: fusedssimCUDA :935-1008 (statistics with an 11 x 11 Gaussian
window, sigma 1.5, the 1-D weights G_00..G_10 of :8-18; zero padding, get_pix_value
:148-154; the SSIM expression :987-995) and the gradient of that map with respect to img1
(fusedssim_backwardCUDA :1011-1136 computes the same three terms, :1085-1121).  Written
with torch conv2d in float64 on the CPU, autograd giving the gradient.
"""
import math

import torch
import torch.nn.functional as F


def window(dtype=torch.float64):
    g = torch.tensor([math.exp(-((i - 5) ** 2) / (2 * 1.5 ** 2)) for i in range(11)], dtype=dtype)
    g = g / g.sum()
    return torch.outer(g, g)


def ssim_map(img1, img2, C1=0.01 ** 2, C2=0.03 ** 2):
    """img1, img2: C x H x W tensors (any float dtype; computed in float64)."""
    x = img1.double().unsqueeze(1)
    y = img2.double().unsqueeze(1)
    w = window().view(1, 1, 11, 11)
    conv = lambda t: F.conv2d(t, w, padding=5)  # noqa: E731
    mu1, mu2 = conv(x), conv(y)
    s11 = conv(x * x) - mu1 * mu1
    s22 = conv(y * y) - mu2 * mu2
    s12 = conv(x * y) - mu1 * mu2
    m = ((2 * mu1 * mu2 + C1) * (2 * s12 + C2)) / ((mu1 * mu1 + mu2 * mu2 + C1) * (s11 + s22 + C2))
    return m.squeeze(1)


def ssim_map_and_grad(img1, img2, dmap, C1=0.01 ** 2, C2=0.03 ** 2):
    x = img1.detach().double().cpu().requires_grad_(True)
    m = ssim_map(x, img2.detach().cpu(), C1, C2)
    m.backward(dmap.detach().double().cpu())
    return m.detach(), x.grad
