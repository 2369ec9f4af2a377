"""Fused SSIM (the ``FusedSSIMMap`` / ``fast_ssim`` surface of cov3d_cuda/python_import.py:43-57,
449-454, used by the training loss's SSIM term, utils/data_utils.py:124-157).

``FusedSSIMMap.apply(C1, C2, img1, img2)`` returns the SSIM map (same shape as the images,
C x H x W); its backward returns the gradient for img1 only, as the reference's does.
``fast_ssim(img1, img2)`` is the mean of that map with the reference's C1 = 0.01^2,
C2 = 0.03^2, computed in the same launch as the map statistics.
"""
import ctypes

import torch

from . import _lib
from .profiling import timed

C1 = 0.01 ** 2
C2 = 0.03 ** 2


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _st(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _check(img1, img2):
    if img1.dim() == 4 and img1.shape[0] == 1:
        img1, img2 = img1[0], img2[0]
    if img1.dim() != 3 or img1.shape != img2.shape:
        raise ValueError("images must be C x H x W (or 1 x C x H x W) with equal shapes")
    if img1.dtype != torch.float32 or img2.dtype != torch.float32 or not img1.is_cuda:
        raise TypeError("images must be float32 CUDA tensors")
    return img1.contiguous(), img2.contiguous()


def _forward(img1, img2, c1, c2, want_map):
    C, H, W = img1.shape
    L = _lib.lib()
    ws = torch.empty(L.cvhrf_ssim_workspace_bytes(C, H, W), dtype=torch.uint8, device=img1.device)
    m = torch.empty_like(img1) if want_map else None
    mean = None if want_map else torch.empty((), dtype=torch.float32, device=img1.device)
    with timed("ssim"):
        _lib.check(L.cvhrf_ssim_forward(_p(img1), _p(img2), C, H, W, float(c1), float(c2), _p(m), _p(mean), _p(ws),
                                        ws.numel(), _st(img1)), "cvhrf_ssim_forward")
    return (m if want_map else mean), ws


def _backward(img1, img2, ws, dmap=None, dmean=None):
    C, H, W = img1.shape
    grad = torch.empty_like(img1)
    with timed("ssim_backward"):
        _lib.check(_lib.lib().cvhrf_ssim_backward(_p(img1), _p(img2), C, H, W, _p(dmap), _p(dmean), _p(grad), _p(ws),
                                                  ws.numel(), _st(img1)), "cvhrf_ssim_backward")
    return grad


class FusedSSIMMap(torch.autograd.Function):
    """python_import.py:43-57: forward(C1, C2, img1, img2) -> map; backward -> (None, None, d img1, None)."""

    @staticmethod
    def forward(ctx, c1, c2, img1, img2):
        shape = img1.shape
        a, b = _check(img1, img2)
        m, ws = _forward(a, b, c1, c2, True)
        ctx.save_for_backward(a, b)
        ctx.ws, ctx.shape = ws, shape
        return m.view(shape)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        grad = _backward(a, b, ctx.ws, dmap=g.reshape(a.shape).contiguous().float())
        return None, None, grad.view(ctx.shape), None


class _FastSSIM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img1, img2):
        shape = img1.shape
        a, b = _check(img1, img2)
        mean, ws = _forward(a, b, C1, C2, False)
        ctx.save_for_backward(a, b)
        ctx.ws, ctx.shape = ws, shape
        return mean

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        grad = _backward(a, b, ctx.ws, dmean=g.float().contiguous())
        return grad.view(ctx.shape), None


def fast_ssim(img1, img2):
    """python_import.py:452-454: mean SSIM of img1 against img2 (gradient to img1 only)."""
    return _FastSSIM.apply(img1, img2)
