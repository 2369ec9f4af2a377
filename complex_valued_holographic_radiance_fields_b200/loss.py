"""L2 intensity loss of the training iteration as two libcvhrf kernels.

``intensity_l2_loss(holo, target)`` = mean((|holo|^2 - target)^2), the loss of
train.py's iteration, which the reference evaluates with torch elementwise ops
(holo.real**2 + holo.imag**2 - target, square, mean: about ten launches forward and
backward).  Here the forward is one deterministic reduction launch and the backward
one elementwise launch; the loss stays on the device.
"""
import ctypes
import threading

import torch

from . import _lib
from .profiling import timed

_ws = {}
_ws_lock = threading.Lock()


def _workspace(device):
    """Per-device workspace (block partials + completion counter), zeroed once."""
    key = torch.device(device)
    with _ws_lock:
        w = _ws.get(key)
        if w is None:
            L = _lib.lib()
            nbytes = L.cvhrf_intensity_loss_workspace_bytes(0)
            w = torch.empty(nbytes, dtype=torch.uint8, device=device)
            _lib.check(L.cvhrf_intensity_loss_init_workspace(ctypes.c_void_p(w.data_ptr()), nbytes,
                                                             ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)),
                       "cvhrf_intensity_loss_init_workspace")
            _ws[key] = w
    return w


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


class IntensityL2Loss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, holo, target):
        if holo.dtype != torch.complex64 or target.dtype != torch.float32:
            raise TypeError("holo must be complex64 and target float32")
        if holo.shape != target.shape:
            raise ValueError("holo and target must have the same shape")
        holo = holo.contiguous()
        target = target.contiguous()
        ws = _workspace(holo.device)
        loss = torch.empty((), dtype=torch.float32, device=holo.device)
        st = ctypes.c_void_p(torch.cuda.current_stream(holo.device).cuda_stream)
        with timed("loss"):
            _lib.check(_lib.lib().cvhrf_intensity_loss(_p(holo), _p(target), holo.numel(), _p(loss), _p(ws), ws.numel(),
                                                       st), "cvhrf_intensity_loss")
        ctx.save_for_backward(holo, target)
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        holo, target = ctx.saved_tensors
        g = grad_loss.to(torch.float32).contiguous()
        grad = torch.empty_like(holo)
        st = ctypes.c_void_p(torch.cuda.current_stream(holo.device).cuda_stream)
        with timed("loss_backward"):
            _lib.check(_lib.lib().cvhrf_intensity_loss_backward(_p(holo), _p(target), holo.numel(), _p(g), _p(grad), st),
                       "cvhrf_intensity_loss_backward")
        return grad, None


def intensity_l2_loss(holo, target):
    """mean((|holo|^2 - target)^2) with the gradient to `holo` (complex64 vs float32, same shape)."""
    return IntensityL2Loss.apply(holo, target)
