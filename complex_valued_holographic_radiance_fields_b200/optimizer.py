"""Optimizers of the reference's ``utils/optimizer.py``: sparse Adam over visible Gaussians
(``SparseGaussianAdam`` / ``adamUpdate``) and Adan (``Adan``, the optimizer the training
script builds, optimizer.py:65), each as one fused libcvhrf launch per step.

* ``SparseGaussianAdam(params, lr, eps)`` with ``.step(visible_chunk)`` mirrors
  utils/optimizer.py:174-265: one tensor per param group, lazily created
  ``exp_avg``/``exp_avg_sq``, betas fixed at 0.9/0.999, no bias correction, 1-D
  parameters updated densely, 2-D/3-D parameters only at the visible rows.  All
  groups are updated by ONE fused kernel launch (cvhrf_sparse_adam).
* ``sparse_adam_update(param, grad, exp_avg, exp_avg_sq, visible_chunk, lr, b1, b2, eps)``
  mirrors python_import.py:457-460: ``grad`` is the compacted (B, V, D) gradient of
  the reference's adamUpdate (conv.cu:1230-1246).
"""
import ctypes
import math

import torch

from . import _lib
from .profiling import timed


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _launch(groups, visible, b1, b2, device):
    if not groups:
        return
    arr = (_lib.AdamGroup * len(groups))(*groups)
    V = 0 if visible is None else visible.numel()
    vp = ctypes.c_void_p(visible.data_ptr()) if V > 0 else ctypes.c_void_p(0)
    _lib.check(_lib.lib().cvhrf_sparse_adam(arr, len(groups), vp, V, float(b1), float(b2),
                                            ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)),
               "cvhrf_sparse_adam")


def _group(param, grad, m, v, N, D, dense, lr, eps):
    return _lib.AdamGroup(param.data_ptr(), grad.data_ptr(), m.data_ptr(), v.data_ptr(), int(N), int(D),
                          int(dense), float(lr), float(eps))


class SparseGaussianAdam(torch.optim.Adam):
    """utils/optimizer.py:174-265."""

    def __init__(self, params, lr, eps):
        super().__init__(params=params, lr=lr, eps=eps)

    @torch.no_grad()
    def step(self, visible_chunk=None, row_mask=None):
        """Update the rows listed in `visible_chunk` (int64 row indices, as the reference)
        or, alternatively, the rows where `row_mask` (uint8/bool, one entry per row) is set.
        1-D parameters are updated densely.  With indices and none visible nothing is
        updated (optimizer.py:197-199); a mask is used as given (no host synchronisation)."""
        groups, keep = [], []
        if row_mask is None:
            vis = visible_chunk.to(torch.int64).contiguous()
            if vis.numel() == 0:
                vis = None
        device = None
        for group in self.param_groups:
            assert len(group["params"]) == 1, "more than one tensor in group"
            param = group["params"][0]
            if param.grad is None:
                continue
            state = self.state[param]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0, dtype=torch.float32)
                state["exp_avg"] = torch.zeros_like(param, memory_format=torch.preserve_format)
                state["exp_avg_sq"] = torch.zeros_like(param, memory_format=torch.preserve_format)
            if row_mask is None and vis is None:
                continue
            if not (param.is_cuda and param.dtype == torch.float32 and param.is_contiguous()):
                raise RuntimeError("SparseGaussianAdam needs contiguous float32 CUDA parameters")
            grad = param.grad.contiguous()
            keep.append(grad)
            if param.dim() == 1:
                groups.append(_group(param, grad, state["exp_avg"], state["exp_avg_sq"], param.shape[0], 1, 1,
                                     group["lr"], group["eps"]))
            elif param.dim() == 2:
                groups.append(_group(param, grad, state["exp_avg"], state["exp_avg_sq"], param.shape[0],
                                     param.shape[1], 0, group["lr"], group["eps"]))
            elif param.dim() == 3:  # (B, N, D): one group per leading slice
                B, N, D = param.shape
                for b in range(B):
                    groups.append(_group(param[b], grad[b], state["exp_avg"][b], state["exp_avg_sq"][b], N, D, 0,
                                         group["lr"], group["eps"]))
            else:
                raise NotImplementedError("parameters with more than 3 dimensions")
            device = param.device
        if groups:
            with timed("sparse_adam"):
                n_rows = max(g.N for g in groups)
                L = _lib.lib()
                st = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
                if row_mask is None:
                    mask = self._mask_buffer(n_rows, device)
                    _lib.check(L.cvhrf_rows_to_mask(ctypes.c_void_p(vis.data_ptr()), vis.numel(),
                                                    ctypes.c_void_p(mask.data_ptr()), n_rows, st),
                               "cvhrf_rows_to_mask")
                else:
                    mask = row_mask.to(torch.uint8).contiguous()
                for i in range(0, len(groups), 16):
                    arr = (_lib.AdamGroup * len(groups[i:i + 16]))(*groups[i:i + 16])
                    _lib.check(L.cvhrf_sparse_adam_masked(arr, len(groups[i:i + 16]), ctypes.c_void_p(mask.data_ptr()),
                                                          mask.numel(), 0.9, 0.999, st), "cvhrf_sparse_adam_masked")

    def _mask_buffer(self, n, device):
        buf = getattr(self, "_row_mask_buf", None)
        if buf is None or buf.numel() < n or buf.device != device:
            buf = self._row_mask_buf = torch.empty(n, dtype=torch.uint8, device=device)
        return buf[:n]


def sparse_adam_update(param, grad, exp_avg, exp_avg_sq, visible_chunk, lr, b1, b2, eps):
    """python_import.py:457-460 / conv.cu:1230-1246: param/exp_avg/exp_avg_sq (B, N, D) in place,
    grad (B, V, D) compacted to the visible rows."""
    B, N, D = param.shape
    V = visible_chunk.numel()
    vis = visible_chunk.to(torch.int64).contiguous()
    # the kernel reads dense rows; scatter the compacted rows into a dense view
    dense = torch.zeros_like(param)
    if V > 0:
        dense[:, vis] = grad.reshape(B, V, D)
    groups = [_group(param[b], dense[b], exp_avg[b], exp_avg_sq[b], N, D, 0, lr, eps) for b in range(B)]
    _launch(groups, vis, b1, b2, param.device)


class Adan(torch.optim.Optimizer):
    """utils/optimizer.py:288-484 with the same constructor, validation, state and step;
    the update runs as one fused launch over all groups (cvhrf_adan) instead of the
    foreach / single-tensor paths, and the optional global-norm clip factor is computed on
    the device (the reference reads it back with .item()).  ``foreach`` and ``fused`` are
    accepted for signature compatibility; they select nothing here.  As in the reference,
    the clip uses the eps of the last parameter group."""

    def __init__(self, params, lr=1e-3, betas=(0.98, 0.92, 0.99), eps=1e-8, weight_decay=0.0, max_grad_norm=0.0,
                 no_prox=False, foreach: bool = True, fused: bool = False):
        if not 0.0 <= max_grad_norm:
            raise ValueError('Invalid Max grad norm: {}'.format(max_grad_norm))
        if not 0.0 <= lr:
            raise ValueError('Invalid learning rate: {}'.format(lr))
        if not 0.0 <= eps:
            raise ValueError('Invalid epsilon value: {}'.format(eps))
        for i in range(3):
            if not 0.0 <= betas[i] < 1.0:
                raise ValueError('Invalid beta parameter at index {}: {}'.format(i, betas[i]))
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, max_grad_norm=max_grad_norm,
                        no_prox=no_prox, foreach=foreach, fused=fused)
        super().__init__(params, defaults)

    def __setstate__(self, state):
        super().__setstate__(state)
        for group in self.param_groups:
            group.setdefault('no_prox', False)

    @torch.no_grad()
    def restart_opt(self):
        for group in self.param_groups:
            group['step'] = 0
            for p in group['params']:
                if p.requires_grad:
                    state = self.state[p]
                    state['exp_avg'] = torch.zeros_like(p)
                    state['exp_avg_sq'] = torch.zeros_like(p)
                    state['exp_avg_diff'] = torch.zeros_like(p)

    def _clip_workspace(self, device):
        ws = getattr(self, "_clip_ws", None)
        if ws is None or ws.device != device:
            L = _lib.lib()
            ws = torch.empty(L.cvhrf_adan_clip_workspace_bytes(), dtype=torch.uint8, device=device)
            _lib.check(L.cvhrf_adan_clip_init_workspace(ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                                        _stream(ws)), "cvhrf_adan_clip_init_workspace")
            self._clip_ws = ws
            self._clip = torch.ones((), dtype=torch.float32, device=device)
        return ws

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        groups, keep, device = [], [], None
        for group in self.param_groups:
            b1, b2, b3 = group['betas']
            group['step'] = group['step'] + 1 if 'step' in group else 1
            t = group['step']
            for p in group['params']:
                if p.grad is None:
                    continue
                if not (p.is_cuda and p.dtype == torch.float32 and p.is_contiguous() and p.grad.is_contiguous()):
                    raise RuntimeError("Adan needs contiguous float32 CUDA parameters and gradients")
                state = self.state[p]
                if len(state) == 0:
                    state['exp_avg'] = torch.zeros_like(p)
                    state['exp_avg_sq'] = torch.zeros_like(p)
                    state['exp_avg_diff'] = torch.zeros_like(p)
                first = 'neg_pre_grad' not in state or t == 1
                if 'neg_pre_grad' not in state:
                    state['neg_pre_grad'] = torch.empty_like(p)
                keep.append(p)
                device = p.device
                lr, wd = float(group['lr']), float(group['weight_decay'])
                groups.append(_lib.AdanGroup(
                    p.data_ptr(), p.grad.data_ptr(), state['exp_avg'].data_ptr(), state['exp_avg_sq'].data_ptr(),
                    state['exp_avg_diff'].data_ptr(), state['neg_pre_grad'].data_ptr(), p.numel(),
                    b1, b2, b3, 1 - b1, 1 - b2, 1 - b3, math.sqrt(1.0 - b3 ** t), float(group['eps']),
                    lr / (1.0 - b1 ** t), lr * b2 / (1.0 - b2 ** t),
                    1 - lr * wd if group['no_prox'] else 1 + lr * wd, int(bool(group['no_prox'])), int(first)))
        if not groups:
            return loss
        if len(groups) > 16:
            raise NotImplementedError("more than 16 parameter tensors")
        L = _lib.lib()
        arr = (_lib.AdanGroup * len(groups))(*groups)
        st = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        clip = ctypes.c_void_p(0)
        if self.defaults['max_grad_norm'] > 0:
            ws = self._clip_workspace(device)
            _lib.check(L.cvhrf_adan_clip_factor(arr, len(groups), float(self.defaults['max_grad_norm']),
                                                float(self.param_groups[-1]['eps']),
                                                ctypes.c_void_p(self._clip.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                                ws.numel(), st), "cvhrf_adan_clip_factor")
            clip = ctypes.c_void_p(self._clip.data_ptr())
        with timed("adan"):
            _lib.check(L.cvhrf_adan(arr, len(groups), clip, st), "cvhrf_adan")
        return loss
