"""Band-limited angular-spectrum propagation (the ``cuda_prop`` operator surface).

Mirrors ``cuda_prop/python_function.py``:

* ``BandlimitedPropagationFunction.apply(field, wavelength, pixel_pitch, distance,
  size, aperture_size=-1.0)`` (python_function.py:109-218) — one field, forward is
  ``crop_S(IFFT2(H * A * FFT2(pad_2S(field))))`` and backward its exact adjoint.
* ``BandlimitedPropagation(field, wavelength, pixel_pitch, distance, size, use_cuda,
  aperture_size=-1.0)`` (python_function.py:220-226).
* ``PlanePropagationFunction`` — the K-plane x C-channel loop of model.py:1251-1272
  (``hologram = sum_p stack_c BandlimitedPropagation(field[p, c], lambda_c, ..., -d_p)``)
  as one fused operator.

All arithmetic runs in ``libcvhrf.so`` (hand-written sm_100a FFT fused with the
transfer function); torch only provides device memory and the current stream.
"""
import ctypes
import threading

import torch

from . import _lib
from .profiling import timed

_plans = {}
_plans_lock = threading.Lock()


def get_plan(S, device):
    """Twiddle/digit-reversal tables for padded size 2S on `device` (created once)."""
    dev = torch.device(device)
    key = (int(S), dev.index if dev.index is not None else torch.cuda.current_device())
    with _plans_lock:
        p = _plans.get(key)
        if p is None:
            L = _lib.lib()
            h = ctypes.c_void_p()
            with torch.cuda.device(key[1]):
                _lib.check(L.cvhrf_asm_plan_create(int(S), ctypes.byref(h)), f"asm plan (S={S})")
            p = _plans[key] = h
    return p


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _square_size(size):
    if isinstance(size, int):
        return int(size)
    size = [int(s) for s in size]
    if len(size) != 2 or size[0] != size[1]:
        # The reference kernel indexes idy*nx+idx (bandlimited_propagation_cuda.cu:54),
        # which is only correct for square padded grids; all its call sites pass [S, S].
        raise ValueError(f"size must be [S, S] (square), got {size}")
    return size[0]


def _check_field(x, name):
    if not x.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (libcvhrf has no CPU path)")
    if x.dtype != torch.complex64:
        raise TypeError(f"{name} must be complex64, got {x.dtype}")
    return x.contiguous()


def _scalar(v):
    return float(v.item()) if torch.is_tensor(v) else float(v)


def _workspace(S, in_items, Hi, out_items, Ho, device):
    nbytes = _lib.lib().cvhrf_asm_workspace_bytes(S, in_items, Hi, 0, out_items, Ho, 0)
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def propagate(field, wavelength, pixel_pitch, distance, S, aperture_size=-1.0, out_hw=None, out=None,
              accumulate=False, use_table=True):
    """Single propagation: field (Hi, Wi) complex64 -> out (Ho, Wo) (default S x S).

    With `use_table` (and no accumulation), a field propagated to the S x S plane, or an
    S x S field propagated and cropped back to (Ho, Wo), reads its transfer function from
    a cached precomputed table (transfer_table, one (2S)^2 table per (wavelength,
    distance, pitch, aperture)) and runs on the tuned table column pass; the values equal
    the per-call evaluation.  Other shapes evaluate the transfer function in the call."""
    field = _check_field(field, "field")
    if field.dim() != 2:
        raise ValueError("field must be 2-D (H, W)")
    Hi, Wi = field.shape
    Ho, Wo = (S, S) if out_hw is None else out_hw
    if out is None:
        out = torch.empty((Ho, Wo), dtype=torch.complex64, device=field.device)
    ws = _workspace(S, 1, Hi, 1, Ho, field.device)
    L = _lib.lib()
    wl, pitch, d, ap = _scalar(wavelength), _scalar(pixel_pitch), _scalar(distance), _scalar(aperture_size)
    plan = get_plan(S, field.device)
    if use_table and not accumulate and ((Ho, Wo) == (S, S) or (Hi, Wi) == (S, S)):
        if (Ho, Wo) == (S, S):
            table = transfer_table(S, 1, 1, [wl], [d], pitch, ap, field.device)
            if table is not None:
                st = L.cvhrf_asm_propagate_planes_table(plan, ctypes.c_void_p(field.data_ptr()), 1, 1, Hi, Wi,
                                                        ctypes.c_void_p(table.data_ptr()),
                                                        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                                        ws.numel(), _stream(field))
                _lib.check(st, "cvhrf_asm_propagate_planes_table")
                return out
        else:
            # the adjoint pass multiplies by the conjugate of its table; conj(H at -d) = H at d
            table = transfer_table(S, 1, 1, [wl], [-d], pitch, ap, field.device)
            if table is not None:
                st = L.cvhrf_asm_propagate_planes_adjoint_table(plan, ctypes.c_void_p(field.data_ptr()), 1, 1, Ho,
                                                                Wo, ctypes.c_void_p(table.data_ptr()),
                                                                ctypes.c_void_p(out.data_ptr()),
                                                                ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                                                _stream(field))
                _lib.check(st, "cvhrf_asm_propagate_planes_adjoint_table")
                return out
    st = L.cvhrf_asm_propagate(plan, ctypes.c_void_p(field.data_ptr()), Hi, Wi,
                               ctypes.c_void_p(out.data_ptr()), Ho, Wo, wl, pitch, d, ap, int(bool(accumulate)),
                               ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(field))
    _lib.check(st, "cvhrf_asm_propagate")
    return out


class BandlimitedPropagationFunction(torch.autograd.Function):
    """python_function.py:109-218 — same arguments, same return, same gradients."""

    @staticmethod
    def forward(ctx, field, wavelength, pixel_pitch, distance, size, aperture_size=-1.0):
        S = _square_size(size)
        ctx.params = (_scalar(wavelength), _scalar(pixel_pitch), _scalar(distance), S, _scalar(aperture_size))
        ctx.input_size = tuple(field.shape[-2:])
        return propagate(field, *ctx.params[:3], S, ctx.params[4])

    @staticmethod
    def backward(ctx, grad_output):
        wl, pitch, dist, S, ap = ctx.params
        grad_field = propagate(grad_output.contiguous(), wl, pitch, -dist, S, ap, out_hw=ctx.input_size)
        return grad_field, None, None, None, None, None


def BandlimitedPropagation(field, wavelength, pixel_pitch, distance, size, use_cuda=True, aperture_size=-1.0):
    """python_function.py:220-226.  Only the CUDA path exists in this package."""
    if not use_cuda:
        raise NotImplementedError("use_cuda=False (the pure-torch CPU path) is not part of this package")
    return BandlimitedPropagationFunction.apply(field, wavelength, pixel_pitch, distance, size, aperture_size)


_tables = {}
_tables_lock = threading.Lock()


def transfer_table(S, K, C, wavelengths, distances, pixel_pitch, aperture_size, device):
    """The precomputed transfer tables of a (K planes x C wavelengths) propagation
    (cvhrf_asm_transfer_table_build), cached per configuration; None where the size has
    no compile-time plan.  Built on first use (make that first call outside stream capture)."""
    L = _lib.lib()
    nbytes = L.cvhrf_asm_transfer_table_bytes(int(S), int(K), int(C))
    if nbytes == 0:
        return None
    key = (torch.device(device), int(S), tuple(wavelengths), tuple(distances), float(pixel_pitch), float(aperture_size))
    with _tables_lock:
        t = _tables.get(key)
        if t is None:
            t = torch.empty(nbytes, dtype=torch.uint8, device=device)
            _lib.check(L.cvhrf_asm_transfer_table_build(get_plan(S, device), int(K), int(C),
                                                        _lib.float_array(wavelengths), _lib.float_array(distances),
                                                        float(pixel_pitch), float(aperture_size),
                                                        ctypes.c_void_p(t.data_ptr()), _stream(t)),
                       "cvhrf_asm_transfer_table_build")
            _tables[key] = t
    return t


class PlanePropagationFunction(torch.autograd.Function):
    """Fused plane/channel loop of model.py:1251-1272.

    fields (K, C, H, W) complex64 -> hologram (C, S, S) = sum_p propagate(fields[p, c],
    wavelengths[c], distances[p]).  `distances` are the signed distances passed to
    BandlimitedPropagation (the model passes -d_p).
    """

    @staticmethod
    def forward(ctx, fields, wavelengths, distances, pixel_pitch, S, aperture_size=-1.0, use_table=True):
        fields = _check_field(fields, "fields")
        K, C, H, W = fields.shape
        wl = [_scalar(w) for w in wavelengths]
        ds = [_scalar(d) for d in distances]
        if len(wl) != C or len(ds) != K:
            raise ValueError("len(wavelengths) must equal C and len(distances) must equal K")
        ctx.cfg = (wl, ds, _scalar(pixel_pitch), int(S), _scalar(aperture_size), (K, C, H, W))
        holo = torch.empty((C, S, S), dtype=torch.complex64, device=fields.device)
        ws = _workspace(S, K * C, H, C, S, fields.device)
        L = _lib.lib()
        table = transfer_table(S, K, C, wl, ds, ctx.cfg[2], ctx.cfg[4], fields.device) if use_table else None
        ctx.table = table
        if table is not None:
            with timed("propagation_forward"):
                st = L.cvhrf_asm_propagate_planes_table(get_plan(S, fields.device), ctypes.c_void_p(fields.data_ptr()),
                                                        K, C, H, W, ctypes.c_void_p(table.data_ptr()),
                                                        ctypes.c_void_p(holo.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                                        ws.numel(), _stream(fields))
            _lib.check(st, "cvhrf_asm_propagate_planes_table")
            return holo
        with timed("propagation_forward"):
            st = L.cvhrf_asm_propagate_planes(get_plan(S, fields.device), ctypes.c_void_p(fields.data_ptr()), K, C, H,
                                          W, _lib.float_array(wl), _lib.float_array(ds), ctx.cfg[2], ctx.cfg[4],
                                          ctypes.c_void_p(holo.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                          ws.numel(), _stream(fields))
        _lib.check(st, "cvhrf_asm_propagate_planes")
        return holo

    @staticmethod
    def backward(ctx, grad_holo):
        wl, ds, pitch, S, ap, (K, C, H, W) = ctx.cfg
        g = _check_field(grad_holo, "grad_holo")
        grad_fields = torch.empty((K, C, H, W), dtype=torch.complex64, device=g.device)
        ws = _workspace(S, C, S, K * C, H, g.device)
        L = _lib.lib()
        if ctx.table is not None:
            with timed("propagation_backward"):
                st = L.cvhrf_asm_propagate_planes_adjoint_table(get_plan(S, g.device), ctypes.c_void_p(g.data_ptr()), K,
                                                                C, H, W, ctypes.c_void_p(ctx.table.data_ptr()),
                                                                ctypes.c_void_p(grad_fields.data_ptr()),
                                                                ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(g))
            _lib.check(st, "cvhrf_asm_propagate_planes_adjoint_table")
            return grad_fields, None, None, None, None, None, None
        with timed("propagation_backward"):
            st = L.cvhrf_asm_propagate_planes_adjoint(get_plan(S, g.device), ctypes.c_void_p(g.data_ptr()), K, C, H, W,
                                                  _lib.float_array(wl), _lib.float_array(ds), pitch, ap,
                                                  ctypes.c_void_p(grad_fields.data_ptr()),
                                                  ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(g))
        _lib.check(st, "cvhrf_asm_propagate_planes_adjoint")
        return grad_fields, None, None, None, None, None, None


def propagate_planes(fields, wavelengths, distances, pixel_pitch, S, aperture_size=-1.0, use_table=True):
    """Sum over planes of the propagated fields.  `use_table` reads the transfer
    function from a cached precomputed table (transfer_table) where the size allows."""
    return PlanePropagationFunction.apply(fields, wavelengths, distances, pixel_pitch, S, aperture_size, use_table)
