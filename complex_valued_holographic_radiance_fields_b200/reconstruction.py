"""SLM -> image-plane reconstruction and the multiplane training loss.

Mirrors the reference's training-loss path (train.py:280-304):

* ``Propagator`` (alias ``propagator``) is utils/propagator.py:172-636: the same
  constructor, ``reconstruct(hologram_phases, amplitude, no_grad, get_complex)`` returning
  the frames x depths x channels reconstructions, and ``__call__(field, channel_id,
  depth_id)``.  The per-(depth, channel) transfer functions are built once, as the
  reference caches them in ``self.kernels`` (:473-520), and uploaded into a libcvhrf
  transfer table (``cvhrf_asm_transfer_table_upload``); one reconstruction is then three
  fused FFT passes for all depths and channels (``cvhrf_asm_propagate_planes_adjoint_table``,
  one forward and K inverse column transforms per channel), and its gradient the fused
  K-plane sum (``cvhrf_asm_propagate_planes_table``).  The reference instead runs
  frames x depths x channels separate odak ``custom`` propagations (27 at K = 3), of which
  the identity laser powers zero two thirds.
* ``MultiplaneLoss`` (alias ``multiplane_loss_odak``) is utils/propagator.py:8-170: the
  quantised-depth targets and masks, the defocus blur, and ``__call__``.
* ``reconstruction_loss(fields, targets, masks, ...)`` is the loop of train.py:293-304
  fused into one libcvhrf launch forward and one backward (``cvhrf_multiplane_loss``):
  crop, clamp and the three MSE terms of every plane, plus GaussianLoss's SSIM term
  (utils/data_utils.py:124-157) on the fused SSIM kernel.

odak 0.2.6 and pytorch_msssim are not installed here.  Their functions on this path are
restated below from their published algorithms (no parity vectors exist for them here):
``get_band_limited_angular_spectrum_kernel`` (the centred band-limited angular-spectrum
transfer function on odak's frequency grid), ``circular_binary_mask``,
``generate_2d_gaussian``, and pytorch_msssim's SSIM (11-tap Gaussian window, sigma 1.5,
valid filtering, C1 = 0.01^2, C2 = 0.03^2), which equals the mean of the zero-padded SSIM
map over the pixels at least 5 from every edge, the pixels whose window lies inside the
image.
"""
import ctypes
import threading

import numpy as np
import torch

from . import _lib
from .profiling import timed
from .propagation import _check_field, _stream, _workspace, get_plan
from .ssim import C1 as SSIM_C1, C2 as SSIM_C2, FusedSSIMMap


# ---- odak helpers (restated; odak 0.2.6 is absent) ------------------------------------
def band_limited_angular_spectrum_kernel(nu, nv, dx=8e-6, wavelength=515e-9, distance=0.0, device="cpu"):
    """odak.learn.wave.get_band_limited_angular_spectrum_kernel: centred nu x nv complex64
    transfer function exp(i 2 pi d sqrt(1/lambda^2 - fx^2 - fy^2)) on the grid
    f = linspace(-1/(2 dx) + 1/(4 n dx), 1/(2 dx) - 1/(4 n dx), n), band-limited to
    |f| < 1 / (lambda sqrt((2 d / (n dx))^2 + 1)) per axis; float32 throughout."""
    x = dx * float(nu)
    y = dx * float(nv)
    fx = torch.linspace(-1 / (2 * dx) + 0.5 / (2 * x), 1 / (2 * dx) - 0.5 / (2 * x), nu, dtype=torch.float32,
                        device=device)
    fy = torch.linspace(-1 / (2 * dx) + 0.5 / (2 * y), 1 / (2 * dx) - 0.5 / (2 * y), nv, dtype=torch.float32,
                        device=device)
    FY, FX = torch.meshgrid(fx, fy, indexing="ij")
    HH_exp = 2 * np.pi * torch.sqrt(1 / wavelength ** 2 - (FX ** 2 + FY ** 2))
    distance = torch.as_tensor([float(distance)], dtype=torch.float32, device=device)
    H_exp = torch.mul(HH_exp, distance)
    fx_max = 1 / torch.sqrt((2 * distance * (1 / x)) ** 2 + 1) / wavelength
    fy_max = 1 / torch.sqrt((2 * distance * (1 / y)) ** 2 + 1) / wavelength
    H_filter = ((torch.abs(FX) < fx_max) & (torch.abs(FY) < fy_max)).float()
    return (H_filter * torch.cos(H_exp) + 1j * H_filter * torch.sin(H_exp)).to(torch.complex64)


def circular_binary_mask(px, py, r):
    """odak.learn.tools.circular_binary_mask: 1 where the distance from the centre of a
    linspace(-p/2, p/2, p) grid is below r."""
    x = torch.linspace(-px / 2.0, px / 2.0, px)
    y = torch.linspace(-py / 2.0, py / 2.0, py)
    X, Y = torch.meshgrid(x, y, indexing="ij")
    Z = (X ** 2 + Y ** 2) ** 0.5
    mask = torch.zeros_like(Z)
    mask[Z < r] = 1
    return mask


def generate_2d_gaussian(kernel_length=(21, 21), nsigma=(3, 3), mu=(0, 0), normalize=False):
    """odak.learn.tools.generate_2d_gaussian: exp(-((X - mu)^2 / (2 sx^2) + (Y - mu)^2 / (2 sy^2)))
    / (2 pi sx sy) on linspace(-L/2, L/2, L) grids (a zero sigma is replaced by 1e-5)."""
    x = torch.linspace(-kernel_length[0] / 2.0, kernel_length[0] / 2.0, kernel_length[0])
    y = torch.linspace(-kernel_length[1] / 2.0, kernel_length[1] / 2.0, kernel_length[1])
    X, Y = torch.meshgrid(x, y, indexing="ij")
    sx = nsigma[0] if nsigma[0] != 0 else 1e-5
    sy = nsigma[1] if nsigma[1] != 0 else 1e-5
    k = 1.0 / (2.0 * np.pi * sx * sy) * torch.exp(
        -((X - mu[0]) ** 2.0 / (2.0 * sx ** 2.0) + (Y - mu[1]) ** 2.0 / (2.0 * sy ** 2.0)))
    if normalize:
        k = k / k.max()
    return k


# ---- the fused reconstruction operator -------------------------------------------------
def upload_table(S, kernels_centred):
    """libcvhrf transfer table from centred transfer functions (items x 2S x 2S complex64,
    item p * C + c)."""
    k = kernels_centred.to(torch.complex64).contiguous()
    items = k.shape[0]
    if tuple(k.shape[1:]) != (2 * S, 2 * S):
        raise ValueError(f"kernels must be items x {2 * S} x {2 * S}, got {tuple(k.shape)}")
    L = _lib.lib()
    nbytes = L.cvhrf_asm_transfer_table_bytes(int(S), int(items), 1)
    if nbytes == 0:
        raise ValueError(f"no compile-time FFT plan for S = {S} or too many items ({items})")
    t = torch.empty(nbytes, dtype=torch.uint8, device=k.device)
    _lib.check(L.cvhrf_asm_transfer_table_upload(get_plan(S, k.device), int(items), ctypes.c_void_p(k.data_ptr()),
                                                 ctypes.c_void_p(t.data_ptr()), _stream(k)),
               "cvhrf_asm_transfer_table_upload")
    return t


class ReconstructFunction(torch.autograd.Function):
    """field (C, S, S) complex64 -> plane fields (K, C, S, S): fields[p, c] =
    crop_S(IFFT2(H[p, c] * FFT2(pad_2S(field[c])))), H the (aperture-multiplied) transfer
    functions of the table, which holds conj(H) (the adjoint column pass multiplies by
    the conjugate of its table).  Backward: the adjoint, summed over planes."""

    @staticmethod
    def forward(ctx, field, table, K):
        field = _check_field(field, "field")
        C, S, S2 = field.shape
        if S != S2:
            raise ValueError("field must be C x S x S")
        out = torch.empty((K, C, S, S), dtype=torch.complex64, device=field.device)
        ws = _workspace(S, C, S, K * C, S, field.device)
        with timed("reconstruct"):
            _lib.check(_lib.lib().cvhrf_asm_propagate_planes_adjoint_table(
                get_plan(S, field.device), ctypes.c_void_p(field.data_ptr()), K, C, S, S,
                ctypes.c_void_p(table.data_ptr()), ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                ws.numel(), _stream(field)), "cvhrf_asm_propagate_planes_adjoint_table")
        ctx.table, ctx.dims = table, (K, C, S)
        return out

    @staticmethod
    def backward(ctx, g):
        K, C, S = ctx.dims
        g = _check_field(g, "grad")
        grad = torch.empty((C, S, S), dtype=torch.complex64, device=g.device)
        ws = _workspace(S, K * C, S, C, S, g.device)
        with timed("reconstruct_backward"):
            _lib.check(_lib.lib().cvhrf_asm_propagate_planes_table(
                get_plan(S, g.device), ctypes.c_void_p(g.data_ptr()), K, C, S, S,
                ctypes.c_void_p(ctx.table.data_ptr()), ctypes.c_void_p(grad.data_ptr()),
                ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(g)), "cvhrf_asm_propagate_planes_table")
        return grad, None, None


class Propagator:
    """utils/propagator.py:172-636 (the constructor arguments, reconstruct and __call__).
    Only 'Bandlimited Angular Spectrum' kernels (the type train.py:876 uses) are built;
    resolution is the S x S hologram size (train.py passes pad_size)."""

    def __init__(self, resolution=(1920, 1080), wavelengths=(515e-9,), pixel_pitch=8e-6, resolution_factor=1,
                 number_of_frames=1, number_of_depth_layers=1, volume_depth=1e-2, image_location_offset=5e-3,
                 propagation_type="Bandlimited Angular Spectrum", propagator_type="back and forth",
                 back_and_forth_distance=0.3, laser_channel_power=None, aperture=None, aperture_size=None,
                 distances=None, aperture_samples=(20, 20, 5, 5), method="conventional", device="cpu"):
        if propagation_type != "Bandlimited Angular Spectrum":
            raise NotImplementedError(f"propagation_type {propagation_type!r}: only 'Bandlimited Angular Spectrum'")
        if propagator_type not in ("forward", "back and forth"):
            raise ValueError(f"unknown propagator_type {propagator_type!r}")
        if method not in ("conventional", "multi-color"):
            raise ValueError(f"unknown method {method!r}")
        self.device = torch.device(device)
        self.resolution = [int(r) for r in resolution]
        if self.resolution[0] != self.resolution[1]:
            raise ValueError("the fused propagation needs a square resolution (S x S)")
        self.S = self.resolution[0]
        self.resolution_factor = 1  # as the reference sets for every type but impulse-response Fresnel (:246-248)
        self.wavelengths = [float(w) for w in wavelengths]
        self.pixel_pitch = float(pixel_pitch)
        self.number_of_frames = int(number_of_frames)
        self.number_of_channels = len(self.wavelengths)
        self.volume_depth = volume_depth
        self.image_location_offset = image_location_offset
        self.propagator_type = propagator_type
        self.zero_mode_distance = torch.tensor(back_and_forth_distance)
        self.method = method
        self.aperture_samples = aperture_samples
        if distances is None:
            self.distances = (torch.linspace(-volume_depth / 2.0, volume_depth / 2.0, number_of_depth_layers)
                              + image_location_offset)
        else:
            self.distances = torch.as_tensor(distances)
        self.number_of_depth_layers = int(self.distances.shape[0])
        if laser_channel_power is None:
            laser_channel_power = torch.eye(self.number_of_frames, self.number_of_channels)
        self.channel_power = torch.as_tensor(laser_channel_power, dtype=torch.float32)
        self.phase_scale = torch.ones(self.number_of_channels, device=self.device)  # :315-329
        self.set_aperture(aperture, aperture_size)
        self._table = None
        self.kernels = None

    def set_aperture(self, aperture=None, aperture_size=None):
        """:331-360: a circular mask of radius aperture_size (default S) on the 2S x 2S grid,
        or a given aperture zero-padded to it."""
        P = 2 * self.S
        if aperture is None:
            if aperture_size is None:
                aperture_size = self.S
            self.aperture = circular_binary_mask(P, P, aperture_size).to(self.device) * 1.0
        else:
            a = torch.as_tensor(aperture, dtype=torch.float32)
            pad = torch.zeros(P, P)
            y0, x0 = P // 2 - a.shape[-2] // 2, P // 2 - a.shape[-1] // 2
            pad[y0:y0 + a.shape[-2], x0:x0 + a.shape[-1]] = a
            self.aperture = pad.to(self.device)
        self._table = None

    def get_laser_powers(self):
        """:362-376."""
        if self.method == "multi-color":
            return torch.abs(torch.cos(self.channel_power))
        return self.channel_power

    def set_laser_powers(self, laser_power):
        self.channel_power = torch.as_tensor(laser_power, dtype=torch.float32)

    def _kernel(self, depth_id, channel_id):
        P = 2 * self.S
        wl = self.wavelengths[channel_id]
        d = float(self.distances[depth_id])
        if self.propagator_type == "forward":
            return band_limited_angular_spectrum_kernel(P, P, self.pixel_pitch, wl, d, self.device)
        zm = float(self.zero_mode_distance)
        back = -(zm + self.image_location_offset - d)
        return (band_limited_angular_spectrum_kernel(P, P, self.pixel_pitch, wl, zm, self.device)
                * band_limited_angular_spectrum_kernel(P, P, self.pixel_pitch, wl, back, self.device))

    def table(self):
        """The transfer table of every (depth, channel), built once (:473-520): the odak kernel
        times the aperture (custom() applies both), stored conjugated for the adjoint pass."""
        if self._table is None:
            K, C = self.number_of_depth_layers, self.number_of_channels
            ks = torch.stack([self._kernel(p, c) for p in range(K) for c in range(C)])
            self.kernels = ks.view(K, C, 2 * self.S, 2 * self.S)
            self._table = upload_table(self.S, torch.conj(ks * self.aperture).resolve_conj())
        return self._table

    def set_kernels(self, kernels):
        """Use the given transfer functions (depths x channels x 2S x 2S complex, centred,
        the layout of the reference's self.kernels) instead of building them.  The phase
        d kz of these kernels is about 4e4 rad, held in float32 (a 4e-3 rad step) by odak
        and by the restatement here, so kernels evaluated on another device or library
        differ at the 1e-3 level; supplying the same kernels removes that difference."""
        K, C = self.number_of_depth_layers, self.number_of_channels
        k = torch.as_tensor(kernels).to(device=self.device, dtype=torch.complex64)
        if tuple(k.shape) != (K, C, 2 * self.S, 2 * self.S):
            raise ValueError(f"kernels must be {K} x {C} x {2 * self.S} x {2 * self.S}")
        self.kernels = k
        self._table = upload_table(self.S, torch.conj(k.reshape(K * C, 2 * self.S, 2 * self.S) * self.aperture)
                                   .resolve_conj())

    def propagate_all(self, field):
        """field (C, S, S) complex64 -> (K, C, S, S): every depth of every channel (differentiable)."""
        return ReconstructFunction.apply(field, self.table(), self.number_of_depth_layers)

    def __call__(self, input_field, channel_id, depth_id):
        """:406-471: one channel's field (S x S) propagated to one depth."""
        C = self.number_of_channels
        f = torch.zeros((C, self.S, self.S), dtype=torch.complex64, device=input_field.device)
        f[channel_id] = input_field
        return self.propagate_all(f)[depth_id, channel_id]

    def channel_scale(self):
        """Sum over frames of each channel's squared laser power: with a diagonal power
        matrix, the factor by which the frame-summed intensities (train.py:293) scale
        |propagated field|^2."""
        if not self.diagonal_power():
            raise ValueError("channel_scale needs one channel per frame (a diagonal laser power matrix)")
        return (self.get_laser_powers().float() ** 2).sum(0)

    def reconstruct(self, hologram_phases, amplitude=None, no_grad=True, get_complex=False):
        """:522-546 / _reconstruct_impl :548-636: frames x depths x channels x S x S
        intensities (or complex fields).  Frame f, channel c is the propagation of
        power[f, c] * amplitude[c] * exp(i phase[f] * phase_scale[c]).  The propagation is
        linear, so the power is applied after it; with a diagonal power matrix (one channel
        per frame, as train.py:878 configures) one fused propagation covers every frame."""
        if no_grad:
            with torch.no_grad():
                return self._reconstruct(hologram_phases, amplitude, get_complex)
        return self._reconstruct(hologram_phases, amplitude, get_complex)

    def hologram_field(self, phase, amplitude=None):
        """amplitude[c] * exp(i phase[c] * phase_scale[c]) for C x S x S phases (odak
        generate_complex_field)."""
        C = self.number_of_channels
        if amplitude is None:
            amplitude = torch.ones((C, self.S, self.S), device=phase.device)
        scale = self.phase_scale.to(phase.device)[:C].view(C, 1, 1)
        return torch.polar(amplitude.float().expand(C, -1, -1), (phase * scale).float()).to(torch.complex64)

    def diagonal_power(self):
        p = self.get_laser_powers()
        F, C = p.shape
        return F == C and bool(torch.all(p * (1.0 - torch.eye(F)) == 0))

    def _reconstruct(self, hologram_phases, amplitude, get_complex):
        phase = hologram_phases.squeeze(0) if hologram_phases.dim() > 3 else hologram_phases
        power = self.get_laser_powers().float()
        F, C = power.shape
        if phase.shape[0] < F:
            raise ValueError(f"{phase.shape[0]} hologram frames for {F} configured frames")
        pw = power.to(phase.device).view(F, 1, C, 1, 1)
        if self.diagonal_power():
            # frame f lights channel f only: channel c's field uses phase[c]
            fields = self.propagate_all(self.hologram_field(phase[:C], amplitude)).unsqueeze(0)
        else:
            fields = torch.stack([self.propagate_all(self.hologram_field(phase[f].expand(C, -1, -1), amplitude))
                                  for f in range(F)])
        if get_complex:
            return pw * fields
        return (pw ** 2) * (fields.real ** 2 + fields.imag ** 2)


propagator = Propagator


# ---- the multiplane loss -----------------------------------------------------------------
class MultiplaneLoss:
    """utils/propagator.py:8-170 (multiplane_loss_odak): targets and masks from a target
    image and a normalised depth map, optional defocus blur, and the three-term loss."""

    def __init__(self, target_image, target_depth, blur_ratio=0.25, target_blur_size=10, number_of_planes=4,
                 weights=(1.0, 2.1, 0.6), multiplier=1.0, scheme="defocus", reduction="mean", split_ratio=1.0,
                 device="cpu"):
        self.device = torch.device(device)
        self.target_image = target_image.float().to(self.device)
        self.target_depth = target_depth.float().to(self.device)
        self.target_blur_size = target_blur_size + (1 if target_blur_size % 2 == 0 else 0)
        self.number_of_planes = number_of_planes
        self.multiplier = multiplier
        self.weights = list(weights)
        self.reduction = reduction
        self.blur_ratio = blur_ratio
        self.split_ratio = split_ratio
        self.set_targets()
        if scheme == "defocus":
            self.add_defocus_blur()
        self.loss_function = torch.nn.MSELoss(reduction=reduction)

    def get_targets(self):
        divider = max(self.number_of_planes - 1, 1)
        return self.targets.detach().clone(), self.masks.detach().clone(), self.target_depth.detach().clone() / divider

    def set_targets(self):
        """:73-110: depth quantised to round(depth^ratio (K - 1)); plane i's target is the
        image where the quantised depth is i, its mask the indicator."""
        ratio = self.split_ratio if self.number_of_planes == 2 else 1.0
        biased = torch.pow(self.target_depth, ratio) * (self.number_of_planes - 1)
        self.target_depth = torch.round(biased, decimals=0)
        K = self.number_of_planes
        masks = (self.target_depth.reshape(1, 1, *self.target_image.shape[-2:])
                 == torch.arange(K, device=self.device).view(K, 1, 1, 1).float())
        masks = masks.expand(K, self.target_image.shape[0], -1, -1).float()
        self.masks = masks.contiguous()
        self.targets = (self.target_image.unsqueeze(0) * self.masks).contiguous()

    def add_defocus_blur(self):
        """:112-136: plane i's target is the sum over planes j holding content of the
        all-plane image blurred by a Gaussian of sigma int(|i - j| blur_ratio), restricted
        to plane j's mask."""
        K, C = self.number_of_planes, self.target_image.shape[0]
        L = [self.target_blur_size, self.target_blur_size]
        new = torch.zeros_like(self.targets)
        for ch in range(C):
            cache = self.targets[:, ch].clone()
            target = cache.sum(0)
            for i in range(K):
                defocus = torch.zeros_like(cache[i])
                for j in range(K):
                    if torch.sum(cache[j]) > 0:
                        ns = 0.0 if i == j else int(abs(i - j) * self.blur_ratio)
                        k = generate_2d_gaussian(L, [ns, ns]).to(self.device)
                        k = (k / torch.sum(k)).view(1, 1, *k.shape)
                        plane = torch.nn.functional.conv2d(target.view(1, 1, *target.shape), k, padding="same")
                        defocus = defocus + plane.view(target.shape) * torch.abs(self.masks[j, ch])
                new[i, ch] = defocus
        self.targets = new * self.multiplier

    def __call__(self, image, target, plane_id=None):
        """:138-169 (without noise injection)."""
        l2 = self.weights[0] * self.loss_function(image, target)
        mask = self.masks if plane_id is None else self.masks[plane_id]
        l2_mask = self.weights[1] * self.loss_function(image * mask, target * mask)
        l2_cor = self.weights[2] * self.loss_function(image * target, target * target)
        return l2 + l2_mask + l2_cor


multiplane_loss_odak = MultiplaneLoss

_loss_ws = {}
_loss_ws_lock = threading.Lock()


def _loss_workspace(device):
    key = torch.device(device)
    with _loss_ws_lock:
        w = _loss_ws.get(key)
        if w is None:
            L = _lib.lib()
            n = L.cvhrf_multiplane_loss_workspace_bytes()
            w = torch.empty(n, dtype=torch.uint8, device=device)
            _lib.check(L.cvhrf_multiplane_loss_init_workspace(ctypes.c_void_p(w.data_ptr()), n, _stream(w)),
                       "cvhrf_multiplane_loss_init_workspace")
            _loss_ws[key] = w
    return w


class MultiplaneLossFunction(torch.autograd.Function):
    """fields (K, C, S, S) complex64 -> (loss, pred): the fused crop / clamp / three-MSE loss
    of every plane (cvhrf_multiplane_loss); pred (K, C, H, W) is the clamped prediction and
    carries its own gradient (e.g. from an SSIM term) into the backward."""

    @staticmethod
    def forward(ctx, fields, targets, masks, weights, channel_scale):
        fields = _check_field(fields, "fields")
        K, C, S, _ = fields.shape
        H, W = targets.shape[-2:]
        targets = targets.float().contiguous()
        masks = masks.float().contiguous()
        if tuple(targets.shape) != (K, C, H, W) or tuple(masks.shape) != (K, C, H, W):
            raise ValueError("targets and masks must be K x C x H x W")
        w = _lib.float_array(weights)
        sc = _lib.float_array(channel_scale)
        pred = torch.empty((K, C, H, W), dtype=torch.float32, device=fields.device)
        loss = torch.empty((), dtype=torch.float32, device=fields.device)
        ws = _loss_workspace(fields.device)
        with timed("multiplane_loss"):
            _lib.check(_lib.lib().cvhrf_multiplane_loss(
                ctypes.c_void_p(fields.data_ptr()), K, C, S, H, W, sc, ctypes.c_void_p(targets.data_ptr()),
                ctypes.c_void_p(masks.data_ptr()), w, ctypes.c_void_p(pred.data_ptr()),
                ctypes.c_void_p(loss.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(fields)),
                "cvhrf_multiplane_loss")
        ctx.save_for_backward(fields, targets, masks)
        ctx.cfg = (list(weights), list(channel_scale))
        return loss, pred

    @staticmethod
    def backward(ctx, g_loss, g_pred):
        fields, targets, masks = ctx.saved_tensors
        weights, scale = ctx.cfg
        K, C, S, _ = fields.shape
        H, W = targets.shape[-2:]
        if g_loss is None:
            g_loss = torch.zeros((), dtype=torch.float32, device=fields.device)
        g_loss = g_loss.float().contiguous()
        gp = None if g_pred is None else g_pred.float().contiguous()
        grad = torch.empty_like(fields)
        with timed("multiplane_loss_backward"):
            _lib.check(_lib.lib().cvhrf_multiplane_loss_backward(
                ctypes.c_void_p(fields.data_ptr()), K, C, S, H, W, _lib.float_array(scale),
                ctypes.c_void_p(targets.data_ptr()), ctypes.c_void_p(masks.data_ptr()), _lib.float_array(weights),
                ctypes.c_void_p(g_loss.data_ptr()), ctypes.c_void_p(0 if gp is None else gp.data_ptr()),
                ctypes.c_void_p(grad.data_ptr()), _stream(fields)), "cvhrf_multiplane_loss_backward")
        return grad, None, None, None, None


def msssim_ssim(pred, target):
    """pytorch_msssim SSIM(data_range=1, size_average=True) of C' x H x W images: the mean of
    the fused SSIM map over the pixels whose 11 x 11 window lies inside the image."""
    m = FusedSSIMMap.apply(SSIM_C1, SSIM_C2, pred.contiguous(), target.contiguous())
    return m[:, 5:-5, 5:-5].mean()


def reconstruction_loss(fields, targets, masks, weights=(1.0, 1.0, 1.0), channel_scale=None, ssim=True,
                        lambda_ssim=0.025):
    """train.py:293-304 for all planes: sum over planes of multiplane_loss_odak(pred_p, t_p, p)
    + GaussianLoss(pred_p, t_p), pred_p = clamp(crop(channel_scale * |fields_p|^2), 0, 1).
    fields (K, C, S, S) complex64; targets, masks (K, C, H, W).  Returns the loss (device
    scalar, differentiable with respect to fields)."""
    K, C = fields.shape[:2]
    scale = [1.0] * C if channel_scale is None else [float(s) for s in channel_scale]
    loss, pred = MultiplaneLossFunction.apply(fields, targets, masks, list(weights)[:3], scale)
    if ssim:
        # GaussianLoss per plane: lambda_ssim * (1 - ssim_p) * 0.2; every plane has the same
        # pixel count, so the sum over planes of ssim_p is K times the mean over all planes
        s = msssim_ssim(pred.view(K * C, *pred.shape[-2:]), targets.reshape(K * C, *targets.shape[-2:]).float())
        loss = loss + lambda_ssim * 0.2 * K * (1.0 - s)
    return loss


_field_ws = {}
_field_ws_lock = threading.Lock()


def _field_workspace(device):
    key = torch.device(device)
    with _field_ws_lock:
        w = _field_ws.get(key)
        if w is None:
            L = _lib.lib()
            n = L.cvhrf_hologram_field_workspace_bytes()
            w = torch.empty(n, dtype=torch.uint8, device=device)
            _lib.check(L.cvhrf_hologram_field_init_workspace(ctypes.c_void_p(w.data_ptr()), n, _stream(w)),
                       "cvhrf_hologram_field_init_workspace")
            _field_ws[key] = w
    return w


class HologramFieldFunction(torch.autograd.Function):
    """hologram (C, S, S) complex64 -> SLM field |h| exp(i (angle(h) mod 2 pi - mean) s_c)
    (train.py:280-283 and utils/propagator.py:612-620) in two libcvhrf launches each way."""

    @staticmethod
    def forward(ctx, holo, phase_scale):
        holo = _check_field(holo, "hologram")
        C = holo.shape[0]
        n = holo[0].numel()
        field = torch.empty_like(holo)
        mean = torch.empty((), dtype=torch.float32, device=holo.device)
        ws = _field_workspace(holo.device)
        with timed("hologram_field"):
            _lib.check(_lib.lib().cvhrf_hologram_field(
                ctypes.c_void_p(holo.data_ptr()), C, n, _lib.float_array(phase_scale), ctypes.c_void_p(field.data_ptr()),
                ctypes.c_void_p(mean.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(holo)),
                "cvhrf_hologram_field")
        ctx.save_for_backward(holo, mean)
        ctx.scale = list(phase_scale)
        return field

    @staticmethod
    def backward(ctx, g):
        holo, mean = ctx.saved_tensors
        g = _check_field(g, "grad")
        grad = torch.empty_like(holo)
        ws = _field_workspace(holo.device)
        with timed("hologram_field_backward"):
            _lib.check(_lib.lib().cvhrf_hologram_field_backward(
                ctypes.c_void_p(holo.data_ptr()), holo.shape[0], holo[0].numel(), _lib.float_array(ctx.scale),
                ctypes.c_void_p(mean.data_ptr()), ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(grad.data_ptr()),
                ctypes.c_void_p(ws.data_ptr()), ws.numel(), _stream(holo)), "cvhrf_hologram_field_backward")
        return grad, None


def hologram_training_loss(prop, hologram, targets, masks, weights=(1.0, 1.0, 1.0), ssim=True, lambda_ssim=0.025):
    """train.py:280-304 after the render: the hologram's phase (mod 2 pi, minus its mean)
    and amplitude are recombined (HologramFieldFunction), reconstructed at every depth
    (prop: a Propagator with one channel per frame) and scored by reconstruction_loss.
    hologram: C x S x S complex64 (differentiable)."""
    C = prop.number_of_channels
    # the phase scale as host floats, read once (a device read here would synchronise,
    # and cannot happen inside a captured graph)
    key = prop.phase_scale.data_ptr()
    if getattr(prop, "_scale_key", None) != key:
        prop._scale_list = prop.phase_scale.detach().float().cpu()[:C].tolist()
        prop._scale_key = key
    fields = prop.propagate_all(HologramFieldFunction.apply(hologram, prop._scale_list))
    return reconstruction_loss(fields, targets, masks, weights, prop.channel_scale().tolist(), ssim, lambda_ssim)
