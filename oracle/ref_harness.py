"""Drive the reference's own CUDA kernels (rebuilt by oracle/build_ref.py).

TEST INFRASTRUCTURE ONLY.  The reference's Python glue cannot be imported as is
(cuda_prop/python_function.py imports odak at :6-8, absent here;
cov3d_cuda/python_import.py runs `setup.py install` at import, :14-16), so the
few lines of glue on the path are restated here, calling the UNMODIFIED
reference kernels in oracle/_ref/:

* ``RefBandlimitedPropagationFunction`` — python_function.py:109-218 with odak's
  zero_pad / crop_center restated as centred placement / centred window.
* ``RefSplatTileCuda`` — python_import.py:283-342 (singleton Rasterizer,
  forward_info kept for backward).
* ``ref_adam_update`` — python_import.py:457-460.
"""
import os
import sys

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
# CVHRF_REF_DIR selects another build of the same modules (oracle/_ref80: compute_80 PTX)
REF_DIR = os.environ.get("CVHRF_REF_DIR") or os.path.join(_HERE, "_ref")


def available():
    return (os.path.exists(os.path.join(REF_DIR, "cov3d_cuda_ref", "cov3d_cuda_ref.so"))
            and os.path.exists(os.path.join(REF_DIR, "cuda_modules_ref", "cuda_modules_ref.so")))


def _import(name):
    p = os.path.join(REF_DIR, name)
    if p not in sys.path:
        sys.path.insert(0, p)
    import importlib
    return importlib.import_module(name)


def cov3d():
    return _import("cov3d_cuda_ref")


def cuda_modules():
    return _import("cuda_modules_ref")


def zero_pad(x, size):
    P, Q = size
    H, W = x.shape[-2:]
    out = torch.zeros(x.shape[:-2] + (P, Q), dtype=x.dtype, device=x.device)
    oy, ox = (P - H) // 2, (Q - W) // 2
    out[..., oy:oy + H, ox:ox + W] = x
    return out


def crop_center(x, size):
    H, W = size
    P, Q = x.shape[-2:]
    oy, ox = (P - H) // 2, (Q - W) // 2
    return x[..., oy:oy + H, ox:ox + W]


def _freq_grids(doubled, pixel_pitch, device):
    nx, ny = doubled
    fx = torch.fft.fftshift(torch.fft.fftfreq(nx, d=pixel_pitch)).to(device)
    fy = torch.fft.fftshift(torch.fft.fftfreq(ny, d=pixel_pitch)).to(device)
    FX, FY = torch.meshgrid(fx, fy, indexing="ij")
    return FX.contiguous(), FY.contiguous()


class RefBandlimitedPropagationFunction(torch.autograd.Function):
    """python_function.py:109-218 around cuda_modules.bandlimited_propagation_{forward,backward}."""

    @staticmethod
    def forward(ctx, field, wavelength, pixel_pitch, distance, size, aperture_size=-1.0):
        M = cuda_modules()
        field = field.contiguous()
        ctx.save_for_backward(field)
        ctx.p = (wavelength, pixel_pitch, distance, tuple(size), aperture_size, tuple(field.shape[-2:]))
        doubled = [i * 2 for i in size]
        f = torch.fft.fftshift(torch.fft.fft2(zero_pad(field, doubled).contiguous())).contiguous()
        FX, FY = _freq_grids(doubled, pixel_pitch, field.device)
        re, im = M.bandlimited_propagation_forward(f.real.contiguous(), f.imag.contiguous(), FX, FY,
                                                   wavelength, distance, aperture_size, pixel_pitch)
        out = torch.fft.ifft2(torch.fft.ifftshift(torch.complex(re.contiguous(), im.contiguous()))).contiguous()
        return crop_center(out, size)

    @staticmethod
    def backward(ctx, grad_output):
        M = cuda_modules()
        field, = ctx.saved_tensors
        wavelength, pixel_pitch, distance, size, aperture_size, input_size = ctx.p
        doubled = [i * 2 for i in size]
        g = torch.fft.fftshift(torch.fft.fft2(zero_pad(grad_output.contiguous(), doubled).contiguous())).contiguous()
        f = torch.fft.fftshift(torch.fft.fft2(zero_pad(field, doubled).contiguous())).contiguous()
        FX, FY = _freq_grids(doubled, pixel_pitch, field.device)
        re, im = M.bandlimited_propagation_backward(g.real.contiguous(), g.imag.contiguous(), f.real.contiguous(),
                                                    f.imag.contiguous(), FX, FY,
                                                    wavelength, distance, aperture_size, pixel_pitch)
        gf = torch.fft.ifft2(torch.fft.ifftshift(torch.complex(re, im))).contiguous()
        return crop_center(gf, input_size).contiguous(), None, None, None, None, None


_rasterizer = None


def get_rasterizer():
    global _rasterizer
    if _rasterizer is None:
        _rasterizer = cov3d().Rasterizer()
    return _rasterizer


def view_buffer(R):
    """(3,3) view of a zeroed 16-float buffer with buf[10] = 1.

    The reference passes the 3x3 view matrix where a 4x4 is read
    (rasterizer_splat.cu:370-377, auxiliary.h:115-133); padding it this way keeps
    that read in bounds and makes its visibility test the intended z-range test
    when R = I.
    """
    buf = torch.zeros(16, dtype=torch.float32, device=R.device)
    buf[:9] = R.reshape(-1).float()
    buf[10] = 1.0
    return buf[:9].view(3, 3)


_last_info = None


def get_rasterizer_info():
    """forward_info (final_Ts, n_contrib, point_list, ranges, visible) of the last RefSplatTileCuda forward."""
    return _last_info


# Bytes of the reference rasterizer's image scratch buffer that its singleton pool holds.
_img_buffer_held = 0


def ref_image_buffer_bytes(W, H, K):
    """The reference's image scratch request: required<ImageState>(num_tiles, H * W, K)
    (rasterizer_splat.cu:483, rasterizer_splat.h:36-39) = tiles x pixels x K x
    sizeof(ImageState) (three pointers) + 128 bytes."""
    tiles = ((W + 15) // 16) * ((H + 15) // 16)
    return tiles * W * H * K * 24 + 128


def _guard_image_buffer(W, H, K, device):
    """The reference prints and ignores a failed cudaMalloc of that buffer and then writes
    through a null pointer (rasterizer_splat.cu:258-264).  Refuse, on the host, any call
    whose buffer cannot be allocated (it is 387 GB at 1008 x 756 x 7 and 1.2 TB at
    1920 x 1080 x 3)."""
    global _img_buffer_held
    need = ref_image_buffer_bytes(W, H, K)
    if need <= _img_buffer_held:
        return
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info(device)
    if need + (4 << 30) > free + _img_buffer_held:
        raise RuntimeError(f"reference rasterizer image scratch of {need / 2**30:.1f} GiB for {W}x{H}x{K} does not fit "
                           f"({(free + _img_buffer_held) / 2**30:.1f} GiB available); not running the reference")
    _img_buffer_held = need


class RefSplatTileCuda(torch.autograd.Function):
    """python_import.py:283-342."""

    @staticmethod
    def forward(ctx, cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs,
                fx, fy, px, py, view_matrix, img_size, near_plane, far_plane, tile_size=(16, 16)):
        _guard_image_buffer(int(img_size[0]), int(img_size[1]), int(plane_probs.shape[1]), cam_means_3D.device)
        ctx.save_for_backward(cam_means_3D, z_vals, quats, scales, colours, phase, opacities, plane_probs, view_matrix)
        ctx.p = (fx, fy, px, py, img_size, tile_size, near_plane, far_plane)
        output, info = get_rasterizer().forward(cam_means_3D, z_vals, quats, scales, colours, phase, opacities,
                                                plane_probs, fx, fy, px, py, view_matrix, img_size, tile_size,
                                                near_plane, far_plane)
        global _last_info
        ctx.info = info
        _last_info = info
        return output, info[-1]

    @staticmethod
    def backward(ctx, grad_output, grad_vis=None):
        cam, z, q, s, col, ph, op, pp, view = ctx.saved_tensors
        fx, fy, px, py, img_size, tile_size, near, far = ctx.p
        final_Ts, n_contrib, point_list, ranges, _ = ctx.info
        g = get_rasterizer().backward(grad_output.contiguous(), cam, z, q, s, col, ph, op, pp, fx, fy, px, py, view,
                                      img_size, tile_size, final_Ts, n_contrib, point_list, ranges, near, far)
        return tuple(g) + (None,) * 9


def ref_adam_update(param, grad, exp_avg, exp_avg_sq, visible, lr, b1, b2, eps):
    cov3d().adamUpdate(param, grad, exp_avg, exp_avg_sq, visible, lr, b1, b2, eps)
