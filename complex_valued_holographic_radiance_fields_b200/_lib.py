"""ctypes binding of ``libcvhrf.so`` (the C ABI declared in ``include/cvhrf.h``).

The CUDA library is the only implementation: if it is missing or cannot be
loaded, every operator raises instead of falling back to another path.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("CVHRF_LIB") or os.path.join(_HERE, "libcvhrf.so")
_lock = threading.Lock()
_lib = None

c_int, c_float, c_size_t, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p
c_float_p = ctypes.POINTER(ctypes.c_float)

# name -> (restype, argtypes); must match include/cvhrf.h
SIGNATURES = {
    "cvhrf_status_string": (ctypes.c_char_p, [c_int]),
    "cvhrf_last_cuda_error": (c_int, []),
    "cvhrf_version": (c_int, []),
    "cvhrf_kernel_launch_count": (ctypes.c_ulonglong, []),
    "cvhrf_asm_plan_create": (c_int, [c_int, ctypes.POINTER(c_void_p)]),
    "cvhrf_asm_plan_destroy": (c_int, [c_void_p]),
    "cvhrf_asm_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "cvhrf_asm_propagate": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_int,
                                    c_float, c_float, c_float, c_float, c_int, c_void_p, c_size_t, c_void_p]),
    "cvhrf_asm_propagate_planes": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float_p, c_float_p,
                                           c_float, c_float, c_void_p, c_void_p, c_size_t, c_void_p]),
    "cvhrf_asm_propagate_planes_adjoint": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float_p,
                                                   c_float_p, c_float, c_float, c_void_p, c_void_p, c_size_t,
                                                   c_void_p]),
    "cvhrf_asm_transfer_table_bytes": (c_size_t, [c_int, c_int, c_int]),
    "cvhrf_asm_transfer_table_build": (c_int, [c_void_p, c_int, c_int, c_float_p, c_float_p, c_float, c_float,
                                               c_void_p, c_void_p]),
    "cvhrf_asm_transfer_table_upload": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "cvhrf_asm_propagate_planes_table": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                                 c_void_p, c_size_t, c_void_p]),
    "cvhrf_asm_propagate_planes_adjoint_table": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                                         c_void_p, c_void_p, c_size_t, c_void_p]),
    "cvhrf_ssim_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "cvhrf_ssim_forward": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float, c_void_p, c_void_p,
                                   c_void_p, c_size_t, c_void_p]),
    "cvhrf_ssim_backward": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_size_t, c_void_p]),
    "cvhrf_adan": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "cvhrf_adan_clip_workspace_bytes": (c_size_t, []),
    "cvhrf_adan_clip_init_workspace": (c_int, [c_void_p, c_size_t, c_void_p]),
    "cvhrf_adan_clip_factor": (c_int, [c_void_p, c_int, c_float, c_float, c_void_p, c_void_p, c_size_t, c_void_p]),
    "cvhrf_sort_pairs_workspace_bytes": (c_size_t, [c_int]),
    "cvhrf_sort_pairs_u32": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "cvhrf_inclusive_scan_workspace_bytes": (c_size_t, [c_int]),
    "cvhrf_inclusive_scan_u32": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "cvhrf_lookback_timeouts": (c_int, []),
    "cvhrf_copy_wait_timeouts": (c_int, []),
    "cvhrf_intensity_loss_workspace_bytes": (c_size_t, [c_int]),
    "cvhrf_intensity_loss_init_workspace": (c_int, [c_void_p, c_size_t, c_void_p]),
    "cvhrf_intensity_loss": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "cvhrf_intensity_loss_backward": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "cvhrf_asm_propagate_noalloc": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_float,
                                            c_float, c_float, c_float, c_int, c_void_p]),
    "cvhrf_raster_geometry_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "cvhrf_raster_forward_geometry": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "cvhrf_raster_binning_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "cvhrf_raster_forward_render": (c_int, [c_void_p, c_void_p, c_size_t, c_int, c_int, c_void_p, c_size_t,
                                            c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "cvhrf_raster_forward_render_capacity": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_int, c_void_p,
                                                     c_size_t] + [c_void_p] * 8),
    "cvhrf_raster_backward_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "cvhrf_raster_backward": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_int, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_void_p, c_void_p, c_size_t] + [c_void_p] * 9),
    "cvhrf_scene_workspace_bytes": (c_size_t, [c_int]),
    "cvhrf_scene_prepare": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_float, c_void_p, c_size_t]
                            + [c_void_p] * 9 + [c_void_p]),
    "cvhrf_scene_prepare_owned": (c_int, [c_void_p, c_void_p, c_void_p, c_float, c_float, ctypes.c_uint32, c_void_p,
                                          c_size_t] + [c_void_p] * 9 + [c_void_p]),
    "cvhrf_scene_backward": (c_int, [c_void_p, c_void_p, c_void_p] + [c_void_p] * 14 + [c_void_p]),
    "cvhrf_sparse_adam": (c_int, [c_void_p, c_int, c_void_p, c_int, c_float, c_float, c_void_p]),
    "cvhrf_sparse_adam_masked": (c_int, [c_void_p, c_int, c_void_p, c_int, c_float, c_float, c_void_p]),
    "cvhrf_rows_to_mask": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p]),
    "cvhrf_hologram_field_workspace_bytes": (c_size_t, []),
    "cvhrf_hologram_field_init_workspace": (c_int, [c_void_p, c_size_t, c_void_p]),
    "cvhrf_hologram_field": (c_int, [c_void_p, c_int, ctypes.c_longlong, c_float_p, c_void_p, c_void_p, c_void_p,
                                     c_size_t, c_void_p]),
    "cvhrf_hologram_field_backward": (c_int, [c_void_p, c_int, ctypes.c_longlong, c_float_p, c_void_p, c_void_p,
                                              c_void_p, c_void_p, c_size_t, c_void_p]),
    "cvhrf_multiplane_loss_workspace_bytes": (c_size_t, []),
    "cvhrf_multiplane_loss_init_workspace": (c_int, [c_void_p, c_size_t, c_void_p]),
    "cvhrf_multiplane_loss": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float_p, c_void_p, c_void_p,
                                      c_float_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "cvhrf_multiplane_loss_backward": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_float_p, c_void_p,
                                               c_void_p, c_float_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "cvhrf_density_workspace_bytes": (c_size_t, [c_int]),
    "cvhrf_density_classify": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "cvhrf_density_apply": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "cvhrf_opacity_regularization": (c_int, [c_void_p, c_int, c_float, c_void_p, c_void_p]),
}


class AdamGroup(ctypes.Structure):
    """cvhrf_adam_group (include/cvhrf.h)."""
    _fields_ = [("param", c_void_p), ("grad", c_void_p), ("exp_avg", c_void_p), ("exp_avg_sq", c_void_p),
                ("N", c_int), ("D", c_int), ("dense", c_int), ("lr", c_float), ("eps", c_float)]


class AdanGroup(ctypes.Structure):
    """cvhrf_adan_group (include/cvhrf.h)."""
    _fields_ = [(n, c_void_p) for n in ("param", "grad", "exp_avg", "exp_avg_sq", "exp_avg_diff", "neg_pre_grad")] + \
               [("n", ctypes.c_longlong)] + \
               [(n, c_float) for n in ("beta1", "beta2", "beta3", "one_minus_beta1", "one_minus_beta2",
                                       "one_minus_beta3", "bias_correction3_sqrt", "eps", "step_size",
                                       "step_size_diff", "decay")] + \
               [("no_prox", c_int), ("first_step", c_int)]


class Gaussians(ctypes.Structure):
    """cvhrf_gaussians (include/cvhrf.h)."""
    _fields_ = [("N", c_int), ("K", c_int), ("C", c_int)] + \
               [(n, c_void_p) for n in ("means", "pre_quats", "pre_scales", "colours", "pre_phase", "pre_opac",
                                        "pre_planes")]


class GaussianSet(ctypes.Structure):
    """cvhrf_gaussian_set (include/cvhrf.h)."""
    _fields_ = [("N", c_int), ("K", c_int), ("C", c_int)] + \
               [(n, c_void_p) for n in ("means", "pre_quats", "pre_scales", "colours", "pre_phase", "pre_opac",
                                        "pre_planes", "grad_means", "grad_pre_quats", "grad_pre_scales",
                                        "grad_colours", "grad_pre_phase", "grad_pre_opac", "grad_pre_planes")]


class DensityParams(ctypes.Structure):
    """cvhrf_density_params (include/cvhrf.h)."""
    _fields_ = [(n, c_float) for n in ("grad_threshold", "opacity_threshold", "small_scale_threshold",
                                       "large_scale_threshold", "split_factor", "clone_offset_factor")]


class RasterScene(ctypes.Structure):
    """cvhrf_raster_scene (include/cvhrf.h)."""
    _fields_ = [(n, c_int) for n in ("N", "K", "C", "W", "H")] + \
               [(n, c_float) for n in ("fx", "fy", "px", "py", "near_plane", "far_plane")] + \
               [(n, c_void_p) for n in ("cam_means", "z_vals", "quats", "scales", "colours", "phase", "opacities",
                                        "plane_probs", "view_matrix")]


class CvhrfError(RuntimeError):
    pass


def lib():
    """Load (once) and return the CUDA library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise CvhrfError(
                    f"{LIB_PATH} is missing: build it with "
                    "`python -m complex_valued_holographic_radiance_fields_b200.build` (no CPU fallback exists)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(status, what):
    if status != 0:
        L = lib()
        msg = L.cvhrf_status_string(status).decode()
        raise CvhrfError(f"{what} failed: {msg} (status {status}, cuda error {L.cvhrf_last_cuda_error()})")


def float_array(values):
    vals = [float(v) for v in values]
    return (ctypes.c_float * len(vals))(*vals)
