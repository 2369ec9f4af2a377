"""GPU: the allocation-free propagation entry point matches the regular one.

cvhrf_asm_propagate_noalloc serves callers that cannot allocate device memory
while they propagate (a frozen or exhausted pool, a plugin host that forbids
allocation in its execute callback, a real-time loop that must stay off the
allocator).  It keeps its scratch in one fixed array inside the library, so this
test calls it straight through the C ABI — no workspace, no plan — twice in a row
with different inputs and sizes, and checks each result against
cvhrf_asm_propagate at the propagation tolerance (1e-4 relative L2).  The file
name sorts last so that a run stopping at the first failure has run everything else.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _field(H, W, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.polar(torch.rand(H, W, generator=g), torch.rand(H, W, generator=g) * 2 * math.pi).to(
        torch.complex64).cuda()


def _rel(a, b):
    a, b = a.to(torch.complex128), b.to(torch.complex128)
    return float((a - b).abs().pow(2).sum().sqrt() / b.abs().pow(2).sum().sqrt())


def test_noalloc_matches_regular_entry_point_twice(cuda):
    from complex_valued_holographic_radiance_fields_b200 import _lib
    from complex_valued_holographic_radiance_fields_b200.propagation import propagate
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    calls = [  # (S, Hi, Wi, wavelength, distance, aperture, seed)
        (384, 384, 320, 532e-9, 2e-3, 300.0, 1),
        (200, 150, 200, 639e-9, -3e-3, -1.0, 2),
    ]
    for S, Hi, Wi, wl, dist, ap, seed in calls:
        x = _field(Hi, Wi, seed)
        out = torch.full((S, S), float("nan"), dtype=torch.complex64, device="cuda")
        rc = L.cvhrf_asm_propagate_noalloc(ctypes.c_void_p(x.data_ptr()), Hi, Wi, ctypes.c_void_p(out.data_ptr()),
                                           S, S, S, wl, 8e-6, dist, ap, 0, stream)
        assert rc == 0, L.cvhrf_status_string(rc)
        expected = propagate(x, wl, 8e-6, dist, S, ap)
        torch.cuda.synchronize()
        assert _rel(out, expected) < TOL


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch(cuda):
    from complex_valued_holographic_radiance_fields_b200 import _lib
    L = _lib.lib()
    x = _field(8, 8, 0)
    out = torch.empty(600, 600, dtype=torch.complex64, device="cuda")
    rc = L.cvhrf_asm_propagate_noalloc(ctypes.c_void_p(x.data_ptr()), 8, 8, ctypes.c_void_p(out.data_ptr()),
                                       600, 600, 600, 532e-9, 8e-6, 1e-3, -1.0, 0, None)
    assert rc == 4  # CVHRF_EUNSUPPORTED
