"""GPU: the allocation-free propagation entry point matches the regular one and the oracle.

cvhrf_asm_propagate_noalloc serves callers that cannot allocate device memory
while they propagate (a frozen or exhausted pool, a plugin host that forbids
allocation in its execute callback, a real-time loop that must stay off the
allocator).  It keeps its scratch in one fixed array inside the library, so this
test calls it straight through the C ABI — no workspace, no plan — several times
in a row with different inputs and sizes, and checks each result against
cvhrf_asm_propagate and against the CPU oracle (oracle/asm_oracle.py) at the
propagation tolerance (1e-4 relative L2).  The calls cover the largest size the
fixed array holds (S = 512), a cropped output (Ho, Wo < S) and accumulation into a
prefilled output.  The file name sorts last so that a run stopping at the first
failure has run everything else.
"""
import ctypes
import math

import numpy as np
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


def _call(L, x, out, S, wl, dist, ap, accumulate):
    Hi, Wi = x.shape
    Ho, Wo = out.shape
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return L.cvhrf_asm_propagate_noalloc(ctypes.c_void_p(x.data_ptr()), Hi, Wi, ctypes.c_void_p(out.data_ptr()),
                                         Ho, Wo, S, wl, 8e-6, dist, ap, accumulate, stream)


CALLS = [  # (S, Hi, Wi, Ho, Wo, wavelength, distance, aperture, accumulate, seed)
    (384, 384, 320, 384, 384, 532e-9, 2e-3, 300.0, 0, 1),
    (200, 150, 200, 200, 200, 639e-9, -3e-3, -1.0, 0, 2),
    (512, 512, 512, 512, 512, 473e-9, 1e-3, -1.0, 0, 3),      # the largest size the array holds
    (256, 200, 256, 180, 240, 532e-9, -2e-3, 200.0, 0, 4),    # cropped output
    (128, 128, 96, 128, 128, 639e-9, 4e-3, -1.0, 1, 5),       # accumulate into a prefilled output
]


def test_noalloc_matches_regular_entry_point_and_oracle(cuda):
    from complex_valued_holographic_radiance_fields_b200 import _lib
    from complex_valued_holographic_radiance_fields_b200.propagation import propagate
    from oracle import asm_oracle as AO
    L = _lib.lib()
    for S, Hi, Wi, Ho, Wo, wl, dist, ap, acc, seed in CALLS:
        x = _field(Hi, Wi, seed)
        prefill = _field(Ho, Wo, seed + 100) if acc else None
        out = prefill.clone() if acc else torch.full((Ho, Wo), float("nan"), dtype=torch.complex64, device="cuda")
        rc = _call(L, x, out, S, wl, dist, ap, acc)
        assert rc == 0, L.cvhrf_status_string(rc)
        full = propagate(x, wl, 8e-6, dist, S, ap)              # the regular entry point (workspace + plan)
        oy, ox = (S - Ho) // 2, (S - Wo) // 2
        expected = full[oy:oy + Ho, ox:ox + Wo]
        if acc:
            expected = expected + prefill
        torch.cuda.synchronize()
        assert _rel(out, expected) < TOL, (S, Ho, Wo, acc)
        ye = AO.propagate(x.cpu().numpy(), wl, 8e-6, dist, S, ap, out_hw=(Ho, Wo))
        if acc:
            ye = ye + prefill.cpu().numpy()
        assert AO.rel_l2(out.cpu().numpy(), ye) < TOL, (S, Ho, Wo, acc)


def test_noalloc_second_identical_call_is_bitwise_repeatable(cuda):
    """The shared array keeps the previous call's contents; a call must not depend on them."""
    from complex_valued_holographic_radiance_fields_b200 import _lib
    L = _lib.lib()
    x = _field(300, 300, 7)
    outs = []
    for S in (320, 512, 320):     # a larger call in between leaves different bytes in the array
        out = torch.empty(S, S, dtype=torch.complex64, device="cuda")
        assert _call(L, x, out, S, 532e-9, 2e-3, -1.0, 0) == 0
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[2])


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch(cuda):
    from complex_valued_holographic_radiance_fields_b200 import _lib
    L = _lib.lib()
    x = _field(8, 8, 0)
    out = torch.empty(600, 600, dtype=torch.complex64, device="cuda")
    rc = L.cvhrf_asm_propagate_noalloc(ctypes.c_void_p(x.data_ptr()), 8, 8, ctypes.c_void_p(out.data_ptr()),
                                       600, 600, 600, 532e-9, 8e-6, 1e-3, -1.0, 0, None)
    assert rc == 4  # CVHRF_EUNSUPPORTED
