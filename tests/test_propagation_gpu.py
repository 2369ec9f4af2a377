"""GPU parity of the fused ASM propagation against the oracle and the reference kernels.

Tolerance: complex fields within 1e-4 relative L2 (fp32).
"""
import math

import numpy as np
import pytest
import torch

from oracle import asm_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-4


def rand_field(H, W, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.rand(H, W, generator=g)
    ph = torch.rand(H, W, generator=g) * 2 * math.pi
    return torch.polar(a, ph).to(torch.complex64)


def rel(a, b):
    a = a.detach().to(torch.complex128).cpu()
    b = b.detach().to(torch.complex128).cpu() if torch.is_tensor(b) else torch.from_numpy(np.asarray(b)).to(torch.complex128)
    return float((a - b).abs().pow(2).sum().sqrt() / b.abs().pow(2).sum().sqrt().clamp_min(1e-30))


@pytest.mark.parametrize("S,H,W", [(8, 8, 8), (16, 12, 16), (40, 40, 30), (60, 60, 60), (96, 64, 96),
                                   (120, 100, 120), (128, 128, 128)])
@pytest.mark.parametrize("dist", [-2e-3, 0.0, 3e-3])
def test_propagate_vs_oracle_small(cuda, S, H, W, dist):
    from complex_valued_holographic_radiance_fields_b200 import propagation as P
    f = rand_field(H, W, seed=S)
    for wl in (639e-9, 473e-9):
        for ap in (-1.0, S * 0.8):
            out = P.propagate(f.to(cuda), wl, 8e-6, dist, S, ap)
            exp = O.propagate(f.numpy(), wl, 8e-6, dist, S, ap)
            assert rel(out, exp) < TOL, (S, H, W, dist, wl, ap)


@pytest.mark.parametrize("S,H,W", [(800, 800, 800), (1024, 1024, 1024), (1920, 1080, 1920)])
def test_propagate_vs_oracle_config_sizes(cuda, S, H, W):
    from complex_valued_holographic_radiance_fields_b200 import propagation as P
    f = rand_field(H, W, seed=1)
    out = P.propagate(f.to(cuda), 532e-9, 8e-6, -2e-3, S, -1.0)
    exp = O.propagate(f.numpy(), 532e-9, 8e-6, -2e-3, S, -1.0)
    assert rel(out, exp) < TOL


def test_adjoint_identity(cuda):
    """<A x, y> == <x, A^H y> for the fused forward/backward (backward = exact adjoint)."""
    from complex_valued_holographic_radiance_fields_b200 import propagation as P
    S, H, W = 96, 80, 96
    x = rand_field(H, W, 3).to(cuda)
    y = rand_field(S, S, 4).to(cuda)
    Ax = P.propagate(x, 532e-9, 8e-6, 2e-3, S)
    AHy = P.propagate(y, 532e-9, 8e-6, -2e-3, S, out_hw=(H, W))
    lhs = torch.vdot(y.flatten().to(torch.complex128), Ax.flatten().to(torch.complex128))
    rhs = torch.vdot(AHy.flatten().to(torch.complex128), x.flatten().to(torch.complex128))
    assert abs(lhs - rhs) / abs(lhs) < 1e-5


@pytest.mark.parametrize("S,H,W,dist,ap", [(1024, 1024, 1024, -2e-3, -1.0), (1024, 1024, 1024, 2e-3, -1.0),
                                           (1024, 1024, 1024, 0.0, -1.0), (800, 800, 800, 4e-3, 800.0),
                                           (64, 48, 64, 1e-3, 40.0)])
def test_forward_backward_vs_reference(cuda, ref, S, H, W, dist, ap):
    from complex_valued_holographic_radiance_fields_b200 import propagation as P
    f = rand_field(H, W, seed=7).to(cuda)
    for wl in (639e-9, 532e-9, 473e-9):
        a = f.clone().requires_grad_(True)
        b = f.clone().requires_grad_(True)
        out = P.BandlimitedPropagationFunction.apply(a, wl, 8e-6, dist, [S, S], ap)
        exp = ref.RefBandlimitedPropagationFunction.apply(b, wl, 8e-6, dist, [S, S], ap)
        assert rel(out, exp) < TOL
        g = rand_field(S, S, seed=9).to(cuda)
        out.backward(g)
        exp.backward(g)
        assert rel(a.grad, b.grad) < TOL


def test_planes_vs_per_call(cuda):
    from complex_valued_holographic_radiance_fields_b200 import propagation as P
    K, C, H, W, S = 3, 3, 80, 80, 80
    fields = torch.stack([torch.stack([rand_field(H, W, 10 * p + c) for c in range(C)]) for p in range(K)]).to(cuda)
    wl = [639e-9, 532e-9, 473e-9]
    ds = [4e-3, 2e-3, 0.0]
    fr = fields.clone().requires_grad_(True)
    holo = P.propagate_planes(fr, wl, ds, 8e-6, S, float(S))
    exp = torch.stack([sum(P.propagate(fields[p, c], wl[c], 8e-6, ds[p], S, float(S)) for p in range(K))
                       for c in range(C)])
    assert rel(holo, exp) < TOL
    g = torch.stack([rand_field(S, S, 50 + c) for c in range(C)]).to(cuda)
    holo.backward(g)
    exp_g = torch.stack([torch.stack([P.propagate(g[c], wl[c], 8e-6, -ds[p], S, float(S), out_hw=(H, W))
                                      for c in range(C)]) for p in range(K)])
    assert rel(fr.grad, exp_g) < TOL


@pytest.mark.parametrize("S,H,W,K,C", [(64, 48, 64, 2, 1), (128, 100, 128, 3, 3), (256, 256, 200, 1, 2),
                                       (800, 800, 800, 3, 3)])
@pytest.mark.parametrize("ap", [-1.0, None])
def test_planes_table_matches_per_call_transfer(cuda, S, H, W, K, C, ap):
    """Precomputed transfer table (K forward + 1 inverse column transforms per channel)
    against the per-call evaluation (one forward + inverse per plane), forward and adjoint."""
    from complex_valued_holographic_radiance_fields_b200 import propagation as P
    ap = float(S) if ap is None else ap
    fields = torch.stack([torch.stack([rand_field(H, W, 7 * p + c) for c in range(C)]) for p in range(K)]).to(cuda)
    wl = [639e-9, 532e-9, 473e-9][:C]
    ds = [4e-3, 2e-3, 0.0][:K]
    g = torch.stack([rand_field(S, S, 90 + c) for c in range(C)]).to(cuda)
    out = []
    for use_table in (True, False):
        fr = fields.clone().requires_grad_(True)
        holo = P.propagate_planes(fr, wl, ds, 8e-6, S, ap, use_table=use_table)
        holo.backward(g)
        out.append((holo.detach(), fr.grad))
    assert P.transfer_table(S, K, C, wl, ds, 8e-6, ap, cuda) is not None
    assert rel(out[0][0], out[1][0]) < 1e-5
    assert rel(out[0][1], out[1][1]) < 1e-5


@pytest.mark.parametrize("S,H,W,dist,ap", [(64, 48, 64, -2e-3, -1.0), (256, 200, 256, 3e-3, 100.0),
                                           (1024, 1024, 1024, 2e-3, -1.0), (800, 800, 800, 0.0, 800.0)])
def test_single_propagate_table_matches_per_call(cuda, S, H, W, dist, ap):
    """propagate() reads a cached transfer table for the S x S output (forward) and the S x S
    input (backward): same results as evaluating the transfer function in the call."""
    from complex_valued_holographic_radiance_fields_b200.propagation import propagate
    x = rand_field(H, W, seed=3).to(cuda)
    a = propagate(x, 532e-9, 8e-6, dist, S, ap, use_table=True)
    b = propagate(x, 532e-9, 8e-6, dist, S, ap, use_table=False)
    assert rel(a, b) <= 1e-5
    g = rand_field(S, S, seed=4).to(cuda)
    a = propagate(g, 532e-9, 8e-6, -dist, S, ap, out_hw=(H, W), use_table=True)
    b = propagate(g, 532e-9, 8e-6, -dist, S, ap, out_hw=(H, W), use_table=False)
    assert rel(a, b) <= 1e-5


@pytest.mark.parametrize("S,H,W,K,C", [(64, 64, 48, 3, 3), (64, 48, 64, 9, 1), (128, 128, 100, 12, 2),
                                       (120, 120, 120, 10, 3), (800, 800, 800, 3, 3)])
@pytest.mark.parametrize("use_table", [False, True])
def test_planes_vs_oracle(cuda, S, H, W, K, C, use_table):
    """The fused K-plane sum and its adjoint against the numpy oracle directly, including
    more planes per channel than the compile-time column pass sums (K > 8), which runs
    the runtime mixed-radix plan at a compile-time size."""
    from complex_valued_holographic_radiance_fields_b200 import propagation as P
    fields = torch.stack([torch.stack([rand_field(H, W, 31 * p + c) for c in range(C)]) for p in range(K)])
    wl = [639e-9, 532e-9, 473e-9][:C]
    ds = [(-4e-3 + 0.9e-3 * p) for p in range(K)]
    fr = fields.to(cuda).requires_grad_(True)
    holo = P.propagate_planes(fr, wl, ds, 8e-6, S, float(S), use_table=use_table)
    f_np = fields.numpy()
    for c in range(C):
        exp = sum(O.propagate(f_np[p, c], wl[c], 8e-6, ds[p], S, float(S)).astype(np.complex128) for p in range(K))
        assert rel(holo[c], exp) < TOL, (c,)
    g = torch.stack([rand_field(S, S, 70 + c) for c in range(C)])
    holo.backward(g.to(cuda))
    g_np = g.numpy()
    for p in (0, K - 1):
        for c in range(C):
            exp_g = O.propagate(g_np[c], wl[c], 8e-6, -ds[p], S, float(S), out_hw=(H, W))
            assert rel(fr.grad[p, c], exp_g) < TOL, (p, c)


def test_no_copy_wait_timeouts(cuda):
    """The column passes' bulk-copy waits never ran out of their limit in this process."""
    from complex_valued_holographic_radiance_fields_b200 import _lib
    from complex_valued_holographic_radiance_fields_b200 import propagation as P
    x = rand_field(800, 800, 3).to(cuda)
    P.propagate(x, 532e-9, 8e-6, 1e-3, 800, 800.0)
    torch.cuda.synchronize()
    assert _lib.lib().cvhrf_copy_wait_timeouts() == 0
