"""Plane-parallel decomposition (PlaneShardedTrainer) on one GPU: the shards' fields are
the full render's planes bit for bit, their holograms sum to the full hologram, and their
Gaussian gradients sum to the full gradients (each Gaussian lives on one plane)."""
import pytest
import torch

from complex_valued_holographic_radiance_fields_b200 import scene as SC
from complex_valued_holographic_radiance_fields_b200.loss import intensity_l2_loss
from complex_valued_holographic_radiance_fields_b200.rasterizer import splat_tile_cuda
from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer, PlaneShardedTrainer

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = a.detach().double() if not a.is_complex() else torch.view_as_real(a.detach()).double()
    b = b.detach().double() if not b.is_complex() else torch.view_as_real(b.detach()).double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("K,world", [(3, 2), (5, 3), (2, 3)])
def test_plane_shards_sum_to_full_step(cuda, K, world):
    kw = dict(N=20000, W=128, H=96, K=K, S=128, seed=7, device=cuda)
    full = HoloTrainer(**kw)
    shards = [PlaneShardedTrainer(rank=r, world=world, **kw) for r in range(world)]
    kin, idxs = full._render_inputs()
    field, vis = splat_tile_cuda(*SC.splat_args(kin))
    holo = full._hologram(field)
    holo_sum, visible = None, torch.zeros(kw["N"], dtype=torch.bool, device=cuda)
    for t in shards:
        if not t.planes:
            continue
        kr, ir = t._render_inputs()
        fr, vr = splat_tile_cuda(*SC.splat_args(kr))
        assert torch.equal(fr, field[t.planes])
        hr = t._hologram(fr)          # world == 1 combine: no collective in this emulation
        holo_sum = hr if holo_sum is None else holo_sum + hr
        visible[ir[vr]] = True
    assert rel(holo_sum, holo) < 1e-6
    full_vis = torch.zeros_like(visible)
    full_vis[idxs[vis]] = True
    assert torch.equal(visible, full_vis)
    intensity_l2_loss(holo, full.target).backward()
    intensity_l2_loss(holo_sum, full.target).backward()
    for k, p in full.params.items():
        g = sum(t.params[k].grad for t in shards if t.planes)
        assert rel(g, p.grad) < 1e-5, k
