"""The host-synchronisation-free rasterizer path and the CUDA-graph training iteration
give the same results as the eager path (same kernels, buffers sized by a capacity)."""
import pytest
import torch

from complex_valued_holographic_radiance_fields_b200 import rasterizer as RZ
from complex_valued_holographic_radiance_fields_b200 import scene as SC
from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer

pytestmark = pytest.mark.gpu


def _inputs(cuda, N=20000, K=3, W=160, H=128, seed=3):
    params = {k: v.requires_grad_(True)
              for k, v in SC.make_gaussians(N, K=K, C=3, seed=seed, device=cuda).items()}
    cam = SC.PinholeCamera(W, H)
    return params, cam


@pytest.mark.parametrize("headroom", [1.0, 2.0])
def test_capacity_forward_backward_matches_eager(cuda, headroom):
    params, cam = _inputs(cuda)
    kw, _ = SC.render_inputs_fused(params, cam)
    args = [a.detach().requires_grad_(a.requires_grad) if torch.is_tensor(a) else a for a in SC.splat_args(kw)]
    field, vis = RZ.SplatTileCuda.apply(*args)
    npairs = RZ.last_num_pairs
    g = torch.randn_like(field)
    ge = torch.autograd.grad(field, [a for a in args if torch.is_tensor(a) and a.requires_grad], g)
    cap = int(npairs * headroom)
    field_c, mask = RZ.SplatTileCudaCapacity.apply(*args, cap)
    assert int(RZ.last_overflow.item()) == 0
    gc = torch.autograd.grad(field_c, [a for a in args if torch.is_tensor(a) and a.requires_grad], g)
    assert torch.equal(field, field_c)
    m = torch.zeros(params["means"].shape[0], dtype=torch.uint8, device=cuda)
    m[vis.long()] = 1
    assert torch.equal(m, mask)
    for a, b in zip(ge, gc):
        assert torch.equal(a, b)


def test_capacity_overflow_is_flagged(cuda):
    params, cam = _inputs(cuda)
    kw, _ = SC.render_inputs_fused(params, cam)
    RZ.SplatTileCuda.apply(*SC.splat_args(kw))
    npairs = RZ.last_num_pairs
    assert npairs > 100
    _, mask = RZ.SplatTileCudaCapacity.apply(*SC.splat_args(kw), npairs // 2)
    torch.cuda.synchronize()
    assert int(RZ.last_overflow.item()) == 1
    _, mask = RZ.SplatTileCudaCapacity.apply(*SC.splat_args(kw), npairs)
    assert int(RZ.last_overflow.item()) == 0


def _trainer(cuda):
    return HoloTrainer(N=30000, W=128, H=128, K=3, device=cuda, seed=5)


def test_graph_iteration_matches_eager(cuda):
    a, b = _trainer(cuda), _trainer(cuda)
    b.capture(headroom=1.5, warmup=2)          # 3 eager-equivalent iterations before capture
    for _ in range(3):
        a.step()
    for it in range(3):
        la = a.step()
        lb = b.replay()
        torch.cuda.synchronize()
        assert torch.equal(la, lb), (it, la.item(), lb.item())
    assert not b.graph_overflowed()
    for k in a.params:
        assert torch.equal(a.params[k], b.params[k]), k
        sa, sb = a.opt.state[a.params[k]], b.opt.state[b.params[k]]
        assert torch.equal(sa["exp_avg"], sb["exp_avg"]), k
        assert torch.equal(sa["exp_avg_sq"], sb["exp_avg_sq"]), k
    assert b.graph_launches > 10


def test_graph_replay_with_new_target(cuda):
    a, b = _trainer(cuda), _trainer(cuda)
    b.capture(headroom=1.5, warmup=2)
    for _ in range(3):
        a.step()
    tgt = torch.rand_like(a.target)
    la = a.step(tgt)
    lb = b.replay(tgt)
    torch.cuda.synchronize()
    assert torch.equal(la, lb)


def test_train_from_host_matches_eager(cuda):
    a, b = _trainer(cuda), _trainer(cuda)
    b.capture(headroom=1.5, warmup=2)
    for _ in range(3):
        a.step()
    g = torch.Generator().manual_seed(9)
    targets = [torch.rand(a.target.shape, generator=g).pin_memory() for _ in range(4)]
    la = [a.step(t.to(cuda)).item() for t in targets]
    lb = b.train_from_host(targets)
    assert la == lb
    for k in a.params:
        assert torch.equal(a.params[k], b.params[k]), k


def test_multiview_graph_matches_eager(cuda):
    import math
    from complex_valued_holographic_radiance_fields_b200.train_step import MultiViewTrainer
    cams = [SC.look_at_camera(96, 80, 2 * math.pi * v / 3, 0.3 * (v - 1)) for v in range(3)]
    kw = dict(N=20000, W=96, H=80, K=3, S=96, device=cuda, seed=6, cameras=cams)
    a, b = MultiViewTrainer(**kw), MultiViewTrainer(**kw)
    b.capture(headroom=1.5, warmup=2)
    for _ in range(3):
        a.step()
    for _ in range(2):
        la, lb = a.step(), b.replay()
        torch.cuda.synchronize()
        assert torch.equal(la, lb)
    assert not b.graph_overflowed()
    for k in a.params:
        assert torch.equal(a.params[k], b.params[k]), k
