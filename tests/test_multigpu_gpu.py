"""Two-GPU (NCCL) checks, skipped with fewer than two GPUs: view-parallel steps captured in
a CUDA graph keep the replicas bit-identical, and plane-parallel steps match one-GPU
training with the same seed."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _checksum(params):
    return torch.stack([p.detach().double().sum() for p in params.values()])


def _worker(rank, world, port, q):
    import math
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    from complex_valued_holographic_radiance_fields_b200 import scene as SC
    from complex_valued_holographic_radiance_fields_b200.distributed import dp_step, graph_exchange
    from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer, PlaneShardedTrainer
    out = {}
    # view-parallel, graph-captured
    cam = SC.look_at_camera(128, 128, 2 * math.pi * rank / world, 0.0)
    tr = HoloTrainer(N=20000, W=128, H=128, K=3, device=dev, camera=cam, seed=3)
    tr.capture(headroom=1.5, exchange=graph_exchange(), warmup=2, eager_step=lambda: dp_step(tr))
    for _ in range(3):
        tr.replay()
    torch.cuda.synchronize()
    cs = _checksum(tr.params)
    allcs = [torch.zeros_like(cs) for _ in range(world)]
    dist.all_gather(allcs, cs)
    out["dp_equal"] = all(torch.equal(allcs[0], c) for c in allcs)
    out["dp_overflow"] = tr.graph_overflowed()
    # plane-parallel
    pt = PlaneShardedTrainer(N=20000, W=128, H=96, K=3, S=128, device=dev, seed=5, rank=rank, world=world)
    losses = [pt.step().item() for _ in range(3)]
    cs = _checksum(pt.params)
    allcs = [torch.zeros_like(cs) for _ in range(world)]
    dist.all_gather(allcs, cs)
    out["planes_equal"] = all(torch.equal(allcs[0], c) for c in allcs)
    if rank == 0:
        ref = HoloTrainer(N=20000, W=128, H=96, K=3, S=128, device=dev, seed=5)
        ref_losses = [ref.step().item() for _ in range(3)]
        out["loss_err"] = max(abs(a - b) / abs(b) for a, b in zip(losses, ref_losses))
        out["param_err"] = max(float((pt.params[k] - ref.params[k]).detach().norm() / ref.params[k].detach().norm())
                               for k in ref.params)
    q.put((rank, out))
    q.close()
    q.join_thread()
    torch.cuda.synchronize()
    # leave without tearing down the communicator (it is referenced by a captured graph)
    os._exit(0)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_view_and_plane_parallel():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        if p.exitcode is None:
            p.kill()
    for r, out in res.items():
        assert out["dp_equal"] and not out["dp_overflow"], out
        assert out["planes_equal"], out
    assert res[0]["loss_err"] < 1e-5, res[0]
    assert res[0]["param_err"] < 1e-3, res[0]   # Adam normalises: near-zero gradients amplify rounding
    assert all(p.exitcode == 0 for p in ps)


def _idle_rank_worker(port, q):
    """One process, NCCL world of 1, a plane-parallel trainer that owns no plane (the case of
    a GPU beyond the plane count, e.g. K = 7 over 8 GPUs): its step must run the same
    collectives as an owning rank and leave the parameters unchanged (zero gradients)."""
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev)
    from complex_valued_holographic_radiance_fields_b200.train_step import PlaneShardedTrainer
    tr = PlaneShardedTrainer(N=5000, W=96, H=96, K=2, device=dev, rank=0, world=1)
    tr.planes, tr.owned_mask = [], 0
    tr.world = 2            # take the multi-rank exchange path (the group itself has one rank)
    before = {k: v.detach().clone() for k, v in tr.params.items()}
    loss = float(tr.step())
    torch.cuda.synchronize()
    same = all(torch.equal(before[k], v.detach()) for k, v in tr.params.items())
    dist.destroy_process_group()
    q.put((loss, same))


def test_rank_without_planes_steps(cuda):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_idle_rank_worker, args=(_free_port(), q))
    p.start()
    p.join(300)
    assert p.exitcode == 0
    loss, same = q.get(timeout=5)
    assert loss == loss and same
