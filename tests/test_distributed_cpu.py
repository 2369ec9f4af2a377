"""CPU (gloo, world_size 2): the view-parallel gradient exchange used before sparse Adam."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from complex_valued_holographic_radiance_fields_b200.distributed import allreduce_gradients_and_visibility
    torch.manual_seed(rank)
    params = {"a": torch.zeros(6, 3, requires_grad=True), "b": torch.zeros(6, requires_grad=True)}
    params["a"].grad = torch.full((6, 3), float(rank + 1))
    params["b"].grad = torch.arange(6, dtype=torch.float32) * (rank + 1)
    vis = torch.tensor([rank, 4]) if rank == 0 else torch.tensor([2, 4])
    u = allreduce_gradients_and_visibility(params, vis, 6)
    q.put((rank, params["a"].grad.tolist(), params["b"].grad.tolist(), u.tolist()))
    dist.destroy_process_group()


def test_allreduce_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, a, b, u in res:
        assert a == [[3.0] * 3] * 6
        assert b == [float(3 * i) for i in range(6)]
        assert u == [0, 2, 4]


def _worker_allreduce_sum(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from complex_valued_holographic_radiance_fields_b200.distributed import all_reduce_sum
    x = torch.full((4,), float(rank + 1), requires_grad=True)
    y = all_reduce_sum(x * 2.0)
    w = torch.arange(4, dtype=torch.float32)
    (y * w).sum().backward()
    q.put((rank, y.tolist(), x.grad.tolist()))
    dist.destroy_process_group()


def test_all_reduce_sum_autograd_two_ranks():
    """The plane-parallel hologram sum: forward sums over ranks, backward passes the
    (replicated) upstream gradient through unchanged."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker_allreduce_sum, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, y, g in res:
        assert y == [6.0] * 4
        assert g == [0.0, 2.0, 4.0, 6.0]


def test_plane_ownership():
    from complex_valued_holographic_radiance_fields_b200.train_step import PlaneShardedTrainer
    owned = [[p for p in range(7) if p % 8 == r] for r in range(8)]
    assert owned[7] == [] and sorted(sum(owned, [])) == list(range(7))
    assert PlaneShardedTrainer.__mro__[1].__name__ == "HoloTrainer"


def _worker_idle_rank(rank, world, port, q):
    """Rank 1 renders nothing (a GPU beyond the plane count): it contributes a zero hologram
    that takes part in autograd, so its loss.backward() runs like rank 0's and both ranks
    issue the same collectives (the hologram sum here)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from complex_valued_holographic_radiance_fields_b200.distributed import all_reduce_sum
    target = torch.ones(3)
    if rank == 0:
        field = torch.tensor([1.0, 2.0, 3.0], requires_grad=True)
        holo = all_reduce_sum(field * 2.0)
    else:
        field = torch.zeros(3, requires_grad=True)
        holo = all_reduce_sum(field)
    loss = ((holo - target) ** 2).mean()
    loss.backward()
    q.put((rank, holo.tolist(), float(loss), field.grad.tolist()))
    dist.destroy_process_group()


def test_idle_rank_backward_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker_idle_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, h0, l0, g0), (_, h1, l1, _) = res
    assert h0 == h1 == [2.0, 4.0, 6.0]
    assert l0 == l1
    expected = [2.0 * 2.0 * (2.0 * (i + 1) - 1.0) / 3.0 for i in range(3)]
    assert all(abs(a - b) <= 1e-6 * abs(b) for a, b in zip(g0, expected))
