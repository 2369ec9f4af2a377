"""Data parallelism over camera views (one process per GPU, torch.distributed/NCCL).

Each rank renders and back-propagates its own view against a full replica of the
Gaussians.  Before the sparse Adam step the ranks exchange exactly two things:

* the dense per-Gaussian gradients, flattened into ONE buffer and summed with a
  single all-reduce (17 + K floats per Gaussian: means 3, scales 3, quats 4,
  colours C, phase C, opacity 1, plane logits K);
* the set of rows any rank saw (a uint8 mask, all-reduce MAX).

Every rank then applies the identical Adam update, so replicas stay bit-identical.
The reference has no multi-GPU path; this is the view-parallel design of its
training loop (train.py:230-324 runs one view per iteration).
"""
import torch
import torch.distributed as dist


def allreduce_gradients_and_visibility(params, visible_rows, n_rows, group=None):
    """Sum .grad of every tensor in `params` (dict) across ranks; return the union of visible rows."""
    grads = [p.grad for p in params.values()]
    flat = torch.cat([g.reshape(-1) for g in grads])
    mask = torch.zeros(n_rows, dtype=torch.uint8, device=flat.device)
    mask[visible_rows] = 1
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(mask, op=dist.ReduceOp.MAX, group=group)
    off = 0
    for p, g in zip(params.values(), grads):
        n = g.numel()
        p.grad = flat[off:off + n].view_as(g)
        off += n
    return torch.nonzero(mask, as_tuple=False).squeeze(1)


def _shared_flat_buffer(params):
    """The flat buffer all .grad tensors are views of (FusedRenderInputs backward), or None."""
    from .scene import FusedRenderInputs
    flat = getattr(FusedRenderInputs, "last_grad_buffer", None)
    if flat is None:
        return None
    base = flat.untyped_storage().data_ptr()
    total = 0
    for p in params.values():
        if p.grad is None or p.grad.untyped_storage().data_ptr() != base:
            return None
        total += p.grad.numel()
    return flat if total == flat.numel() else None


class _AllReduceSum(torch.autograd.Function):
    """Sum of a tensor over the ranks; its gradient is the incoming gradient itself (the
    summed tensor feeds an identical computation on every rank, so every rank receives
    the same upstream gradient)."""

    @staticmethod
    def forward(ctx, x, group):
        y = x.contiguous().clone()
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


def all_reduce_sum(x, group=None):
    """Differentiable all-reduce (sum) across the process group."""
    return _AllReduceSum.apply(x, group)


def exchange_and_step(trainer, visible, group=None):
    """Sum the gradients and union the visible rows across ranks, then step the optimizer.
    Ranks that produced no gradients (nothing rendered) contribute zeros."""
    from . import _lib
    import ctypes
    n = trainer.params["means"].shape[0]
    dev = trainer.params["means"].device
    if any(p.grad is None for p in trainer.params.values()):
        total = sum(p.numel() for p in trainer.params.values())
        flat = torch.zeros(total, dtype=torch.float32, device=dev)
        off = 0
        for p in trainer.params.values():
            if p.grad is None:
                p.grad = flat[off:off + p.numel()].view_as(p)
            else:
                flat[off:off + p.numel()].copy_(p.grad.reshape(-1))
                p.grad = flat[off:off + p.numel()].view_as(p)
            off += p.numel()
    else:
        flat = _shared_flat_buffer(trainer.params)
        if flat is None:
            rows = allreduce_gradients_and_visibility(trainer.params, visible, n, group)
            trainer.opt.step(rows)
            return
    mask = torch.empty(n, dtype=torch.uint8, device=dev)
    vis = visible.to(torch.int64).contiguous()
    _lib.check(_lib.lib().cvhrf_rows_to_mask(ctypes.c_void_p(vis.data_ptr()), vis.numel(),
                                             ctypes.c_void_p(mask.data_ptr()), n,
                                             ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)),
               "cvhrf_rows_to_mask")
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(mask, op=dist.ReduceOp.MAX, group=group)
    trainer.opt.step(row_mask=mask)


def dp_step(trainer, target=None, group=None):
    """One view-parallel training iteration on `trainer` (a HoloTrainer).

    The gradients are summed with one in-place all-reduce of the flat buffer they share
    and the visible rows with one all-reduce (MAX) of a row mask that goes straight to
    the masked sparse Adam, so the exchange needs no copy and no host synchronisation.
    """
    from . import _lib
    import ctypes
    for p in trainer.params.values():
        p.grad = None
    loss, visible = trainer.forward(target)
    loss.backward()
    n = trainer.params["means"].shape[0]
    flat = _shared_flat_buffer(trainer.params)
    if flat is None:  # gradients not in one buffer: fall back to the concatenating exchange
        visible = allreduce_gradients_and_visibility(trainer.params, visible, n, group)
        trainer.opt.step(visible)
        return loss.detach()
    mask = torch.empty(n, dtype=torch.uint8, device=flat.device)
    vis = visible.to(torch.int64).contiguous()
    _lib.check(_lib.lib().cvhrf_rows_to_mask(ctypes.c_void_p(vis.data_ptr()), vis.numel(),
                                             ctypes.c_void_p(mask.data_ptr()), n,
                                             ctypes.c_void_p(torch.cuda.current_stream(flat.device).cuda_stream)),
               "cvhrf_rows_to_mask")
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(mask, op=dist.ReduceOp.MAX, group=group)
    trainer.opt.step(row_mask=mask)
    return loss.detach()


def graph_exchange(group=None):
    """The exchange of `dp_step` as a callback for `HoloTrainer.capture(exchange=...)`:
    both all-reduces are recorded into the trainer's CUDA graph (NCCL supports capture)."""
    def exchange(trainer, row_mask):
        flat = _shared_flat_buffer(trainer.params)
        if flat is None:
            raise RuntimeError("graph capture needs the gradients in one flat buffer (render_inputs_fused)")
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(row_mask, op=dist.ReduceOp.MAX, group=group)
        return row_mask
    return exchange
