"""One training iteration of the hot path (train.py:230-324 restated).

    render (model.py:1365-1416)   -> splat_tile_cuda           (libcvhrf rasterizer)
    per-plane propagation + sum   -> propagate_planes          (libcvhrf fused FFT/ASM)
    loss = mean((|holo|^2 - target)^2)   -> intensity_l2_loss         (libcvhrf, 2 launches)
    backward                      -> libcvhrf adjoints
    SparseGaussianAdam.step(visible)                            (libcvhrf fused Adam)

Optics follow train.py:839-865 with the config's overrides: wavelengths 639/532/473 nm,
planes at linspace(-V/2, V/2, K) + d_val (V = 4 mm, d_val = -2 mm -> -4, -2, 0 mm for
K = 3), each plane propagated by -d_p (model.py:1259), pad_size = aperture = max(W, H),
pixel pitch 8 um (the config's value; the script default is 3.74 um).

``capture()`` records one whole iteration (forward, backward, optimizer) in a CUDA graph
through the host-synchronisation-free rasterizer path (fixed pair capacity, visibility as
a row mask); ``replay()`` then runs an iteration with a single graph launch.  A device
flag records whether any replayed iteration needed more pairs than the capacity
(``graph_overflowed()``); such an iteration's outputs are invalid and the caller
re-captures with a larger capacity.

The reference optimizer receives the rasterizer's ``visible_indices``, which index the
depth-sorted subset, not the parameter rows; here they are mapped back through the
sort permutation (``idxs[visible]``) so the update lands on the rows that were seen.
"""
import torch

from . import scene as SC
from .density import density_control, opacity_regularization
from .loss import intensity_l2_loss
from .optimizer import Adan, SparseGaussianAdam
from .propagation import propagate_planes
from .reconstruction import MultiplaneLoss, Propagator, hologram_training_loss
from . import rasterizer as RZ
from .rasterizer import SplatTileCudaCapacity, splat_tile_cuda

WAVELENGTHS = [639e-9, 532e-9, 473e-9]


def plane_distances(K, volume_depth=4e-3, d_val=-2e-3):
    if K == 1:
        return torch.tensor([d_val], dtype=torch.float32)
    return torch.linspace(-volume_depth / 2.0, volume_depth / 2.0, K) + d_val


class HoloTrainer:
    def __init__(self, N=300000, W=800, H=800, K=3, pitch=8e-6, lr=1e-3, eps=1e-15, seed=0, device="cuda",
                 camera=None, wavelengths=None, target=None, S=None, frustum=None, optimizer="sparse_adam",
                 loss="l2", image=None, depth=None):
        self.device = torch.device(device)
        self.W, self.H, self.K = W, H, K
        self.S = S or max(W, H)   # pad size (train.py: max(W, H) unless configured)
        self.aperture = float(self.S)
        self.pitch = pitch
        self.wavelengths = list(wavelengths or WAVELENGTHS)
        d = plane_distances(K)
        self.prop_distances = [float(-d[p]) for p in range(K)]
        self.camera = camera or SC.PinholeCamera(W, H)
        self.params = {k: v.requires_grad_(True) for k, v in
                       SC.make_gaussians(N, K=K, C=len(self.wavelengths), seed=seed, device=self.device,
                                         frustum=frustum).items()}
        if optimizer not in ("adan", "sparse_adam"):
            raise ValueError(f"unknown optimizer {optimizer!r}")
        self.optimizer, self.lr, self.eps = optimizer, lr, eps
        self.opt = self._make_optimizer()
        if loss not in ("l2", "multiplane"):
            raise ValueError(f"unknown loss {loss!r}")
        self.loss_mode = loss
        if loss == "multiplane":
            # the training script's loss (train.py:256-304): the hologram is reconstructed at
            # every depth (utils/propagator.py, configured as train.py:868-883) and scored
            # against defocus-blurred multiplane targets (utils/data_utils.py:244-259)
            C = len(self.wavelengths)
            self.propagator = Propagator(resolution=[self.S, self.S], wavelengths=self.wavelengths,
                                         pixel_pitch=pitch, number_of_frames=C, number_of_depth_layers=K,
                                         volume_depth=4e-3, image_location_offset=-2e-3,
                                         propagator_type="forward", laser_channel_power=torch.eye(C),
                                         aperture_size=self.aperture, device=self.device)
            if target is None:
                g = torch.Generator().manual_seed(1)
                image = torch.rand(C, H, W, generator=g) if image is None else image
                depth = torch.rand(1, H, W, generator=g) if depth is None else depth
                ml = MultiplaneLoss(image, depth, target_blur_size=20, number_of_planes=K, blur_ratio=8,
                                    weights=[1.0, 1.0, 1.0, 0.0], scheme="defocus", reduction="mean",
                                    device=self.device)
                targets, masks, _ = ml.get_targets()
                target = torch.stack([targets, masks])   # 2 x K x C x H x W: targets, masks
        elif target is None:
            g = torch.Generator().manual_seed(1)
            target = torch.rand(len(self.wavelengths), self.S, self.S, generator=g)
        self.target = target.to(self.device)

    def _make_optimizer(self):
        if self.optimizer == "adan":
            # the reference training script's optimizer and per-group learning rates
            # (utils/optimizer.py:44-65); dense, eager steps only (its scalars change every step)
            lrs = {"pre_act_scales": 0.005, "pre_act_phase": 0.0025, "colours": 0.0025, "means": self.lr,
                   "pre_act_opacities": 0.025, "pre_act_plane_assignment": self.lr, "pre_act_quats": 0.001}
            return Adan([{"params": [p], "lr": lrs[k]} for k, p in self.params.items()], lr=0, eps=1e-8)
        return SparseGaussianAdam([{"params": [p], "lr": self.lr} for p in self.params.values()], lr=self.lr,
                                  eps=self.eps)

    def densify(self, grad_threshold=0.000005, decrease_amount=0.001, **kw):
        """The densification block of train.py:327-337, after an optimizer step: density
        control (clone / split / prune from the last step's gradients), opacity
        regularisation, and a new optimizer whose per-parameter state is carried over only
        where the shape did not change (utils/optimizer.py:67-101).  A captured graph is
        dropped (the Gaussian count changed); call capture() again.  Returns the counts."""
        old_params, old_opt = self.params, self.opt
        self.params, counts = density_control(old_params, grad_threshold=grad_threshold, **kw)
        counts["affected"] = opacity_regularization(self.params, decrease_amount)
        self.opt = self._make_optimizer()
        for k, p in self.params.items():
            q = old_params[k]
            if p.shape == q.shape and q in old_opt.state:
                self.opt.state[p] = old_opt.state[q]
        self.graph = None
        return counts

    # The planes this trainer renders: all of them here; a plane-parallel trainer
    # (PlaneShardedTrainer) renders its share and sums the holograms across GPUs.
    planes = None
    owned_mask = 0xFFFFFFFF

    def _render_inputs(self):
        kw, idxs = SC.render_inputs_fused(self.params, self.camera, self.owned_mask)
        if self.planes is not None:
            kw["plane_probs"] = kw["plane_probs"].index_select(1, self._plane_idx)
        return kw, idxs

    def _hologram(self, field):
        ds = self.prop_distances if self.planes is None else [self.prop_distances[p] for p in self.planes]
        return self._combine(propagate_planes(field, self.wavelengths, ds, self.pitch, self.S, self.aperture))

    def _combine(self, holo):
        return holo

    def _loss(self, holo, target):
        if self.loss_mode == "multiplane":
            return hologram_training_loss(self.propagator, holo, target[0], target[1])
        return intensity_l2_loss(holo, target)

    def forward(self, target=None):
        kw, idxs = self._render_inputs()
        field, visible = splat_tile_cuda(*SC.splat_args(kw))
        holo = self._hologram(field)
        tgt = self.target if target is None else target
        loss = self._loss(holo, tgt)
        return loss, idxs[visible]

    def step(self, target=None):
        for p in self.params.values():
            p.grad = None
        loss, visible = self.forward(target)
        loss.backward()
        if self.optimizer == "adan":
            self.opt.step()
        else:
            self.opt.step(visible)
        return loss.detach()

    # ---- CUDA-graph mode ------------------------------------------------------------
    def _forward_capacity(self, target):
        kw, idxs = self._render_inputs()
        field, vis_mask = SplatTileCudaCapacity.apply(*SC.splat_args(kw), self.pairs_capacity)
        holo = self._hologram(field)
        loss = self._loss(holo, target)
        n = self.params["means"].shape[0]
        row_mask = torch.zeros(n, dtype=torch.uint8, device=self.device)
        row_mask.scatter_(0, idxs, vis_mask)
        torch.maximum(self._overflow_acc, RZ.last_overflow, out=self._overflow_acc)
        return loss, row_mask

    def _step_capacity(self, exchange=None):
        for p in self.params.values():
            p.grad = None
        loss, row_mask = self._forward_capacity(self._static_target)
        loss.backward()
        if exchange is not None:
            row_mask = exchange(self, row_mask)
        self.opt.step(row_mask=row_mask)
        return loss.detach()

    def capture(self, headroom=1.5, exchange=None, warmup=2, eager_step=None):
        """Capture one iteration in a CUDA graph (runs `warmup` + 1 eager iterations first,
        which train like normal steps).  The pair capacity is `headroom` x the pair count
        of an eager iteration.  `exchange(trainer, row_mask) -> row_mask` is called between
        backward and optimizer (the data-parallel gradient exchange); `eager_step` replaces
        the first (eager) iteration, e.g. with its data-parallel form."""
        (eager_step or self.step)()
        self.pairs_capacity = int(RZ.last_num_pairs * headroom) + 4096
        self._static_target = self.target.clone()
        self._overflow_acc = torch.zeros(1, dtype=torch.int32, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._step_capacity(exchange)
        torch.cuda.current_stream(self.device).wait_stream(side)
        self._overflow_acc.zero_()
        self.graph = torch.cuda.CUDAGraph()
        launches0 = RZ._lib.lib().cvhrf_kernel_launch_count()
        with torch.cuda.graph(self.graph):
            self._static_loss = self._step_capacity(exchange)
        self.graph_launches = RZ._lib.lib().cvhrf_kernel_launch_count() - launches0
        return self

    def replay(self, target=None):
        """One iteration through the captured graph; returns the (static) loss tensor."""
        if target is not None:
            self._static_target.copy_(target, non_blocking=True)
        self.graph.replay()
        return self._static_loss

    def train_from_host(self, host_targets):
        """One captured iteration per target in `host_targets` (CPU tensors, ideally pinned),
        returning each iteration's loss as a host float.  Pipelined so the GPU never waits
        on the host: the next target's host->device copy runs on a side stream during the
        current iteration, each iteration starts with a device-to-device copy of its target
        into the graph's input buffer, its loss is copied to pinned host memory right after
        it, and the host reads loss i once iteration i + 1 has been queued."""
        dev = self.device
        main = torch.cuda.current_stream(dev)
        side = getattr(self, "_copy_stream", None)
        if side is None:
            side = self._copy_stream = torch.cuda.Stream(dev)
            self._staging = torch.empty_like(self._static_target)
        targets = list(host_targets)
        n = len(targets)
        # pinned loss slots and events are kept between calls (allocating pinned memory costs)
        if getattr(self, "_host_loss", None) is None or self._host_loss.numel() < 2:
            self._host_loss = torch.empty(2, dtype=torch.float32, pin_memory=True)
            self._done = [torch.cuda.Event(), torch.cuda.Event()]
            self._ready, self._consumed = torch.cuda.Event(), torch.cuda.Event()
        host_loss, done, ready, consumed = self._host_loss, self._done, self._ready, self._consumed
        losses = []
        side.wait_stream(main)
        if n:
            with torch.cuda.stream(side):
                self._staging.copy_(targets[0], non_blocking=True)
                ready.record(side)
        for i in range(n):
            main.wait_event(ready)
            self._static_target.copy_(self._staging, non_blocking=True)
            consumed.record(main)
            if i + 1 < n:
                with torch.cuda.stream(side):
                    side.wait_event(consumed)
                    self._staging.copy_(targets[i + 1], non_blocking=True)
                    ready.record(side)
            self.graph.replay()
            host_loss[i % 2].copy_(self._static_loss, non_blocking=True)
            done[i % 2].record(main)
            if i >= 1:
                done[(i - 1) % 2].synchronize()
                losses.append(float(host_loss[(i - 1) % 2]))
        if n:
            done[(n - 1) % 2].synchronize()
            losses.append(float(host_loss[(n - 1) % 2]))
        return losses

    def graph_overflowed(self):
        """True if any replay since capture exceeded the pair capacity (synchronises)."""
        return bool(self._overflow_acc.item())


class PlaneShardedTrainer(HoloTrainer):
    """Plane-parallel training (one process per GPU): GPU r renders, propagates and
    back-propagates only the planes it owns (p % world == rank) and the Gaussians whose
    one-hot plane is one of them; the per-channel holograms are summed across GPUs with
    one all-reduce before the loss (whose gradient is then the same on every GPU), and
    the Gaussian gradients (disjoint between GPUs: each Gaussian lives on one plane) and
    the visibility masks are combined before the identical sparse Adam step.  With one
    process it is the plain trainer.  A GPU that owns no plane (world > K) contributes
    zeros.  Parameters must be identical on every rank (same seed)."""

    def __init__(self, *args, rank=0, world=1, group=None, **kw):
        super().__init__(*args, **kw)
        self.rank, self.world, self.group = rank, world, group
        self.planes = [p for p in range(self.K) if p % world == rank]
        self.owned_mask = sum(1 << p for p in self.planes)
        self._plane_idx = torch.tensor(self.planes, dtype=torch.long, device=self.device)

    def _combine(self, holo):
        import torch.distributed as dist
        if self.world == 1 or not dist.is_initialized():
            return holo
        from .distributed import all_reduce_sum
        return all_reduce_sum(holo, self.group)

    def forward(self, target=None):
        if self.planes:
            return super().forward(target)
        from .distributed import all_reduce_sum
        C = len(self.wavelengths)
        # the zeros take part in autograd so that loss.backward() runs on this rank as on the
        # others (its Gaussian gradients stay absent and are sent as zeros in the exchange)
        zeros = torch.zeros((C, self.S, self.S), dtype=torch.complex64, device=self.device, requires_grad=True)
        holo = all_reduce_sum(zeros, self.group)
        loss = self._loss(holo, self.target if target is None else target)
        return loss, torch.empty(0, dtype=torch.long, device=self.device)

    def step(self, target=None):
        from .distributed import exchange_and_step
        for p in self.params.values():
            p.grad = None
        loss, visible = self.forward(target)
        loss.backward()
        import torch.distributed as dist
        if self.world > 1 and dist.is_initialized():
            exchange_and_step(self, visible, self.group)
        else:
            self.opt.step(visible)
        return loss.detach()


class MultiViewTrainer(HoloTrainer):
    """Multi-view training (config 4): one iteration trains on every camera in `cameras`
    (one seeded target per view), accumulating the Gaussian gradients over the views before
    one sparse Adam step.  With N processes (one per GPU) the views are split across them
    (rank r takes views r, r + N, ...) and the gradients and visibility masks are summed
    with the same exchange as view-parallel training, so an iteration does the same work
    at any N (strong scaling).  Eager (`step`) and graph-captured (`capture` + `replay`)."""

    def __init__(self, *args, cameras, rank=0, world=1, group=None, **kw):
        super().__init__(*args, camera=cameras[0], **kw)
        self.cameras = list(cameras)
        self.rank, self.world, self.group = rank, world, group
        self.views = list(range(rank, len(self.cameras), world))
        C = len(self.wavelengths)
        self.view_targets = []
        for v in range(len(self.cameras)):
            g = torch.Generator().manual_seed(1000 + v)
            self.view_targets.append(torch.rand(C, self.S, self.S, generator=g).to(self.device))
        self.max_pairs = 0

    def _exchange(self, flat, mask):
        import torch.distributed as dist
        if self.world > 1 and dist.is_initialized():
            dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
            dist.all_reduce(mask, op=dist.ReduceOp.MAX, group=self.group)

    def _views(self, capacity):
        n = self.params["means"].shape[0]
        mask = torch.zeros(n, dtype=torch.uint8, device=self.device)
        flat, total = None, None
        for v in self.views:
            self.camera = self.cameras[v]
            if capacity:
                loss, m = self._forward_capacity(self.view_targets[v])
            else:
                loss, visible = self.forward(self.view_targets[v])
                self.max_pairs = max(self.max_pairs, RZ.last_num_pairs)
                m = torch.zeros(n, dtype=torch.uint8, device=self.device)
                m[visible] = 1
            loss.backward()   # gradients accumulate in place into the first view's buffer
            if flat is None:
                flat = SC.FusedRenderInputs.last_grad_buffer
            torch.maximum(mask, m, out=mask)
            total = loss.detach() if total is None else total + loss.detach()
        if flat is None:  # no views on this rank: contribute zeros
            flat = torch.zeros(sum(p.numel() for p in self.params.values()), device=self.device)
            off = 0
            for p in self.params.values():
                p.grad = flat[off:off + p.numel()].view_as(p)
                off += p.numel()
            total = torch.zeros((), device=self.device)
        self._exchange(flat, mask)
        self.opt.step(row_mask=mask)
        return total / max(len(self.views), 1)

    def step(self, target=None):
        for p in self.params.values():
            p.grad = None
        return self._views(capacity=False)

    def _step_capacity(self, exchange=None):
        for p in self.params.values():
            p.grad = None
        return self._views(capacity=True)

    def capture(self, headroom=1.5, exchange=None, warmup=2, eager_step=None):
        self.step()
        self.pairs_capacity = int(self.max_pairs * headroom) + 4096
        self._static_target = self.view_targets[0]
        self._overflow_acc = torch.zeros(1, dtype=torch.int32, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._step_capacity()
        torch.cuda.current_stream(self.device).wait_stream(side)
        self._overflow_acc.zero_()
        self.graph = torch.cuda.CUDAGraph()
        launches0 = RZ._lib.lib().cvhrf_kernel_launch_count()
        with torch.cuda.graph(self.graph):
            self._static_loss = self._step_capacity()
        self.graph_launches = RZ._lib.lib().cvhrf_kernel_launch_count() - launches0
        return self
