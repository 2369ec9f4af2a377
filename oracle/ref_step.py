"""The reference's own CUDA kernels (oracle/_ref, rebuilt for sm_100a) driving the
config-3 training step on the GPU (TEST INFRASTRUCTURE ONLY — timed as the
"reference kernels on B200" comparison in bench.py).

Glue mirrors the reference: Scene.splat (model.py:1178-1272) calls SplatTileCuda,
then BandlimitedPropagation once per (plane, channel) and sums the planes; the
optimizer is SparseGaussianAdam.step (utils/optimizer.py:180-265: index_select of
the visible gradient rows, then adamUpdate per group; 1-D groups dense torch Adam).
"""
import torch

from oracle import ref_harness as R


class RefGpuHoloStep:
    def __init__(self, trainer):
        self.t = trainer
        self.state = {k: (torch.zeros_like(v), torch.zeros_like(v)) for k, v in trainer.params.items()}

    def step(self):
        from complex_valued_holographic_radiance_fields_b200 import scene as SC
        t = self.t
        for p in t.params.values():
            p.grad = None
        kw, idxs = SC.render_inputs(t.params, t.camera)
        args = list(SC.splat_args(kw))
        args[12] = R.view_buffer(kw["view_matrix"])
        field, vis = R.RefSplatTileCuda.apply(*args)
        holo = 0
        for p in range(t.K):
            holo = holo + torch.stack([R.RefBandlimitedPropagationFunction.apply(
                field[p, c], t.wavelengths[c], t.pitch, t.prop_distances[p], [t.S, t.S], t.aperture)
                for c in range(len(t.wavelengths))])
        loss = ((holo.abs() ** 2 - t.target) ** 2).mean()
        loss.backward()
        visible = idxs[vis]
        self.last_visible = visible
        with torch.no_grad():
            for k, prm in t.params.items():
                m, v = self.state[k]
                if prm.dim() == 1:
                    m.mul_(0.9).add_(prm.grad, alpha=0.1)
                    v.mul_(0.999).addcmul_(prm.grad, prm.grad, value=0.001)
                    prm.addcdiv_(m, v.sqrt().add_(1e-15), value=-1e-3)
                else:
                    gv = torch.zeros(1, visible.shape[0], prm.shape[1], device=prm.device)
                    gv[0] = prm.grad.index_select(0, visible)
                    R.ref_adam_update(prm.data.view(1, *prm.shape), gv, m.view(1, *prm.shape),
                                      v.view(1, *prm.shape), visible, 1e-3, 0.9, 0.999, 1e-15)
        return loss.detach()
