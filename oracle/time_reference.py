"""Time the reference's own CUDA kernels on one GPU (TEST INFRASTRUCTURE ONLY).

Times the reference's components, one JSON line each:

* B3: Rasterizer.forward at config 2 (100k Gaussians, 800x800, K = 3);
* B4: the reference propagation (torch.fft cuFFT + bandlimited_propagation_{forward,backward},
  python_function.py:109-218 glue) per call, forward and backward, at config 1 (S = 1024),
  config 3 (S = 800) and config 4 (S = 1920, field 1080x1920);
* B5: the full config-3 training step on the reference kernels (oracle/ref_step.py);
* B6: adamUpdate (conv.cu:1230-1246) over the 6 two-dimensional parameter groups of config 3
  (the 1-D opacity group is a dense torch Adam in the reference), all rows visible.

With CVHRF_REF_DIR=oracle/_ref80 (built by `python oracle/build_ref.py --ptx80`) the same
runs use the compute_80 PTX build JIT-compiled by the driver (B7).  Times are CUDA events,
median of `--steps` after `--warmup`; one JSON line per measurement.

usage: python oracle/time_reference.py [--steps 20] [--warmup 5]
"""
import argparse
import json
import math
import os
import statistics
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def _median_ms(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def _field(H, W, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.polar(torch.rand(H, W, generator=g), torch.rand(H, W, generator=g) * 2 * math.pi).to(
        torch.complex64).cuda()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args()
    from oracle import ref_harness as R
    from complex_valued_holographic_radiance_fields_b200 import scene as SC
    build = "compute_80 PTX (JIT)" if os.environ.get("CVHRF_REF_DIR") else "sm_100a"
    out = lambda d: print(json.dumps(dict(d, build=build)), flush=True)  # noqa: E731

    # B3: rasterizer forward, config 2
    params = SC.make_gaussians(100000, K=3, C=3, seed=0, device="cuda")
    kw, _ = SC.render_inputs(params, SC.PinholeCamera(800, 800))
    args = list(SC.splat_args({k: (v.detach() if torch.is_tensor(v) else v) for k, v in kw.items()}))
    args[12] = R.view_buffer(args[12])
    ms = _median_ms(lambda: R.RefSplatTileCuda.apply(*args), a.steps, a.warmup)
    out({"row": "B3", "what": "Rasterizer.forward, config 2", "ms": ms})

    # B4: propagation per call
    F = R.RefBandlimitedPropagationFunction
    for name, H, W, S in (("config 1", 1024, 1024, 1024), ("config 3", 800, 800, 800), ("config 4", 1080, 1920, 1920)):
        x = _field(H, W, 0).requires_grad_(True)
        g = _field(S, S, 1)
        fwd = _median_ms(lambda: F.apply(x, 532e-9, 8e-6, 2e-3, [S, S], float(S)), a.steps, a.warmup)

        def fb():
            y = F.apply(x, 532e-9, 8e-6, 2e-3, [S, S], float(S))
            y.backward(g)
        both = _median_ms(fb, a.steps, a.warmup)
        out({"row": "B4", "what": f"propagation per call, {name} (S={S}, field {H}x{W})", "fwd_ms": fwd,
             "bwd_ms": both - fwd})
        del x, g

    # B5: full config-3 step
    from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer
    from oracle.ref_step import RefGpuHoloStep
    tr = HoloTrainer(N=300000, W=800, H=800, K=3, device="cuda")
    rs = RefGpuHoloStep(tr)
    ms = _median_ms(rs.step, a.steps, a.warmup)
    out({"row": "B5", "what": "full config-3 training step", "ms": ms, "iters_per_s": 1000.0 / ms})

    # B6: adamUpdate over the config-3 groups, every row visible
    n = 300000
    vis = torch.arange(n, device="cuda", dtype=torch.int64)
    groups = []
    for d in (3, 4, 3, 3, 3, 3):   # means, quats, scales, colours, phase, plane logits (K = 3)
        p = torch.randn(1, n, d, device="cuda")
        groups.append((p, torch.randn(1, n, d, device="cuda"), torch.zeros_like(p), torch.zeros_like(p)))

    def adam():
        for p, gr, m, v in groups:
            R.ref_adam_update(p, gr, m, v, vis, 1e-3, 0.9, 0.999, 1e-15)
    ms = _median_ms(adam, a.steps, a.warmup)
    nbytes = n * 19 * 28 + 6 * n * 8   # 2-D groups (19 floats per row): p, g, m, v read; p, m, v written
    out({"row": "B6", "what": "adamUpdate, 6 two-dimensional groups of config 3, all rows", "ms": ms,
         "GBps": nbytes / (ms * 1e-3) / 1e9})


if __name__ == "__main__":
    main()
