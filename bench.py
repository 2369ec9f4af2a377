"""Benchmark: training iterations/sec of the wave-optics hot path.

One step = render 300k Gaussians into K=3 complex planes at 800x800 (libcvhrf
rasterizer), propagate every (plane, channel) to the SLM with 2x padding and sum
(libcvhrf fused FFT/ASM), L2 intensity loss against a seeded target, backward
through both, sparse Adam over the visible Gaussians (libcvhrf fused Adam).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]

N > 1 (launched by torch.distributed.run, one rank per GPU) is view-parallel weak
scaling: each rank renders its own camera view of the same scene with a full
replica, gradients are all-reduced over NCCL before Adam; `value` is the whole-job
number of view-iterations per second.

`--impl reference` times the reference's CPU implementation of the path (the
oracle port: scalar-C rasterizer restatement on all host cores + the reference's
pure-torch propagation on torch CPU) on rank 0, and, beside it, the reference's own
CUDA kernels rebuilt for sm_100a on this GPU (field `reference_cuda_sm100a`).
"""
import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train iters/sec (fwd+bwd+sparse Adam) @300k Gaussians, 800x800, K=3"
N_GAUSS, IMG, K_PLANES = 300000, 800, 3
CONFIG = {"workload": "config3: full training step, 300k Gaussians, 800x800, K=3 planes, 3 wavelengths, "
                      "2x-padded ASM propagation (1600^2) at 8 um, L2 intensity loss, sparse Adam",
          "gaussians": N_GAUSS, "image": [IMG, IMG], "planes": K_PLANES, "pad": 2 * IMG,
          "l2_policy": "inputs larger than L2 (per-step working set > 300 MB)"}

METRIC_MP = "train iters/sec (fwd+bwd+sparse Adam, multiplane reconstruction loss) @300k Gaussians, 800x800, K=3"
CONFIG_MP = dict(CONFIG, workload="config3mp: the config-3 step with the training script's loss (train.py:280-304): "
                                  "the hologram reconstructed at the 3 depths and scored with the defocus multiplane "
                                  "loss plus SSIM, instead of the L2 intensity loss")


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        if os.environ.get("CVHRF_BENCH_NO_CLOCKS"):
            return self
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def fp32_peak_tflops(sm_mhz):
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    return props.multi_processor_count * 128 * 2 * sm_mhz * 1e6 / 1e12


# arithmetic of the reference's per-(pixel, Gaussian) backward body (backward_splat.cu:184-300)
# for C = 3, counted once: power 6, alpha 3, T 2, 3 channels x 21, alpha/geometry/conic/cov 36.
# Only a contributing evaluation (power <= 0 and alpha >= 1/255) runs that body; any other
# evaluation of a (pixel, Gaussian) pair of the tile lists stops after the offset, the
# quadratic form and the alpha test (about 10 FLOP).  The share of contributing evaluations
# among the 256 x pairs was counted once with the CVHRF_BWD_STATS build of
# render_backward_kernel at this workload (87,050,739 of 632,232,960;
# profiles/ncu_render_backward_config3.md).
BWD_FLOP_PER_EVAL = 110
BWD_FLOP_PER_SKIPPED_EVAL = 10
BWD_CONTRIB_FRACTION = 87050739 / 632232960
# FMA-pipe utilisation of render_backward_kernel<3> measured by ncu at this workload (same file)
BWD_FMA_PIPE_PCT = 36.9
# dram__bytes_read.sum + dram__bytes_write.sum of render_backward_kernel<3> at this workload
# (profiles/ncu_render_backward_config3.md)
BWD_NCU_TRAFFIC = 283.5e6
# the same for the forward propagation's three kernels (fs_rows_fwd, fs_cols_sum, fs_rows_inv;
# profiles/ncu_propagation_config3.md)
PROP_NCU_TRAFFIC = 417.0e6


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def propagation_bytes(K, C, H, W, S):
    """Algorithmic HBM bytes of one fused multi-plane propagation forward (the kernels as built):
    rows: read K C H W, write K C H P; columns (K planes summed on chip): read K C H P, write C S P;
    inverse rows: read C S P, write C S S  (complex64 = 8 B, P = 2 S)."""
    P = 2 * S
    return 8 * (K * C * H * W + 2 * K * C * H * P + 2 * C * S * P + C * S * S)


def run_mine(args, world, rank, local):
    from complex_valued_holographic_radiance_fields_b200 import _lib, scene as SC
    from complex_valued_holographic_radiance_fields_b200.distributed import dp_step
    from complex_valued_holographic_radiance_fields_b200.profiling import op_timing
    from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer
    import math

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cam = SC.look_at_camera(IMG, IMG, 2 * math.pi * rank / max(world, 1), 0.0) if world > 1 else None
    multiplane = args.workload == "config3mp"
    tr = HoloTrainer(N=N_GAUSS, W=IMG, H=IMG, K=K_PLANES, device=dev, camera=cam,
                     loss="multiplane" if multiplane else "l2")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    graph = os.environ.get("CVHRF_BENCH_EAGER", "0") != "1"
    sampler = ClockSampler(local)   # sampling starts with the warm-up so the loaded period is covered
    sampler.__enter__()
    L = _lib.lib()
    if graph:
        # one CUDA graph per iteration (forward, backward, exchange, optimizer); capture()
        # runs eager warm-up iterations itself, then W replays warm the graph
        from complex_valued_holographic_radiance_fields_b200.distributed import graph_exchange
        ex = graph_exchange() if world > 1 else None
        tr.capture(headroom=1.5, exchange=ex, warmup=2,
                   eager_step=(lambda: dp_step(tr)) if world > 1 else None)
        step = tr.replay
    else:
        step = (lambda t=None: dp_step(tr, t)) if world > 1 else (lambda t=None: tr.step(t))
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # --- device-timed region: inputs resident in HBM ---
    barrier()
    launches0 = L.cvhrf_kernel_launch_count()
    with contextlib.nullcontext() if graph else op_timing() as ops:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        h0 = time.perf_counter()
        for _ in range(args.steps):
            loss = step()
        host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
        t1.record()
        barrier()
    sampler.__exit__()
    launches = L.cvhrf_kernel_launch_count() - launches0
    if graph:
        launches = tr.graph_launches * args.steps   # replays launch the captured kernels
        if tr.graph_overflowed():
            raise RuntimeError("pair capacity exceeded during the timed replays; raise the headroom")
        # per-operator device times (roofline) from a few eager iterations, outside the timed region
        with op_timing() as ops:
            for _ in range(3):
                (dp_step(tr) if world > 1 else tr.step())
        barrier()
    ms = t0.elapsed_time(t1) / args.steps
    opsum = ops.summary()
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())

    # --- end to end: target H2D from pinned host memory + loss D2H every step ---
    host_tgt = tr.target.cpu().pin_memory()
    dev_tgt = torch.empty_like(tr.target)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    if graph:
        # every step: host->device copy of its target (pipelined on a side stream) and a
        # device->host read of its loss, through the trainer's public entry point
        tr.train_from_host([host_tgt] * args.steps)
    else:
        for _ in range(args.steps):
            dev_tgt.copy_(host_tgt, non_blocking=True)
            float(step(dev_tgt).item())
    e1.record()
    barrier()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    if rank != 0:
        return None
    clocks = sampler.summary()
    hbm, hbm_src = peaks()
    # roofline of the dominant operator
    dom = max(opsum.items(), key=lambda kv: kv[1][1])
    prop_ms = opsum.get("propagation_forward", (1, float("nan")))[1]
    pbytes = propagation_bytes(K_PLANES, 3, IMG, IMG, IMG)
    roof_prop = {"op": "propagation_forward (3 fused FFT/ASM kernels)", "bound": "hbm",
                 "achieved": pbytes / (prop_ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                 "peak_source": hbm_src, "algorithmic_bytes": pbytes, "traffic": PROP_NCU_TRAFFIC}
    roof_prop["frac"] = roof_prop["achieved"] / hbm
    # dominant operator: the rasterizer backward, bound by the FP32 pipe (not HBM, not tensor cores)
    from complex_valued_holographic_radiance_fields_b200 import rasterizer as RZ
    evals = 256.0 * RZ.last_num_pairs          # pixel x (tile, Gaussian) pair evaluations, one plane each
    contrib = evals * BWD_CONTRIB_FRACTION
    bwd_flop = contrib * BWD_FLOP_PER_EVAL + (evals - contrib) * BWD_FLOP_PER_SKIPPED_EVAL
    bwd_ms = opsum.get("raster_backward", (1, float("nan")))[1]
    sm_mhz = clocks.get("sm_mhz") or 1965.0
    peak_tf = fp32_peak_tflops(sm_mhz)
    roof = {"op": "raster_backward (render_backward_kernel + gaussian_grad_kernel)", "bound": "fp32",
            "achieved": bwd_flop / (bwd_ms * 1e-3) / 1e12, "peak": peak_tf, "unit": "TFLOP/s",
            "peak_source": f"SMs x 128 FMA lanes x 2 x median SM clock {sm_mhz:.0f} MHz (no tensor-core work)",
            "algorithmic_flop": bwd_flop,
            "work_unit": (f"{BWD_FLOP_PER_EVAL} FLOP per contributing pixel-Gaussian evaluation "
                          f"({BWD_CONTRIB_FRACTION:.4f} of 256 x {RZ.last_num_pairs} pairs), "
                          f"{BWD_FLOP_PER_SKIPPED_EVAL} per other evaluation"),
            "fma_pipe_pct_ncu": BWD_FMA_PIPE_PCT,
            "traffic": BWD_NCU_TRAFFIC}
    roof["frac"] = roof["achieved"] / peak_tf
    line = {
        "metric": METRIC_MP if multiplane else METRIC, "value": world * 1000.0 / ms_max, "unit": "iters/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32/c64", "data": "synthetic (seeded, config-3 shapes)",
        "config": dict(CONFIG_MP if multiplane else CONFIG, parallelism=f"view-dp{world}" if world > 1 else "single"),
        "e2e": {"value": world * 1000.0 / e2e_ms, "unit": "iters/s",
                "h2d_bytes_per_step": host_tgt.numel() * 4, "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches),
        "host_issue_ms_per_step": round(host_ms, 4),
        "execution": "cuda_graph (one replay per iteration; pair capacity %d)" % tr.pairs_capacity if graph
                     else "eager",
        "ops_ms": {k: round(v[1], 4) for k, v in opsum.items()},
        "dominant_op": dom[0],
        "roofline": roof,
        "roofline_propagation": roof_prop,
        "clocks": clocks,
        "loss": float(loss.item()),
    }
    return line


def cpu_baseline(samples=3, warmup=1):
    """The config-3 step on the host cores: `warmup` untimed steps, then the median of
    `samples` timed ones."""
    from oracle.cpu_step import CpuHoloStep, num_threads
    st = CpuHoloStep(N=N_GAUSS, W=IMG, H=IMG, K=K_PLANES)
    for _ in range(warmup):
        st.step()
    ts = []
    for _ in range(samples):
        t = time.perf_counter()
        st.step()
        ts.append(time.perf_counter() - t)
    v = 1.0 / statistics.median(ts)
    return {"value": v, "unit": "iters/s", "cores": num_threads(), "kind": "port",
            "sample": f"{warmup} warm-up + {samples} timed full config-3 step(s) (median) on the host: "
                      "oracle/raster_oracle.c (OpenMP) rasterizer fwd/bwd + the reference's pure-torch propagation "
                      "(python_function.py:35-78) on torch CPU + torch Adam",
            "ms_per_step_samples": [round(t * 1e3, 1) for t in ts]}


def ref_cuda_step_rate(steps, warmup):
    """The reference's own kernels (oracle/_ref, sm_100a rebuild) on this GPU, same step.
    Its steps allocate fresh tensors whose sizes change every step (the pair count), and
    some steps take several times the typical time in the allocator; so both the mean
    throughput over the timed steps and the median step time are reported."""
    from oracle import ref_harness
    if not ref_harness.available():
        return {"unavailable": "oracle/_ref not built"}
    from oracle.ref_step import RefGpuHoloStep
    from complex_valued_holographic_radiance_fields_b200.train_step import HoloTrainer
    tr = HoloTrainer(N=N_GAUSS, W=IMG, H=IMG, K=K_PLANES, device="cuda")
    rs = RefGpuHoloStep(tr)
    for _ in range(warmup):
        rs.step()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        rs.step()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    mean = sum(times) / len(times)
    med = statistics.median(times)
    return {"value": 1000.0 / mean, "unit": "iters/s", "ms_per_step": mean, "median_ms_per_step": med,
            "value_at_median": 1000.0 / med, "steps": steps,
            "what": "reference CUDA kernels (cov3d_cuda + cuda_modules, rebuilt sm_100a) + cuFFT, same step"}


METRIC5 = "train iters/sec (fwd+bwd+sparse Adam) @1M Gaussians, 1008x756, K=7, planes sharded over GPUs"
CONFIG5 = {"workload": "config5: full training step, 1M Gaussians in a depth-[1,10] frustum, 1008x756, K=7 planes, "
                       "3 wavelengths, 2x-padded ASM propagation (2048^2) at 8 um, L2 intensity loss, sparse Adam",
           "gaussians": 1000000, "image": [1008, 756], "planes": 7, "pad": 2048,
           "l2_policy": "inputs larger than L2"}


def run_config5(args, world, rank, local):
    """Plane-parallel config 5 (strong scaling: one training iteration split over the GPUs by plane)."""
    import math
    from complex_valued_holographic_radiance_fields_b200 import _lib, scene as SC
    from complex_valued_holographic_radiance_fields_b200.train_step import PlaneShardedTrainer
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    W, H = 1008, 756
    cam = SC.PinholeCamera(W, H)
    ht = math.tan(cam.fov / 2.0)
    tr = PlaneShardedTrainer(N=1000000, W=W, H=H, K=7, S=1024, device=dev, camera=cam, rank=rank, world=world,
                             frustum=(1.0, 10.0, ht, ht * H / W, -5.0, 0.7, 4.0))
    for _ in range(args.warmup):
        tr.step()
    L = _lib.lib()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    l0 = L.cvhrf_kernel_launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        loss = tr.step()
    t1.record()
    barrier()
    ms = torch.tensor([t0.elapsed_time(t1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    if rank != 0:
        return None
    return {"metric": METRIC5, "value": 1000.0 / ms, "unit": "iters/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32/c64", "data": "synthetic (seeded, config-5 shapes)",
            "config": dict(CONFIG5, parallelism=f"plane-shard{world}", planes_on_rank0=tr.planes),
            "execution": "eager", "gpu_launches": int(L.cvhrf_kernel_launch_count() - l0),
            "loss": float(loss.item())}


METRIC4 = "train iters/sec (8 views per iteration, fwd+bwd+sparse Adam) @500k Gaussians, 1920x1080, K=3"
CONFIG4 = {"workload": "config4: one iteration = 8 look-at views (radius 4, azimuths 2 pi v / 8, elevation +-20 deg), "
                       "500k Gaussians, 1920x1080, K=3 planes, 3 wavelengths, 2x-padded ASM propagation (3840^2) at "
                       "8 um, L2 intensity loss per view, gradients summed, one sparse Adam step",
           "gaussians": 500000, "image": [1920, 1080], "planes": 3, "pad": 3840, "views": 8,
           "l2_policy": "inputs larger than L2"}


def run_config4(args, world, rank, local):
    """Multi-view config 4 (strong scaling: the 8 views of an iteration split over the GPUs)."""
    import math
    from complex_valued_holographic_radiance_fields_b200 import scene as SC
    from complex_valued_holographic_radiance_fields_b200.train_step import MultiViewTrainer
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    W, H = 1920, 1080
    cams = [SC.look_at_camera(W, H, 2 * math.pi * v / 8, math.radians(20.0 if v % 2 == 0 else -20.0))
            for v in range(8)]
    tr = MultiViewTrainer(N=500000, W=W, H=H, K=3, S=1920, device=dev, cameras=cams, rank=rank, world=world)
    graph = os.environ.get("CVHRF_BENCH_EAGER", "0") != "1"
    if graph:
        tr.capture(headroom=1.5, warmup=2)
        step = tr.replay
    else:
        step = tr.step
    for _ in range(args.warmup):
        step()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        loss = step()
    t1.record()
    barrier()
    if graph and tr.graph_overflowed():
        raise RuntimeError("pair capacity exceeded during the timed replays")
    ms = torch.tensor([t0.elapsed_time(t1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    if rank != 0:
        return None
    return {"metric": METRIC4, "value": 1000.0 / ms, "unit": "iters/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32/c64", "data": "synthetic (seeded, config-4 shapes)",
            "config": dict(CONFIG4, parallelism=f"view-shard{world}", views_on_rank0=tr.views),
            "execution": "cuda_graph" if graph else "eager", "loss": float(loss.item())}


def run_reference(args, world, rank):
    """The reference arm: the config-3 step on the host cores (the reference's CPU path),
    `--warmup` untimed steps then exactly `--steps` timed ones, with the same metric and
    config as this build's line; the reference's CUDA kernels rebuilt for sm_100a are timed
    beside it on this GPU."""
    if rank != 0:
        return None
    from oracle.cpu_step import CpuHoloStep, num_threads
    st = CpuHoloStep(N=N_GAUSS, W=IMG, H=IMG, K=K_PLANES)
    for _ in range(args.warmup):
        st.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        st.step()
    ms = (time.perf_counter() - t0) * 1e3 / args.steps
    value = 1000.0 / ms
    base = {"value": value, "unit": "iters/s", "cores": num_threads(), "kind": "port",
            "sample": f"{args.warmup} warm-up + {args.steps} timed full config-3 steps on the host: "
                      "oracle/raster_oracle.c (OpenMP) rasterizer fwd/bwd + the reference's pure-torch "
                      "propagation (python_function.py:35-78) on torch CPU + torch Adam"}
    line = {"metric": METRIC, "value": value, "unit": "iters/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32/c64", "data": "synthetic (seeded, config-3 shapes)",
            "config": dict(CONFIG, parallelism=f"view-dp{world}" if world > 1 else "single"), "impl": "reference",
            "execution": "host cpu (rank 0 only)", "cpu_baseline": base,
            "e2e": {"value": value, "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if torch.cuda.is_available():
        try:
            line["reference_cuda_sm100a"] = ref_cuda_step_rate(max(min(args.steps, 20), 10), max(min(args.warmup, 5), 3))
        except Exception as e:  # the CPU number above stands on its own
            line["reference_cuda_sm100a"] = {"unavailable": repr(e)[:200]}
    return line


# ---- component workloads: config 1 (propagation alone), config 2 (rasterizer forward alone)
METRIC1 = "ASM propagations/s (one field 1024x1024 -> 2048^2 padded, lambda x d sweep)"
CONFIG1 = {"workload": "config1: 1024x1024 complex64 field (amplitude U[0,1], phase U[0,2pi), seed 0), S=1024 "
                       "(2048^2 padding), lambda in {639,532,473} nm x d in {-2,0,+2} mm, each P_d then P_-d: "
                       "18 single-field propagations per step, pitch 8 um, aperture off",
           "field": [1024, 1024], "pad": 2048, "calls_per_step": 18,
           "l2_policy": "inputs larger than L2 (each call streams 84 MB)"}
METRIC2 = "rasterizer forwards/s @100k Gaussians, 800x800, K=3"
CONFIG2 = {"workload": "config2: splat_tile_cuda forward alone (binning + render), 100k Gaussians, 800x800, K=3 "
                       "planes, C=3, means U[-1,1]^3 seen by a camera with R = I, T = (0, 0, 4) (seed 0)",
           "gaussians": 100000, "image": [800, 800], "planes": 3,
           "l2_policy": "field output 46 MB + binning arrays per call; L2 not flushed"}
FWD_FLOP_PER_EVAL = 32   # forward convention: d 2, conic 8, alpha and T 6, 3 channels x (re, im) FMA 12


def _config1_field():
    g = torch.Generator().manual_seed(0)
    a = torch.rand(1024, 1024, generator=g)
    ph = torch.rand(1024, 1024, generator=g) * 2 * math.pi
    return torch.polar(a, ph).to(torch.complex64)


CONFIG1_CALLS = [(wl, d) for wl in (639e-9, 532e-9, 473e-9) for d in (-2e-3, 0.0, 2e-3)]


def _timed_loop(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / steps


def _base_line(metric, config, value, ms, unit, args, world):
    return {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32/c64", "data": "synthetic (seeded)",
            "config": dict(config, parallelism=f"replicas{world}" if world > 1 else "single")}


def run_config1(args, world, rank, local):
    from complex_valued_holographic_radiance_fields_b200 import _lib
    from complex_valued_holographic_radiance_fields_b200.propagation import propagate
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    S = 1024
    x = _config1_field().to(dev)
    buf = [torch.empty(S, S, dtype=torch.complex64, device=dev) for _ in range(2)]

    def step(src=None):
        src = x if src is None else src
        for wl, d in CONFIG1_CALLS:
            propagate(src, wl, 8e-6, d, S, -1.0, out=buf[0])
            propagate(buf[0], wl, 8e-6, -d, S, -1.0, out=buf[1])
        return buf[1]

    # device throughput: the 18 calls captured once in a CUDA graph and replayed, so the
    # host-side cost of 18 separate Python calls (the e2e number below keeps it) is not timed
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    L = _lib.lib()
    n0 = L.cvhrf_kernel_launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    per_step_launches = L.cvhrf_kernel_launch_count() - n0
    sampler = ClockSampler(local)
    sampler.__enter__()
    ms = _timed_loop(graph.replay, args.steps, args.warmup)
    sampler.__exit__()
    launches = per_step_launches * args.steps
    # end to end through the eager API: the field from pinned host memory and the last output
    # back, every step
    host_in = x.cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    dev_in = torch.empty_like(x)

    def e2e_step():
        dev_in.copy_(host_in, non_blocking=True)
        host_out.copy_(step(dev_in), non_blocking=True)

    e2e_ms = _timed_loop(e2e_step, args.steps, 2)
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
    if rank != 0:
        return None
    calls = len(CONFIG1_CALLS) * 2
    hbm, src = peaks()
    per_call = 8 * S * S + 16 * S * 2 * S + 16 * S * 2 * S + 8 * S * S   # row, column, inverse-row passes
    achieved = per_call * calls / (ms * 1e-3) / 1e9
    line = _base_line(METRIC1, CONFIG1, world * calls * 1000.0 / ms, ms, "propagations/s", args, world)
    line.update({
        "e2e": {"value": world * calls * 1000.0 / e2e_ms, "unit": "propagations/s",
                "h2d_bytes_per_step": host_in.numel() * 8, "d2h_bytes_per_step": host_out.numel() * 8},
        "gpu_launches": int(launches),
        "execution": "cuda_graph of the 18 calls (value); eager calls (e2e)",
        "roofline": {"op": "cvhrf_asm_propagate (3 fused FFT/ASM kernels per call)", "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "peak_source": src,
                     "frac": achieved / hbm, "algorithmic_bytes_per_call": per_call, "traffic": None},
        "clocks": sampler.summary()})
    return line


def _config2_inputs(dev):
    from complex_valued_holographic_radiance_fields_b200 import scene as SC
    cam = SC.PinholeCamera(800, 800)
    params = SC.make_gaussians(100000, K=3, C=3, seed=0, device=dev)
    kw, _ = SC.render_inputs(params, cam)
    return {k: (v.detach().contiguous() if torch.is_tensor(v) else v) for k, v in kw.items()}


_KW_TENSORS = ("cam_means_3D", "z_vals", "quats", "scales", "colours", "phase", "opacities", "plane_probs")


def run_config2(args, world, rank, local):
    from complex_valued_holographic_radiance_fields_b200 import _lib, rasterizer as RZ, scene as SC
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    kw = _config2_inputs(dev)
    sargs = SC.splat_args(kw)
    sampler = ClockSampler(local)
    sampler.__enter__()
    L = _lib.lib()
    n0 = L.cvhrf_kernel_launch_count()
    ms = _timed_loop(lambda: RZ.splat_tile_cuda(*sargs), args.steps, args.warmup)
    launches = (L.cvhrf_kernel_launch_count() - n0) * args.steps // (args.steps + args.warmup)
    sampler.__exit__()
    pairs = RZ.last_num_pairs
    # end to end through the same call: the rasterizer inputs from pinned host memory, the field back
    host = {k: kw[k].cpu().pin_memory() for k in _KW_TENSORS}
    dkw = dict(kw)
    for k in _KW_TENSORS:
        dkw[k] = torch.empty_like(kw[k])
    field0, _ = RZ.splat_tile_cuda(*sargs)
    host_out = torch.empty(field0.shape, dtype=field0.dtype).pin_memory()

    def e2e_step():
        for k in _KW_TENSORS:
            dkw[k].copy_(host[k], non_blocking=True)
        f, _ = RZ.splat_tile_cuda(*SC.splat_args(dkw))
        host_out.copy_(f, non_blocking=True)

    e2e_ms = _timed_loop(e2e_step, args.steps, 2)
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
    if rank != 0:
        return None
    clocks = sampler.summary()
    sm_mhz = clocks.get("sm_mhz") or 1965.0
    peak = fp32_peak_tflops(sm_mhz)
    flop = 256.0 * pairs * FWD_FLOP_PER_EVAL
    line = _base_line(METRIC2, CONFIG2, world * 1000.0 / ms, ms, "forwards/s", args, world)
    line.update({
        "e2e": {"value": world * 1000.0 / e2e_ms, "unit": "forwards/s",
                "h2d_bytes_per_step": sum(h.numel() * 4 for h in host.values()),
                "d2h_bytes_per_step": host_out.numel() * 8},
        "gpu_launches": int(launches),
        "roofline": {"op": "splat_tile_cuda forward (whole call: binning + render)", "bound": "fp32",
                     "achieved": flop / (ms * 1e-3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "peak_source": f"SMs x 128 FMA lanes x 2 x median SM clock {sm_mhz:.0f} MHz",
                     "frac": flop / (ms * 1e-3) / 1e12 / peak,
                     "work_unit": f"{FWD_FLOP_PER_EVAL} FLOP per pixel-pair evaluation x 256 x {pairs} pairs",
                     "traffic": None},
        "clocks": clocks})
    return line


def run_reference_component(args, world, rank):
    """--impl reference for config1 / config2: the reference's CPU path on the host cores
    (value), and its CUDA kernels rebuilt for sm_100a on this GPU beside it."""
    if rank != 0:
        return None
    from oracle import cpu_step
    threads = torch.get_num_threads()
    if args.workload == "config1":
        x = _config1_field()
        sample = CONFIG1_CALLS[:2]
        t = time.perf_counter()
        for wl, d in sample:
            cpu_step.torch_asm(cpu_step.torch_asm(x, wl, 8e-6, d, 1024), wl, 8e-6, -d, 1024)
        cpu_v = 2 * len(sample) / (time.perf_counter() - t)
        line = _base_line(METRIC1, CONFIG1, cpu_v, 1000.0 * 18 / cpu_v, "propagations/s", args, world)
        line["cpu_baseline"] = {"value": cpu_v, "unit": "propagations/s", "cores": threads, "kind": "port",
                                "sample": f"{2 * len(sample)} propagations: the reference's pure-torch "
                                          "propagation (python_function.py:35-78) on torch CPU"}
    else:
        from oracle import raster_oracle as RO
        kw = _config2_inputs("cuda" if torch.cuda.is_available() else "cpu")
        inp = {"cam_means": kw["cam_means_3D"], "z_vals": kw["z_vals"], "quats": kw["quats"],
               "scales": kw["scales"], "colours": kw["colours"], "phase": kw["phase"], "opacities": kw["opacities"],
               "plane_probs": kw["plane_probs"], "view": kw["view_matrix"]}
        inp = {k: v.detach().cpu().numpy() for k, v in inp.items()}
        t = time.perf_counter()
        RO.forward(inp, 800, 800, kw["fx"], kw["fy"], kw["px"], kw["py"], kw["near_plane"], kw["far_plane"])
        cpu_v = 1.0 / (time.perf_counter() - t)
        threads = cpu_step.num_threads()
        line = _base_line(METRIC2, CONFIG2, cpu_v, 1000.0 / cpu_v, "forwards/s", args, world)
        line["cpu_baseline"] = {"value": cpu_v, "unit": "forwards/s", "cores": threads, "kind": "port",
                                "sample": "1 forward: oracle/raster_oracle.c (OpenMP restatement of the "
                                          "reference rasterizer)"}
    line["impl"] = "reference"
    line["execution"] = "host cpu (rank 0 only)"
    line["cpu_baseline"]["cores"] = threads
    line["e2e"] = {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    if torch.cuda.is_available():
        try:
            line["reference_cuda_sm100a"] = _ref_cuda_component(args)
        except Exception as e:
            line["reference_cuda_sm100a"] = {"unavailable": repr(e)[:200]}
    return line


def _ref_cuda_component(args):
    from oracle import ref_harness
    if not ref_harness.available():
        return {"unavailable": "oracle/_ref not built"}
    steps, warmup = max(min(args.steps, 20), 5), 3
    if args.workload == "config1":
        x = _config1_field().cuda()
        F = ref_harness.RefBandlimitedPropagationFunction

        def step():
            for wl, d in CONFIG1_CALLS:
                F.apply(F.apply(x, wl, 8e-6, d, [1024, 1024], -1.0), wl, 8e-6, -d, [1024, 1024], -1.0)

        ms = _timed_loop(step, steps, warmup)
        return {"value": 18 * 1000.0 / ms, "unit": "propagations/s", "ms_per_step": ms,
                "what": "reference cuda_modules transfer kernel + torch cuFFT (python_function.py:109-163 glue)"}
    from complex_valued_holographic_radiance_fields_b200 import scene as SC
    kw = _config2_inputs("cuda")
    a = list(SC.splat_args(kw))
    a[12] = ref_harness.view_buffer(kw["view_matrix"])
    ms = _timed_loop(lambda: ref_harness.RefSplatTileCuda.apply(*a), steps, warmup)
    return {"value": 1000.0 / ms, "unit": "forwards/s", "ms_per_step": ms,
            "what": "reference cov3d_cuda Rasterizer.forward (rebuilt sm_100a)"}


def strong_records(args, world, rank, local):
    """The two strong-scaling workloads, measured in the same process after the headline
    (which is config-3 weak scaling): config 4 (the 8 views of one iteration split over
    the GPUs) and config 5 (the 7 planes of one iteration split over the GPUs).  Each is
    timed like its own --workload line (warm-up, then device-timed steps, max over ranks)."""
    import gc
    out = {}
    for key, fn, steps, warmup in (("strong_config4", run_config4, min(args.steps, 5), 2),
                                   ("strong_config5", run_config5, min(args.steps, 10), 3)):
        gc.collect()
        torch.cuda.empty_cache()
        sub = argparse.Namespace(**vars(args))
        sub.steps, sub.warmup = steps, warmup
        try:
            r = fn(sub, world, rank, local)
        except Exception as e:  # a failed sub-record must not lose the headline line
            r = {"unavailable": repr(e)[:300]}
        if r is not None:
            keep = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling", "config",
                    "execution", "unavailable")
            out[key] = {k: v for k, v in r.items() if k in keep}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the strong-scaling sub-records (config 4 and 5) of the default line")
    ap.add_argument("--workload", default="config3", choices=["config1", "config2", "config3", "config3mp", "config4",
                                                           "config5"],
                    help="config1 / config2 (the propagation / rasterizer forward alone), "
                         "config3 (default, the BASELINE metric), config3mp (config 3 with the multiplane "
                         "reconstruction loss), config4 (8 views per iteration split over the GPUs) or config5 "
                         "(planes split over the GPUs); config4/5 scale strongly")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    try:
        if args.impl == "reference" and args.workload in ("config1", "config2"):
            line = run_reference_component(args, world, rank)
        elif args.impl == "reference":
            line = run_reference(args, world, rank)
        elif args.workload == "config1":
            line = run_config1(args, world, rank, local)
        elif args.workload == "config2":
            line = run_config2(args, world, rank, local)
        elif args.workload == "config5":
            line = run_config5(args, world, rank, local)
        elif args.workload == "config4":
            line = run_config4(args, world, rank, local)
        else:
            line = run_mine(args, world, rank, local)
            if line is not None and world == 1 and not args.no_cpu_baseline and args.workload == "config3":
                line["cpu_baseline"] = cpu_baseline(samples=3, warmup=1)
            if args.workload == "config3" and not args.no_strong:
                strong = strong_records(args, world, rank, local)
                if line is not None:
                    line.update(strong)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
