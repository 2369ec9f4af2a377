"""Build the UNMODIFIED reference CUDA extensions for sm_100a into ``oracle/_ref/``.

Test infrastructure only: the resulting modules are the parity checker that the
GPU tests and ``bench.py --impl reference`` compare against; nothing in the
product imports them.

Two torch extensions are compiled straight from the reference tree (the sources
are read where they lie; nothing is copied into this repository):

* ``cov3d_cuda_ref``  — the source list of ``cuda_prop/cov3d_cuda/setup.py:53-60``
  (binding.cpp, wave_rasterizer/{forward,backward,forward_splat,backward_splat,
  rasterizer_splat}.cu, conv.cu) with the GLM include path of setup.py:12 and the
  nvcc flags of setup.py:37-40, the arch flags (setup.py:41-42, sm_80/sm_86)
  replaced by ``-gencode arch=compute_100a,code=sm_100a``.
* ``cuda_modules_ref`` — the source list of ``cuda_prop/build_cuda_extension.py:17-30``.

Only the module names differ from the reference (``TORCH_EXTENSION_NAME``), so the
two can be loaded next to this package's own library. The outputs stay under
``oracle/_ref/`` (git-ignored); on the GPU box the prebuilt ``.so`` files are used
and the reference tree is never read.

usage: python oracle/build_ref.py [--ref /path/to/reference]
"""
import argparse
import os

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"
# --ptx80: the same sources as compute_80 PTX only (JIT-compiled by the driver on a B200),
# into oracle/_ref80/ -- the "reference's own sm_80 build run on a B200" comparison point
OUT80 = os.path.join(HERE, "_ref80")
ARCH80 = "-gencode=arch=compute_80,code=compute_80"


def _load(name, sources, include_dirs, cuda_flags, build_dir):
    from torch.utils.cpp_extension import load
    os.makedirs(build_dir, exist_ok=True)
    return load(name=name, sources=sources, extra_include_paths=include_dirs,
                extra_cflags=["-O3"], extra_cuda_cflags=cuda_flags,
                build_directory=build_dir, verbose=False, is_python_module=True)


def build(ref_root="/root/reference", arch=ARCH, out=OUT):
    cov = os.path.join(ref_root, "cuda_prop", "cov3d_cuda")
    prop = os.path.join(ref_root, "cuda_prop")
    if not os.path.isdir(cov):
        raise FileNotFoundError(f"reference tree not found at {ref_root}")
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    wr = os.path.join(cov, "wave_rasterizer")
    _load("cov3d_cuda_ref",
          [os.path.join(cov, "binding.cpp")]
          + [os.path.join(wr, f) for f in ("forward.cu", "backward.cu", "forward_splat.cu",
                                           "backward_splat.cu", "rasterizer_splat.cu")]
          + [os.path.join(cov, "conv.cu")],
          [os.path.join(cov, "third_party", "glm")],
          ["-O3", "-DTORCH_USE_CUDA_DSA", "-diag-suppress=20012", arch],
          os.path.join(out, "cov3d_cuda_ref"))
    cpp = os.path.join(prop, "cpp")
    cu = os.path.join(prop, "cuda")
    _load("cuda_modules_ref",
          [os.path.join(cpp, f) for f in ("bandlimited_propagation.cpp", "batch_matrix_mult.cpp",
                                          "sum_last_dim.cpp", "element_wise_mult.cpp", "module_def.cpp")]
          + [os.path.join(cu, f) for f in ("bandlimited_propagation_cuda.cu", "batch_matrix_mult_cuda.cu",
                                           "sum_last_dim_cuda.cu", "element_wise_mult_cuda.cu")],
          [], ["-O3", arch], os.path.join(out, "cuda_modules_ref"))


def built():
    return (os.path.exists(os.path.join(OUT, "cov3d_cuda_ref", "cov3d_cuda_ref.so"))
            and os.path.exists(os.path.join(OUT, "cuda_modules_ref", "cuda_modules_ref.so")))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--ptx80", action="store_true")
    a = ap.parse_args()
    build(a.ref, ARCH80, OUT80) if a.ptx80 else build(a.ref)
    print("built reference modules under", OUT80 if a.ptx80 else OUT)
