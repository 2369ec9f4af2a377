"""B200-native (sm_100a) differentiable wave-optics hot path.

Drop-in operator surfaces of complight/Complex_Valued_Holographic_Radiance_Fields:
  * ``BandlimitedPropagation`` / ``BandlimitedPropagationFunction`` (cuda_prop/python_function.py)
  * ``splat_tile_cuda`` / ``SplatTileCuda`` (cuda_prop/cov3d_cuda/python_import.py)
  * ``SparseGaussianAdam`` / ``sparse_adam_update`` (utils/optimizer.py, python_import.py)
All arithmetic runs in ``libcvhrf.so``; there is no CPU fallback.
"""
from .propagation import (BandlimitedPropagation, BandlimitedPropagationFunction,  # noqa: F401
                          PlanePropagationFunction, propagate, propagate_planes)
from .rasterizer import SplatTileCuda, splat_tile_cuda  # noqa: F401,E402
from .optimizer import SparseGaussianAdam, sparse_adam_update  # noqa: F401,E402

__version__ = "0.1.0"
