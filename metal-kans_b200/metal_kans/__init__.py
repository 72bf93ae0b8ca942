"""metal_kans -- B200 (sm_100a) engine behind the metal-KANs inference API.

Drop-in for the forward path of Shuril/metal-kans v0.6.0 (``metal_kans/__init__.py``): the layer
classes ChebyKAN / FastKAN / BSplineKAN (KAN) / WavKAN / ReLUKAN / FourierKAN / JacobiKAN /
RationalKAN / MultKAN / LowRankKAN, the GatedKAN block, the MetalKAN stack, ``.half()``, the
quantisers (INT8/INT4/ternary/INT2 with the same packed layouts), the torch modules
(differentiable), ``set_async``/``sync`` and the parameter utilities.  fp32 layers of the Chebyshev, RBF, B-spline and ReLU bases also have the
reference's backward (weight, bias and input gradients); Chebyshev, RBF and B-spline layers its
fused training step (forward, MSE gradient, backward, AdamW in one call), and ``optim`` has the
SGD / Adam / AdamW / Lion optimisers, stepping on the GPU.  The compute runs in ``libkan_cuda.so``
(hand-written CUDA for sm_100a); there is no CPU fallback.

Muon / RMSprop, checkpointing, pruning and symbolic export are not part of this engine.
"""
from .device import (KanError, get_metal_bridge, is_cuda_available, is_metal_available,
                     set_async, sync)
from .cheby_kan import ChebyKAN
from .fast_kan import FastKAN
from .wav_kan import WavKAN
from .bspline_kan import BSplineKAN, KAN
from .relu_kan import ReLUKAN
from .fourier_kan import FourierKAN
from .jacobi_kan import JacobiKAN
from .rational_kan import RationalKAN
from .mult_kan import MultKAN
from .low_rank_kan import LowRankKAN
from .metal_kan import MetalKAN
from .gated_kan import GatedKAN
from .quantization import (Int2QuantizedWeight, QuantizedWeight, TernaryQuantizedWeight,
                           quantize, to_int2, to_int4, to_int8, to_ternary)
from .utils import build_train_step, count_parameters, get_model_size
from . import optim

try:
    from .torch_module import TorchGatedKAN, TorchMetalKAN, TorchMetalKANLinear
except ImportError:  # torch is optional for the NumPy API
    TorchMetalKANLinear = None
    TorchMetalKAN = None
    TorchGatedKAN = None

__version__ = "0.6.0+b200"

__all__ = [
    "set_async", "sync", "is_metal_available", "is_cuda_available", "get_metal_bridge",
    "KanError",
    "ChebyKAN", "FastKAN", "WavKAN", "BSplineKAN", "KAN", "ReLUKAN", "FourierKAN", "JacobiKAN",
    "RationalKAN", "MultKAN", "LowRankKAN",
    "MetalKAN", "GatedKAN",
    "QuantizedWeight", "TernaryQuantizedWeight", "Int2QuantizedWeight",
    "quantize", "to_int8", "to_int4", "to_ternary", "to_int2",
    "count_parameters", "get_model_size", "build_train_step", "optim",
    "TorchMetalKANLinear", "TorchMetalKAN", "TorchGatedKAN",
]
