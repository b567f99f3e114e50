"""wxx_b200: the wxx tensor API on hand-written sm_100a (B200) kernels.

Drop-in for the reference's ``wxx`` package (Mo-Ehab/wxx): ``Tensor``,
``functional``, ``autograd``, ``nn`` (GPT2, ResNet18, Hyena) and ``.npz``
``save``/``load`` keep their names and signatures; the WebGPU/WGSL kernel
layer is replaced by libwxx_cuda.so (tcgen05 TF32 GEMM and implicit-GEMM
convolution, fused FFT convolution, single-pass reductions / softmax / norms).
``import wxx_b200 as wxx`` runs code written for the reference.
"""

from .Tensor import Parameter, Tensor
from . import autograd, backend, functional, graph, nn, serialization
from .backend.device import get_device
from .functional import get_matmul_mode, manual_seed, set_matmul_mode
from .serialization import load, save

__all__ = [
    "Tensor",
    "Parameter",
    "autograd",
    "functional",
    "graph",
    "nn",
    "backend",
    "serialization",
    "get_device",
    "save",
    "load",
    "manual_seed",
    "set_matmul_mode",
    "get_matmul_mode",
]
