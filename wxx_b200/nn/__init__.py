"""Neural-network modules and models (reference: src/wxx/nn/__init__.py)."""

from .gpt import GPT2, GPT2Block
from .hyena import (
    CausalShortConv1d,
    Hyena,
    HyenaBlock,
    HyenaOperator,
    ImplicitFilter,
    PositionalEncoding,
    Sine,
    SwiGLU,
    TiedLinear,
)
from .module import (
    GELU,
    AdaptiveAvgPool2d,
    Attention,
    AvgPool1d,
    AvgPool2d,
    BatchNorm,
    Conv2D,
    Conv2DTranspose,
    Dropout,
    Embedding,
    LayerNorm,
    Linear,
    MaxPool1d,
    MaxPool2d,
    Module,
    ModuleList,
    MultiHeadAttention,
    RMSNorm,
    Sequential,
)
from .loss import CCELoss, MAELoss, loss
from .optimizer import AdamW, Optimizer, SGD
from .resnet import ResBlock, ResNet18

__all__ = [
    "AdaptiveAvgPool2d", "Attention", "AvgPool1d", "AvgPool2d", "BatchNorm", "CausalShortConv1d",
    "Conv2D", "Conv2DTranspose", "Dropout", "Embedding", "GELU", "GPT2", "GPT2Block", "Hyena",
    "HyenaBlock", "HyenaOperator", "ImplicitFilter", "LayerNorm", "Linear", "MaxPool1d",
    "MaxPool2d", "Module", "ModuleList", "MultiHeadAttention", "PositionalEncoding", "RMSNorm",
    "ResBlock", "ResNet18", "Sequential", "Sine", "SwiGLU", "TiedLinear",
    "loss", "CCELoss", "MAELoss", "Optimizer", "SGD", "AdamW",
]
