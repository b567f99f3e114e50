"""Losses (interface: src/wxx/nn/loss.py): called as ``loss(prediction, truth)``
and returning a scalar tensor whose ``backward()`` trains the model."""

import math

from .. import autograd


class loss:
    """Base of the losses."""

    def __call__(self, *args, **kwargs):
        raise NotImplementedError


class CCELoss(loss):
    """Mean softmax cross-entropy of (B, K) logits against (B,) u32 targets
    (``CrossEntropyLoss`` per row, then the mean).  With ``mask`` (B values)
    the rows are weighted and the sum is divided by ``mask.sum()``."""

    def __call__(self, prediction, truth, mask=None):
        rows = autograd.CrossEntropyLoss(prediction).forward(prediction, truth)
        if mask is None:
            return rows.mean()
        if math.prod(mask.shape) != prediction.shape[0]:
            raise ValueError(f"mask must contain one value per prediction row; got "
                             f"{math.prod(mask.shape)} values for {prediction.shape[0]} rows")
        weights = mask.reshape((prediction.shape[0], 1))
        return (rows * weights).sum() / weights.sum()


class MAELoss(loss):
    """Mean absolute error."""

    def __call__(self, prediction, truth):
        return (truth - prediction).abs().mean()
