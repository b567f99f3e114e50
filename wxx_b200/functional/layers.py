"""Embedding and dropout (reference: src/wxx/functional/layers.py)."""

import random

import numpy as np

from ._common import F, check, dense, empty


def embed(tensor1, tensor2, n_token, embed_dim):
    """Row gather ``out[t, :] = W[ids[t], :]`` (functional/layers.py:161-206).

    ``tensor1`` holds u32 ids of shape (B, S); the output is (B, S, embed_dim).
    Ids outside the table produce zero rows and set the device error word."""
    ids = dense(tensor1)
    w = dense(tensor2)
    if ids.type != "u32":
        raise TypeError(f"embed expects u32 ids, got {ids.type!r}")
    if len(ids.shape) < 2:
        raise ValueError(f"embed expects (batch, seq) ids, got shape {ids.shape}")
    vocab = w.shape[0]
    out = empty((ids.shape[0], ids.shape[1], embed_dim), "f32")
    check(F.wxx_embed(out.buffer.ptr, ids.ptr, w.ptr, int(n_token), int(embed_dim), int(vocab)),
          "embed")
    return out


def dropout(tensor1, p, seed=None):
    """Inverted dropout (training mode): zero with probability ``p``, scale by
    1/(1-p).  The mask is drawn on the host from ``seed`` (``random`` when
    omitted, as functional/layers.py:81 does)."""
    x = dense(tensor1)
    if seed is None:
        seed = random.randint(0, 2**31 - 1)
    return _apply_dropout_mask(x, p, seed), seed


def _apply_dropout_mask(x, p, seed):
    """x * keep / (1 - p) with keep drawn on the host from ``seed``."""
    keep = (np.random.default_rng(seed).random(tuple(x.shape)) >= p).astype(np.float32)
    from .utils import from_numpy
    from .pointwise import pointwise

    scale = 0.0 if p >= 1.0 else 1.0 / (1.0 - p)
    return pointwise(pointwise(x, from_numpy(keep), 2), scale, 2)


def dropoutdx(tensor1, p, seed):
    """Gradient of ``dropout(x, p)`` drawn with ``seed`` (functional/layers.py:117):
    the same mask and scale applied to the upstream gradient."""
    return _apply_dropout_mask(dense(tensor1), p, seed)
