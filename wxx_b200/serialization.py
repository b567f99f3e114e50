"""``.npz`` checkpoints of state dicts (interface: src/wxx/serialization.py).

File format (shared with the reference, so either side reads the other's
files): a numpy ``.npz`` archive holding one array per entry of
``Module.state_dict()``, stored under the entry's dotted name
(``blocks.0.attn.q.weight`` ...), in the tensor's shape and dtype.  A single
tensor or array is stored under the key ``"tensor"``.

``save(obj, path)`` appends ``.npz`` when the name lacks it and returns the
path written.  ``load(path)`` returns ``{name: ndarray}``; ``load(path,
model)`` also copies the arrays into ``model`` (``load_state_dict``) and
returns the model.
"""

import os

import numpy as np

_SINGLE_KEY = "tensor"


def _host_array(value):
    """A numpy copy of a Tensor (device download) or any array-like."""
    if isinstance(value, np.ndarray):
        return value
    download = getattr(value, "numpy", None)
    return np.asarray(download() if callable(download) else value)


def _archive_entries(obj):
    from .nn.module import Module

    state = obj.state_dict() if isinstance(obj, Module) else obj
    if isinstance(state, dict):
        return {str(name): _host_array(v) for name, v in state.items()}
    return {_SINGLE_KEY: _host_array(state)}


def save(obj, path):
    """Writes a Module's state dict, a ``{name: tensor}`` dict or one tensor."""
    target = os.fspath(path)
    if not target.endswith(".npz"):
        target += ".npz"
    np.savez(target, **_archive_entries(obj))
    return target


def load(path, model=None):
    """Reads a checkpoint written by ``save`` (here or by the reference)."""
    source = os.fspath(path)
    if not os.path.exists(source) and not source.endswith(".npz"):
        source += ".npz"
    with np.load(source) as archive:
        state = {name: archive[name] for name in archive.files}
    if model is None:
        return state
    model.load_state_dict(state)
    return model
