"""``.npz`` save / load of state dicts (reference: src/wxx/serialization.py).

One array per parameter, keyed by the dotted name from ``Module.state_dict``
-- the same files the reference writes and reads.
"""

import os

import numpy as np


def _to_arrays(obj):
    from .nn.module import Module

    if isinstance(obj, Module):
        obj = obj.state_dict()
    if isinstance(obj, dict):
        out = {}
        for k, v in obj.items():
            if hasattr(v, "numpy") and not isinstance(v, np.ndarray):
                v = v.numpy()
            out[str(k)] = np.asarray(v)
        return out
    if hasattr(obj, "numpy") and not isinstance(obj, np.ndarray):
        obj = obj.numpy()
    return {"tensor": np.asarray(obj)}


def save(obj, path):
    path = str(path)
    if not path.endswith(".npz"):
        path = path + ".npz"
    np.savez(path, **_to_arrays(obj))
    return path


def load(path, model=None):
    path = str(path)
    if not path.endswith(".npz") and not os.path.exists(path):
        path = path + ".npz"
    with np.load(path) as data:
        state = {k: data[k] for k in data.files}
    if model is not None:
        model.load_state_dict(state)
        return model
    return state
