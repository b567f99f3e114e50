"""Optimisers (interface: src/wxx/nn/optimizer.py): built from
``module.parameters()`` (``("", parameter)`` pairs) and stepping the
parameters in place from their ``.grad``."""

import numpy as np

from .. import functional
from ..Tensor import Tensor
from ..functional.utils import mark_written


class Optimizer:
    def __init__(self, parameters):
        self.parameters = list(parameters)

    def step(self):
        raise NotImplementedError

    def zero_grad(self, wait=False):
        for _, w in self.parameters:
            w.grad = None
        if wait:
            from ..backend import device

            device.synchronize()


class SGD(Optimizer):
    """``w -= lr * grad`` in place."""

    def __init__(self, parameters, lr=0.01):
        super().__init__(parameters)
        self.lr = float(lr)

    def step(self):
        for _, w in self.parameters:
            if w.grad is not None:
                functional._pointwise(w, functional.scalarpointwise(w.grad, -self.lr, 2), 0)


class AdamW(Optimizer):
    """Adam with decoupled weight decay, one ``wxx_adamw_device`` launch per
    parameter: ``m = b1 m + (1 - b1) g``, ``v = b2 v + (1 - b2) g^2``,
    ``w -= lr (m / bc1 / (sqrt(v / bc2) + eps) + weight_decay w)`` with the bias
    corrections bc = 1 - beta^t (nn/optimizer.py:38-84, adamw.wgsl).

    The step count t and the bias corrections live in device memory and are
    advanced by a kernel at the start of each step, so a training step
    recorded with ``wxx_b200.graph.capture`` replays as step t + 1, t + 2, ...
    (``step_count`` counts the host calls)."""

    def __init__(self, parameters, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-7,
                 weight_decay=1e-4):
        super().__init__(parameters)
        self.params = self.parameters
        self.lr = float(lr)
        self.beta1, self.beta2 = float(beta1), float(beta2)
        self.eps = float(eps)
        self.weight_decay = float(weight_decay)
        self.step_count = 0
        self.state = [{"exp_avg": Tensor(p.shape, value=0.0),
                       "exp_avg_sq": Tensor(p.shape, value=0.0)} for _, p in self.params]
        self._t = Tensor((1,), value=0, dtype="u32")       # device step count
        self._bc = Tensor((2,), value=1.0)                 # device {bc1, bc2}

    def step(self):
        """One step of every parameter that has a gradient: the step count
        kernel, then one multi-tensor launch per 128 parameters."""
        import ctypes

        from ..backend.lib import F, check

        self.step_count += 1
        check(F.wxx_adamw_advance(self._t.ptr, self._bc.ptr, self.beta1, self.beta2),
              "adamw_advance")
        rows = []
        keep = []
        for (_, w), st in zip(self.params, self.state):
            if w.grad is None:
                continue
            g = functional.contiguous(w.grad)
            if tuple(g.shape) != tuple(w.shape):
                raise ValueError(f"adamw: grad shape {tuple(g.shape)} != {tuple(w.shape)}")
            keep.append(g)
            rows.append((w.ptr, g.ptr, st["exp_avg"].ptr, st["exp_avg_sq"].ptr,
                         int(np.prod(w.shape))))
            for t in (w, st["exp_avg"], st["exp_avg_sq"]):
                mark_written(t)
        if not rows:
            return
        n = len(rows)
        ptrs = [(ctypes.c_void_p * n)(*[r[i] for r in rows]) for i in range(4)]
        lens = (ctypes.c_int64 * n)(*[r[4] for r in rows])
        check(F.wxx_adamw_device_multi(n, *ptrs, lens, self.lr, self.beta1, self.beta2,
                                       self.eps, self.weight_decay, self._bc.ptr), "adamw")
        del keep
