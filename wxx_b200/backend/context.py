"""Global train / inference mode (reference: src/wxx/backend/context.py:1-15).

``MODE`` is 0 in training mode and 1 under :class:`inferenceMode`.  It gates
dropout and BatchNorm's use of batch statistics, exactly as in the reference.
"""

MODE = 0


class inferenceMode:
    """Context manager that switches to inference mode (``MODE = 1``).

    Unlike the reference, the previous mode is restored on exit, so nesting an
    ``inferenceMode`` inside another one keeps the outer one in effect.
    """

    def __init__(self):
        self._prev = 0

    def __enter__(self):
        global MODE
        self._prev = MODE
        MODE = 1
        return MODE

    def __exit__(self, exc_type, exc_val, exc_tb):
        global MODE
        MODE = self._prev
