"""CUDA backend: library binding, device runtime and launch helpers."""

from .context import inferenceMode
from .device import (
    CommandStream,
    CudaContext,
    DeviceBuffer,
    DeviceBufferPool,
    Event,
    PinnedHostBuffer,
    device_status,
    get_buffer_pool,
    get_cmd_buffer,
    get_ctx,
    get_device,
    synchronize,
)

__all__ = [
    "inferenceMode",
    "CommandStream",
    "CudaContext",
    "DeviceBuffer",
    "DeviceBufferPool",
    "Event",
    "PinnedHostBuffer",
    "device_status",
    "get_buffer_pool",
    "get_cmd_buffer",
    "get_ctx",
    "get_device",
    "synchronize",
]
