"""Device runtime: devices and their resolution, the native caching allocator, stream pools,
device tensors and the tensor-op dispatch.

Reference: PredictiveCoding.Device/Device.cs:11-39, DeviceRuntime.cs:14-83, DeviceRegistry.cs:14-67,
DeviceTensor.cs:20-142, TensorOps.cs:17-104, TensorExtensions.cs, Allocators/CudaAllocator.cs:19-104,
Streams/CudaStreamManager.cs:17-83.  The allocator and the stream pool are native (C++ in the
extension); this package is their Python face.
"""
from .device import Device, DeviceKind, DeviceRegistry, DeviceRuntime
from .allocator import DeviceAllocator
from .streams import StreamManager
from .tensor import DeviceTensor, TensorOps
