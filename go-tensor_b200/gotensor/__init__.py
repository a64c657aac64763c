"""go-tensor's B200 backend, Python side.

* ``gotensor.backend.CudaBackend`` — the CUDA device behind go-tensor's
  ``backend.Backend`` interface (the primitive path);
* ``gotensor.model.Model`` — the native fused training step of a Sequential
  model (the fused path), with data parallelism over NCCL.

Both call the C interfaces in ``include/`` through ctypes; nothing here runs
on the CPU in their place.
"""
from ._lib import ACT_NONE, ACT_RELU, ACT_SIGMOID, ACT_TANH, FLOAT32, FLOAT64, GTError  # noqa: F401
