"""B200-native streaming-step runtime.

A drop-in for the per-event hot path of vishalkishore/streaming-transformer
(``Stream::Runtime::step``): hand-written sm_100a CUDA kernels behind a C ABI
(include/streaming_b200.h), with this package as the Python host binding and
include/Runtime.hpp as the C++ one.
"""
from .model import CheckpointError, Model, ModelConfig, tensor_shapes, write_checkpoint
from .runtime import (Backend, BACKEND_NAMES, Runtime, RuntimeOptions, Snapshot, StreamError, TensorParallel,
                      library, probe, transport_bench)

__all__ = ["Backend", "BACKEND_NAMES", "CheckpointError", "Model", "ModelConfig", "Runtime",
           "RuntimeOptions", "Snapshot", "StreamError", "TensorParallel", "library", "probe", "tensor_shapes", "transport_bench",
           "write_checkpoint"]
