"""femtotron_b200: a B200-native (sm_100a) 3D-parallel LLaMA pretraining framework."""
import os as _os

# Each training process drives several CUDA streams at once (compute, copy-engine gathers,
# reduce-scatter, NCCL).  Streams that share one of the device's hardware work queues are
# serialised, which would turn an overlapped gather or a flag-gated GEMM into a sequential
# one; more queues than the driver's default of 8 keep them apart.  Must be set before the
# process creates its CUDA context; an explicit setting by the user wins.
_os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

__version__ = "0.1.0"
