"""rocknpu_b200: RockNPU's ggml MUL_MAT offload, B200-native.

librocknpu.so (built from csrc/ by ``python -m rocknpu_b200.build``) exports
the reference C ABI (include/rocknpu.h) and the B200 additions
(include/rocknpu_b200.h).  ``capi`` binds them with ctypes; ``device`` calls
the device-pointer entry points on torch tensors.
"""
from .capi import (BLOCK_BYTES, Q4_K, Q5_K, Q6_K, STATUS_DEVICE_ERROR, STATUS_EXECUTION_ERROR,
                   STATUS_INVALID_ARGUMENT, STATUS_OK, Context, apply_default_env, device_count, host_empty,
                   lib, mul_mat_supported, synth_encode, synth_normal, synth_q_weights)

__all__ = ["BLOCK_BYTES", "Q4_K", "Q5_K", "Q6_K", "STATUS_OK", "STATUS_INVALID_ARGUMENT", "STATUS_DEVICE_ERROR",
           "STATUS_EXECUTION_ERROR", "Context", "apply_default_env", "device_count", "host_empty", "lib",
           "mul_mat_supported",
           "synth_encode", "synth_normal", "synth_q_weights"]
