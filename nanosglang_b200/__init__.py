"""nanosglang_b200 -- B200-native (sm_100a) quantized-linear path for nanoSGLang.

Drop-in replacements for ``nano_sglang.decode.quantization`` (AWQLinear,
FP8Linear, quantize_model) and ``nano_sglang.distributed.tensor_parallel``,
backed by libnsq.so: hand-written CUDA kernels behind a C ABI (include/nsq.h).
"""

from .quantization import AWQLinear, FP8Linear, quantize_model  # noqa: F401

__version__ = "0.1.0"
