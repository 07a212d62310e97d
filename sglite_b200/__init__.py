"""B200-native (sm_100a) AWQ W4A16 quantized-linear path for SGLite.

The compute lives in the C-ABI library ``lib/libawqb200.so`` (CUDA kernels for
sm_100a, NCCL); this package is the PyTorch-facing host side that mirrors the
reference's linear-method interface (``layers/quantization/base_config.py``).
"""

__version__ = "0.1.0"
