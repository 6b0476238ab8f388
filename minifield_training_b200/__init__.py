"""B200-native (sm_100a) hot path of minifield-training.

Hand-written CUDA kernels (libmfb200.so, C ABI in include/mfb200.h) for the
masked GQA attention forward/backward, the KV-cached decode step and the QAT
fake-quant + GEMM chain, behind Python functions named after the reference's
``minifield_training.kernels`` / ``layers`` modules. Build with
``python -m minifield_training_b200.build``.
"""

__version__ = "0.1.0"
