"""prana_b200: Prana's batch-1 decode path (block-quantized GEMV, GQA decode
attention over an f16 KV cache, RMSNorm/RoPE/SwiGLU glue) as sm_100a CUDA
kernels behind a C ABI (include/prana_cuda.h).

Modules: `kernels` (the prana-kernels surface), `model` (the prana-model decode
API), `synth` (seeded random-init GGUF models), `build` (in-tree native build).
"""
__version__ = "0.1.0"
