"""simdonnx_b200: a B200 (sm_100a) CUDA execution backend for SimdOnnx's fused conv/GEMM hot path.

Layers:
  * ``libsdxcuda.so`` (csrc/, C ABI in include/sdxcuda.h): tcgen05/TMEM implicit-GEMM conv, Gemm
    and ConvT kernels, bandwidth kernels, runtime, graph-captured sessions;
  * ``_native``: ctypes binding; ``backend``: per-device context + op wrappers on torch tensors;
  * ``plan``: the reference's ExecPlan restated (fused node params, arena offsets) and the plan
    builders of the benchmark configs; ``session``: CudaGraphModel / CudaInferenceSession.
"""
__all__ = ["build", "_native", "backend", "synth"]
