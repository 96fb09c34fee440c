"""spirv_inference_b200 — a B200 (sm_100a) backend for the per-op kernel
dispatch of SPIRV_INFERENCE-style graphs.

Modules:
  _lib       ctypes binding of libspx.so (include/spx.h)
  dispatch   drop-in boundary: KernelRun / KernelOutput / run_kernel / registry
  lowering   reference-scheduler lowering of TFLite-style graphs onto run_kernel
  graph      device-resident graph API (stream, buffers, NHWC ops, CUDA graphs)
  executor   fused NHWC executor for the CNN graphs
  nets       TFLite-style MobileNetV2 / EfficientNet-Lite0 graphs, seeded weights
  build      nvcc build of libspx.so for sm_100a
"""
__version__ = "0.1.0"
