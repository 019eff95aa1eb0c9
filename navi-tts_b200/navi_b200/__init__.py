"""navi-b200: the navi-tts per-frame decode path on NVIDIA B200 (sm_100a).

The compute lives in libnavi_b200.so (CUDA kernels + C ABI, include/navi_b200.h);
this package is its Python host mirror (engine), the .navi format (navi_file),
the synthetic model writer (model_spec) and the build step (build).
"""
