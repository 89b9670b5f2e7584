"""B200-native F-16 parallel-environment hot path (drop-in for the reference's cuda_fdm GPU env).

Modules mirror the reference's names for the path:
  gpu_env     GpuDogfight                         (cuda_fdm/gpu_env.py)
  ic          IC geodesy, sampling, GPU seeding   (cuda_fdm/ic.py, rl_env.py:57-174)
  _lib        ctypes binding of libf16env.so (include/f16env.h)
  build       in-tree nvcc build of libf16env.so for sm_100a

The package directory name is not a Python identifier; import it with
``importlib.import_module("2026_ai_pilot_challenge-1st_solution_b200")``.
"""
__version__ = "0.1.0"
