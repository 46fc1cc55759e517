"""hive_neuralnet_b200 -- B200-native (sm_100a) self-play hot path for Hive.

Drop-in for the reference's ``hive_gpu.load_extension()`` operator module
(:mod:`hive_neuralnet_b200.hive_gpu`), backed by hand-written CUDA kernels
behind the C ABI in ``include/hive_b200.h``.
"""
from . import _lib  # noqa: F401

__all__ = ["hive_gpu"]
