"""noise_b200: B200-native (sm_100a) forward-only ES training step of Noise.

The compute lives in libnoise_b200.so (hand-written CUDA behind the C ABI of include/noise_b200.h);
this package holds the host-side mirror of the reference's estimator and optimizer interfaces.
"""
from . import _lib  # noqa: F401

__all__ = ['_lib']
