"""B200-native zeroth-order hot path with the zotitan.train_zo API.

Public surface: ``zotitan_b200.train_zo`` (ZOConfig, ZOOptimizer, train_zo), the raw
kernels in ``zotitan_b200.kernels`` and the C ABI in include/zotitan_b200.h.
"""
__version__ = "0.1.0"
