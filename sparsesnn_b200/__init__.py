"""B200 (sm_100a) backend for SparseSNN's fused 2:4-sparse Conv/Linear + BN +
LIF layer.

The compute lives in ``libsnnb200.so`` (C ABI, ``include/snn_b200.h``);
Python here only binds it, owns device memory through torch tensors and
mirrors the reference sengine interfaces that sit above the kernel.
"""
from .runtime import SnnError, load  # noqa: F401

__all__ = ["SnnError", "load"]
