"""B200 engine for the NeuroGen spiking language core and isolated-tick spiking networks.

The compute lives in ``lib/libneurogen_native.so`` (sm_100a CUDA kernels behind the C ABI of
``include/neurogen_b200.h``); this package is the ctypes host side.
"""
from ._lib import library, library_path, EXPORTS  # noqa: F401
