"""B200 (sm_100a) probe path of cuda_micro_bench.

The compute path is the native library ``lib/libcmb_b200.so`` (hand-written
CUDA for sm_100a behind the C ABI of ``include/cmb_b200.h``) and the C++ CLI
``bin/cmb_b200``.  This package only loads the library (``capi``) and builds
it (``build``); there is no Python or CPU fallback for any probe.
"""

from .capi import CmbError, lib, check, library_path  # noqa: F401

__all__ = ["CmbError", "lib", "check", "library_path"]
