"""B200 (sm_100a) probe path of cuda_micro_bench.

The compute path is the native library ``lib/libcmb_b200.so`` (hand-written
CUDA for sm_100a behind the C ABI of ``include/cmb_b200.h``) and the C++ CLI
``bin/cmb_b200``.  This package only loads the library (``capi``) and builds
it (``build``); there is no Python or CPU fallback for any probe.
"""

__all__ = ["CmbError", "lib", "check", "library_path", "sm_die_map", "set_sm_die_map"]


def __getattr__(name):
    # The library loads on first use of any of these names, so that
    # `python -m cuda_micro_bench_b200.build` works before it exists; using
    # them without the built library raises ImportError (no fallback).
    if name in __all__:
        from . import capi

        return getattr(capi, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
