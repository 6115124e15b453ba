"""ctypes loader of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
this module, and only as the checker or the timed CPU baseline.  It builds
``oracle/_build/liboracle.so`` with make on first use if it is missing.
"""

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_LOGGER = os.path.join(HERE, "_ref", "ref_logger")
REF_DROPIN = os.path.join(HERE, "_ref", "ref_dropin")

_lib = None


def build(ref: bool = False, ref_root: str = None) -> None:
    """make all; with ref=True also the test builds of the reference's own
    sources (its result logger and its main.cu against libcmb_b200.so), read
    from ref_root (default: the Makefile's)."""
    targets = ["all"] + (["ref", "ref-dropin"] if ref else [])
    extra = [f"REF_ROOT={ref_root}"] if ref_root else []
    proc = subprocess.run(["make", "-C", HERE, "-j8", *targets, *extra], stdout=subprocess.PIPE,
                          stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{proc.stdout}")


def load():
    """Returns the oracle library with argument types set."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    u8, u16, u32, u64 = ctypes.c_uint8, ctypes.c_uint16, ctypes.c_uint32, ctypes.c_uint64
    i, sz, p, f, d = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float, ctypes.c_double
    sig = {
        "orc_splitmix64_at": (u64, [u64, u64]),
        "orc_hash32": (u32, [u32]),
        "orc_fill_hash_u32": (None, [p, sz]),
        "orc_fill_uniform_f32": (None, [p, sz, u64]),
        "orc_fill_bytes": (None, [p, sz, u64]),
        "orc_chase_build": (None, [p, sz, u64]),
        "orc_chase_walk": (u32, [p, u64, u32]),
        "orc_chase_is_single_cycle": (i, [p, sz]),
        "orc_sum_f64": (d, [p, sz, i]),
        "orc_memcpy_mt": (d, [p, p, sz, i]),
        "orc_hw_threads": (i, []),
        "orc_bf16_to_f32": (f, [u16]),
        "orc_f32_to_bf16_rne": (u16, [f]),
        "orc_e4m3_to_f32": (f, [u8]),
        "orc_f32_to_e4m3_satfinite": (u8, [f]),
        "orc_amax_bf16": (f, [p, sz]),
        "orc_quantize_e4m3": (None, [p, sz, f, p]),
        "orc_gemm_tile_f64": (None, [p, p, i, i, i, i, i, i, i, i, d, d, p]),
        "orc_gemm_tiles_f64": (None, [p, p, i, i, i, i, i, p, d, d, p, i]),
        "orc_gemm_bf16_rows_f32": (None, [p, p, p, i, i, i, i, i]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def ptr(array) -> int:
    """Address of a C-contiguous numpy array.  The caller keeps the array
    alive (bound to a name) for as long as the address is used."""
    assert array.flags["C_CONTIGUOUS"]
    return array.ctypes.data
