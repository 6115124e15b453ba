"""ctypes binding of the C ABI in include/cmb_b200.h.

Loading fails loudly (ImportError) when ``lib/libcmb_b200.so`` has not been
built: the probes have no other implementation.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
library_path = os.path.join(HERE, "lib", "libcmb_b200.so")

if not os.path.exists(library_path):
    raise ImportError(
        f"{library_path} is missing: build it with `python -m cuda_micro_bench_b200.build` "
        "(the probe path has no CPU fallback)"
    )

lib = ctypes.CDLL(library_path)

_i, _u32, _u64, _sz = ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t
_p, _f, _d, _s = ctypes.c_void_p, ctypes.c_float, ctypes.c_double, ctypes.c_char_p

# name -> (restype, argtypes); the stream argument is a raw handle (c_void_p).
SIGNATURES = {
    "cmb_status_string": (_s, [_i]),
    "cmb_last_error": (_s, []),
    "cmb_version": (_s, []),
    "cmb_device_reset": (_i, []),
    "cmb_fill_hash_u32": (_i, [_p, _sz, _p]),
    "cmb_fill_uniform_f32": (_i, [_p, _sz, _u64, _p]),
    "cmb_fill_bytes": (_i, [_p, _sz, _u64, _p]),
    "cmb_fill_normal_bf16": (_i, [_p, _sz, _u64, _f, _p]),
    "cmb_stream_copy": (_i, [_p, _p, _sz, _p]),
    "cmb_stream_copy_tuned": (_i, [_p, _p, _sz, _i, _i, _i, _p]),
    "cmb_stream_sum_workspace_bytes": (_sz, [_sz]),
    "cmb_stream_sum_f32": (_i, [_p, _sz, _p, _p, _sz, _p]),
    "cmb_stream_sum_f32_noalloc": (_i, [_p, _sz, _p, _p]),
    "cmb_stream_sum_noalloc_max_ctas": (_sz, []),
    "cmb_l2_read": (_i, [_p, _sz, _i, _i, _p, _p]),
    "cmb_l2_read_bulk": (_i, [_p, _sz, _i, _p, _p, _p]),
    "cmb_stream_copy_host": (_i, [_p, _p, _sz, _p, _p, _sz, _sz]),
    "cmb_chase_build_links": (_i, [_p, _sz, _u64]),
    "cmb_chase_run": (_i, [_p, _sz, _u64, _u64, _i, _p, _p]),
    "cmb_chase_host_walk": (_i, [_p, _sz, _u64, _p]),
    "cmb_tma_tile_copy_bf16": (_i, [_p, _p, _i, _i, _i, _i, _i, _i, _p, _p]),
    "cmb_tma_tile_copy_tuned": (_i, [_p, _p, _i, _i, _i, _i, _i, _i, _i, _p, _p]),
    "cmb_tma_tile_load_bf16": (_i, [_p, _i, _i, _i, _i, _i, _p, _sz, _p, _p]),
    "cmb_tma_1d_latency": (_i, [_p, _sz, _sz, _i, _p, _p, _p, _p]),
    "cmb_gemm_bf16": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p]),
    "cmb_gemm_e4m3": (_i, [_p, _p, _p, _i, _i, _i, _p, _p, _i, _p, _p]),
    "cmb_gemm_tuned": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p]),
    "cmb_gemm_bf16_out": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _p]),
    "cmb_sm_die_map": (_i, [_p, _i, _p, _p, _p]),
    "cmb_gemm_set_sm_die_map": (_i, [_p, _i]),
    "cmb_mma_rate": (_i, [_i, _i, _i, _p, _p, _p, _p]),
    "cmb_quantize_e4m3": (_i, [_p, _sz, _p, _p, _p]),
    "cmb_mma_sync_latency": (_i, [_i, _i, _p, _p, _p]),
    "cmb_mma_sync_throughput": (_i, [_i, _i, _i, _i, _p, _p]),
    "cmb_p2p_alloc": (_i, [_sz, _p]),
    "cmb_p2p_free": (_i, [_p]),
    "cmb_ipc_handle_bytes": (_sz, []),
    "cmb_ipc_get_handle": (_i, [_p, _p]),
    "cmb_ipc_open": (_i, [_p, _p]),
    "cmb_ipc_close": (_i, [_p]),
    "cmb_p2p_enable_peer": (_i, [_i]),
    "cmb_p2p_scatter_store": (_i, [_p, _p, _p, _i, _i, _p]),
    "cmb_p2p_scatter_store_tuned": (_i, [_p, _p, _p, _i, _i, _i, _p]),
    "cmb_p2p_scatter_bulk": (_i, [_p, _p, _p, _i, _i, _p, _p]),
    "cmb_p2p_scatter_bulk_tuned": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p]),
    "cmb_p2p_scatter_copy_engine": (_i, [_p, _p, _p, _i, _p]),
    "cmb_p2p_scatter_copy_engine_tuned": (_i, [_p, _p, _p, _i, _i, _p]),
    "cmb_p2p_scatter_hybrid": (_i, [_p, _p, _p, _i, _i, _i, _p]),
    "cmb_selftest_wait_timeout": (_i, [_u64, _p, _p, _p]),
    "cmb_compare_bytes": (_i, [_p, _p, _sz, _p, _p]),
    "cmb_benchmark_global_memory": (_i, []),
    "cmb_benchmark_cache": (_i, []),
    "cmb_benchmark_tma": (_i, []),
    "cmb_benchmark_tensor_core": (_i, []),
    "cmb_benchmark_tensor_core_extended": (_i, []),
    "cmb_benchmark_multi_gpu": (_i, []),
    "cmb_benchmark_memory_more": (_i, []),
    "cmb_benchmark_pcie": (_i, []),
    "cmb_results_log_report_placeholders": (_i, []),
    "cmb_report_key_count": (ctypes.c_size_t, []),
    "cmb_report_key": (_i, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_char_p),
                            ctypes.POINTER(ctypes.c_char_p)]),
    "cmb_run_cli": (_i, [_i, _p, _s]),
    "cmb_results_set_device": (_i, [_s, _s, _i, _i, _i, _i]),
    "cmb_results_log": (_i, [_s, _s, _d, _s]),
    "cmb_results_write_json": (_i, [_s]),
    "cmb_results_clear": (_i, []),
    "cmb_results_set_sink": (_i, [_p, _p, _p]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class CmbError(RuntimeError):
    """A cmb_* call returned a non-zero cmb_status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        name = lib.cmb_status_string(status).decode()
        detail = lib.cmb_last_error().decode()
        super().__init__(f"{fn} -> {name}: {detail}")


def check(fn: str, *args) -> int:
    """Calls lib.<fn>(*args) and raises CmbError on a non-zero status."""
    rc = getattr(lib, fn)(*args)
    if rc != 0:
        raise CmbError(fn, rc)
    return rc


def sm_die_map(stream=None):
    """Measures the die of every SM of the current device (cmb_sm_die_map).
    Returns (labels, near_cycles, far_cycles): labels[id] is 0 or 1 for each
    SM id, 0xFF for ids without an SM (a uint8 numpy array)."""
    import numpy as np

    labels = np.full(256, 0xFF, np.uint8)
    n_ids = ctypes.c_int(0)
    near_far = (ctypes.c_float * 2)()
    check("cmb_sm_die_map", ctypes.c_void_p(labels.ctypes.data), len(labels), ctypes.byref(n_ids),
          near_far, stream)
    return labels[:n_ids.value].copy(), float(near_far[0]), float(near_far[1])


def set_sm_die_map(labels):
    """Installs `labels` (as sm_die_map returns them) for the GEMMs on the
    current device; None removes the map (cmb_gemm_set_sm_die_map)."""
    import numpy as np

    if labels is None:
        check("cmb_gemm_set_sm_die_map", None, 0)
        return
    a = np.ascontiguousarray(labels, dtype=np.uint8)
    check("cmb_gemm_set_sm_die_map", ctypes.c_void_p(a.ctypes.data), len(a))
