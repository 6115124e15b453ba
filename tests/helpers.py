"""Shared helpers for the tests: device buffers via torch, calls via ctypes."""

import ctypes

import numpy as np


def stream_handle(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def to_numpy(t):
    return t.detach().cpu().numpy()


def hptr(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)
