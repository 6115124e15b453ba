"""GPU test: the copy and sum entry points can be captured into a CUDA graph
(torch.cuda.graph on the caller's stream) and replayed, with the same
bit-exact copy and the same sum as direct calls."""

import ctypes

import pytest

from tests.helpers import dptr

pytestmark = pytest.mark.gpu


def test_copy_and_sum_replay_from_a_graph(cuda, cmb):
    n = (1 << 26) + 5
    src = cuda.empty(n, dtype=cuda.float32, device="cuda")
    dst = cuda.zeros(n, dtype=cuda.float32, device="cuda")
    ws_bytes = cmb.lib.cmb_stream_sum_workspace_bytes(n)
    ws = cuda.empty(ws_bytes, dtype=cuda.uint8, device="cuda")
    out = cuda.zeros(1, dtype=cuda.float64, device="cuda")
    direct = cuda.zeros(1, dtype=cuda.float64, device="cuda")
    s = cuda.cuda.Stream()
    h = ctypes.c_void_p(s.cuda_stream)
    with cuda.cuda.stream(s):
        cmb.check("cmb_fill_uniform_f32", dptr(src), n, ctypes.c_uint64(17), h)
        cmb.check("cmb_stream_sum_f32", dptr(src), n, dptr(direct), dptr(ws), ws_bytes, h)
    s.synchronize()
    g = cuda.cuda.CUDAGraph()
    with cuda.cuda.graph(g, stream=s):
        hc = ctypes.c_void_p(cuda.cuda.current_stream().cuda_stream)
        cmb.check("cmb_stream_copy", dptr(dst), dptr(src), 4 * n, hc)
        cmb.check("cmb_stream_sum_f32", dptr(dst), n, dptr(out), dptr(ws), ws_bytes, hc)
    for _ in range(3):
        dst.zero_()
        out.zero_()
        g.replay()
        cuda.cuda.synchronize()
        assert cuda.equal(src.view(cuda.int32), dst.view(cuda.int32))
        assert float(out.item()) == float(direct.item())
