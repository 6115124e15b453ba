"""GPU tests of the NVLink probe: the scatter kernels and copy-engine
scatter are bit-exact (local destinations on one GPU); with two or more GPUs
the CLI's --p2p section and a two-process IPC exchange deliver every byte."""

import ctypes
import json
import os
import socket
import subprocess

import pytest

from tests.helpers import dptr, stream_handle

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "cuda_micro_bench_b200", "bin", "cmb_b200")


def _local_jobs(cuda, sizes):
    src = [cuda.randint(0, 255, (s,), dtype=cuda.uint8, device="cuda") for s in sizes]
    dst = [cuda.zeros(s + 64, dtype=cuda.uint8, device="cuda") for s in sizes]
    n = len(sizes)
    d = (ctypes.c_void_p * n)(*[t.data_ptr() for t in dst])
    s_ = (ctypes.c_void_p * n)(*[t.data_ptr() for t in src])
    nb = (ctypes.c_size_t * n)(*sizes)
    return src, dst, d, s_, nb


def _check_jobs(cuda, src, dst, sizes):
    for a, b, sz in zip(src, dst, sizes):
        assert cuda.equal(a, b[:sz])
        assert int(b[sz:].count_nonzero()) == 0


@pytest.mark.parametrize("method", ["store", "bulk", "copy_engine"])
@pytest.mark.parametrize("sizes", [[1 << 20], [4096 + 48, 7 << 16, 16], [5 << 20] * 8,
                                   [(32 << 10) * 149 + 13, 0, 15, 1 << 16]])
def test_scatter_local_bit_exact(cuda, cmb, method, sizes):
    n = len(sizes)
    src, dst, d, s_, nb = _local_jobs(cuda, sizes)
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    if method == "store":
        cmb.check("cmb_p2p_scatter_store", d, s_, nb, n, 0, stream_handle(cuda))
    elif method == "bulk":
        cmb.check("cmb_p2p_scatter_bulk", d, s_, nb, n, 0, dptr(status), stream_handle(cuda))
    else:
        cmb.check("cmb_p2p_scatter_copy_engine", d, s_, nb, n, stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    _check_jobs(cuda, src, dst, sizes)


@pytest.mark.parametrize("permille,streams", [(0, 1), (1, 1), (500, 1), (700, 2), (999, 3),
                                              (1000, 1)])
@pytest.mark.parametrize("sizes", [[1 << 20], [4096 + 48, 7 << 16, 16], [5 << 20] * 8,
                                   [(32 << 10) * 149 + 13, 0, 15, 1 << 16]])
def test_scatter_hybrid_local_bit_exact(cuda, cmb, permille, streams, sizes):
    """Copy-engine heads and peer-store tails of every job meet exactly,
    from all-peer-stores (0) to all-copy-engine (1000), on ragged sizes."""
    n = len(sizes)
    src, dst, d, s_, nb = _local_jobs(cuda, sizes)
    cmb.check("cmb_p2p_scatter_hybrid", d, s_, nb, n, permille, streams, stream_handle(cuda))
    cuda.cuda.synchronize()
    _check_jobs(cuda, src, dst, sizes)


def test_scatter_hybrid_rejects_bad_args(cuda, cmb):
    t = cuda.zeros(1 << 16, dtype=cuda.uint8, device="cuda")
    one = lambda off: (ctypes.c_void_p * 1)(t.data_ptr() + off)
    nb = (ctypes.c_size_t * 1)(4096)
    s = stream_handle(cuda)
    assert cmb.lib.cmb_p2p_scatter_hybrid(one(0), one(4096), nb, 1, 1001, 1, s) == 1
    assert cmb.lib.cmb_p2p_scatter_hybrid(one(0), one(4096), nb, 1, -1, 1, s) == 1
    assert cmb.lib.cmb_p2p_scatter_hybrid(one(0), one(4096), nb, 1, 500, 0, s) == 1
    assert cmb.lib.cmb_p2p_scatter_hybrid(one(0), one(4096), nb, 1, 500, 9, s) == 1
    assert cmb.lib.cmb_p2p_scatter_hybrid(one(8), one(0), nb, 1, 500, 1, s) == 1  # alignment
    assert cmb.lib.cmb_p2p_scatter_hybrid(one(0), one(4096), nb, 9, 500, 1, s) == 1  # > 8 jobs


@pytest.mark.parametrize("chunk,stages,ctas", [(16, 4, 3), (4096, 8, 0), (56 << 10, 4, 1),
                                               (16 << 10, 8, 200), (32 << 10, 4, 0)])
def test_scatter_bulk_shapes(cuda, cmb, chunk, stages, ctas):
    """Ring depths, chunk sizes from one 16-byte line to 64 KiB, more CTAs
    than chunks, one CTA walking every chunk, ragged tails."""
    sizes = [(3 << 20) + 16 * 7 + 5, 4096, 17, (1 << 20) + 32]
    n = len(sizes)
    src, dst, d, s_, nb = _local_jobs(cuda, sizes)
    status = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    cmb.check("cmb_p2p_scatter_bulk_tuned", d, s_, nb, n, ctas, chunk, stages, dptr(status),
              stream_handle(cuda))
    cuda.cuda.synchronize()
    assert int(status.item()) == 0
    _check_jobs(cuda, src, dst, sizes)


def test_scatter_bulk_rejects_bad_args(cuda, cmb):
    t = cuda.zeros(1 << 16, dtype=cuda.uint8, device="cuda")
    one = lambda off: (ctypes.c_void_p * 1)(t.data_ptr() + off)
    nb = (ctypes.c_size_t * 1)(4096)
    s = stream_handle(cuda)
    assert cmb.lib.cmb_p2p_scatter_bulk(one(8), one(0), nb, 1, 0, None, s) == 1  # alignment
    assert cmb.lib.cmb_p2p_scatter_bulk_tuned(one(0), one(4096), nb, 1, 0, 24, 4, None, s) == 1
    assert cmb.lib.cmb_p2p_scatter_bulk_tuned(one(0), one(4096), nb, 1, 0, 4096, 6, None, s) == 1
    assert cmb.lib.cmb_p2p_scatter_bulk_tuned(one(0), one(4096), nb, 1, 0, 65536, 8, None, s) == 1
    assert cmb.lib.cmb_p2p_scatter_bulk(one(0), one(4096), nb, 9, 0, None, s) == 1  # > 8 jobs


def test_cli_p2p_section(cuda, tmp_path):
    out = tmp_path / "r.json"
    p = subprocess.run([EXE, "--p2p", f"--out={out}"], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout + p.stderr
    res = json.loads(out.read_text())["results"]
    count = cuda.cuda.device_count()
    assert res["pcie"]["device_count"]["value"] == count
    if count >= 2:
        for k in ("ring_store", "ring_bulk", "ring_copy_engine", "alltoall_store",
                  "alltoall_bulk", "alltoall_copy_engine"):
            assert res["p2p"][k + "_verified"]["value"] == 1.0
            assert res["p2p"][k + "_link_gbps"]["value"] > 10.0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


ALL_METHODS = ("store", "bulk", "copy_engine", "copy_engine_1stream", "copy_engine_2stream",
               "hybrid_500_1", "hybrid_300_2")


def _rank(rank, world, port, q, device=None, backend="nccl"):
    device = rank if device is None else device
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(device),
                       "NCCL_NVLS_ENABLE": "0"})
    import torch

    torch.cuda.set_device(device)
    import bench
    from cuda_micro_bench_b200 import multi_gpu

    ranks = bench.Ranks(backend)
    ex = multi_gpu.PeerExchange(ranks, 16 << 20, 77)
    bad = {}
    sh = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for mode in ("ring", "alltoall"):
        for method in ALL_METHODS:
            ranks.barrier()
            ex.launch(mode, method, sh)
            torch.cuda.synchronize()
            ranks.barrier()
            bad[(mode, method)] = ex.mismatches(mode, sh)
    ex.close()
    ranks.close()
    q.put((rank, bad))


def test_two_process_ipc_exchange(cuda):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, bad in res:
        assert all(v == 0 for v in bad.values()), (rank, bad)


def test_two_process_ipc_exchange_on_one_gpu(cuda):
    """The same two-rank exchange with both ranks on GPU 0 (gloo for the
    host side): every receive buffer is another process's CUDA IPC mapping,
    written by the peer-store and bulk-copy kernels and the copy engines
    exactly as across NVLink, and checked bit for bit.  The kernels never wait
    on each other; the host barriers order the steps."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, 0, "gloo")) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, bad in res:
        assert len(bad) == 2 * len(ALL_METHODS)
        assert all(v == 0 for v in bad.values()), (rank, bad)
