"""CPU tests of the multi-GPU host logic: the ring and all-to-all plans move
every byte exactly once (simulated with N ranks as host buffers), and the
rank plumbing bench.py uses (barrier, max/sum reductions, handle exchange)
works across two gloo processes."""

import os
import socket

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from cuda_micro_bench_b200 import multi_gpu


def _simulate(mode, world, nbytes):
    rng = np.random.default_rng(world)
    send = [rng.integers(0, 256, nbytes, dtype=np.uint8) for _ in range(world)]
    recv = [np.zeros(nbytes, np.uint8) for _ in range(world)]
    written = [np.zeros(nbytes, np.int32) for _ in range(world)]
    for r in range(world):
        for j in multi_gpu.plan(mode, r, world, nbytes):
            recv[j.dst_rank][j.dst_off:j.dst_off + j.nbytes] = send[r][j.src_off:j.src_off + j.nbytes]
            written[j.dst_rank][j.dst_off:j.dst_off + j.nbytes] += 1
    return send, recv, written


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("mode", ["ring", "alltoall"])
def test_plans_deliver_every_byte_once(mode, world):
    nbytes = 16 * world * 64
    send, recv, written = _simulate(mode, world, nbytes)
    for r in range(world):
        assert np.all(written[r] == 1)  # every receive byte written exactly once
        for s in multi_gpu.sources(mode, r, world, nbytes):
            got = recv[r][s.recv_off:s.recv_off + s.nbytes]
            assert np.array_equal(got, send[s.src_rank][s.src_off:s.src_off + s.nbytes])


@settings(max_examples=60, deadline=None)
@given(st.sampled_from(["ring", "alltoall"]), st.integers(min_value=1, max_value=8),
       st.integers(min_value=1, max_value=64))
def test_plans_any_world_and_size(mode, world, units):
    """Every receive byte written once, from the byte the plan names, for
    any world size and any size the plan accepts (16-byte chunks)."""
    nbytes = 16 * world * units
    send, recv, written = _simulate(mode, world, nbytes)
    total_egress = 0
    for r in range(world):
        assert np.all(written[r] == 1)
        for s in multi_gpu.sources(mode, r, world, nbytes):
            assert np.array_equal(recv[r][s.recv_off:s.recv_off + s.nbytes],
                                  send[s.src_rank][s.src_off:s.src_off + s.nbytes])
        total_egress += multi_gpu.egress_bytes(mode, r, world, nbytes)
    # bytes that cross between GPUs: all of them on a ring of 2+, (N-1)/N of them all-to-all
    expect = (world * nbytes if world > 1 else 0) if mode == "ring" else (world - 1) * nbytes
    assert total_egress == expect


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_alltoall_plan_is_staggered(world):
    """At every position of the job lists, each rank is the destination of
    exactly one sender, and every rank's own chunk comes last."""
    nbytes = 16 * world * 8
    plans = [multi_gpu.plan("alltoall", r, world, nbytes) for r in range(world)]
    for k in range(world):
        assert sorted(p[k].dst_rank for p in plans) == list(range(world))
    assert all(p[-1].dst_rank == r for r, p in enumerate(plans))


def test_egress_bytes():
    n = 1 << 28
    for world in (2, 4, 8):
        assert multi_gpu.egress_bytes("ring", 0, world, n) == n
        assert multi_gpu.egress_bytes("alltoall", 1, world, n) == n * (world - 1) // world
    with pytest.raises(ValueError):
        multi_gpu.chunk_bytes(3, 100)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import bench

    ranks = bench.Ranks("gloo")
    ranks.barrier()
    mx = ranks.max(float(rank + 1))
    sm = ranks.sum(float(rank + 1))
    handles = [None] * world
    ranks.dist.all_gather_object(handles, bytes([rank]) * 64)
    ranks.close()
    q.put((rank, mx, sm, [h[0] for h in handles]))


def test_rank_plumbing_two_gloo_processes():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, mx, sm, hs in res:
        assert mx == 2.0 and sm == 3.0 and hs == [0, 1]


def _dropper(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import time

    import bench

    ranks = bench.Ranks("gloo", timeout_s=5.0)
    ranks.barrier()
    if rank == 1:
        q.put((rank, "left"))
        return  # leaves between steps, without its next collective
    t0 = time.time()
    try:
        ranks.max(1.0)
        q.put((rank, "no error"))
    except Exception as e:  # the collective fails instead of hanging
        q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def test_peer_that_leaves_is_detected_by_timeout():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropper, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]


def test_hybrid_method_names():
    assert multi_gpu.parse_hybrid("hybrid_500_1") == (500, 1)
    assert multi_gpu.parse_hybrid("hybrid_0_8") == (0, 8)
    assert multi_gpu.parse_hybrid("hybrid_1000_2") == (1000, 2)
    for bad in ("hybrid_1001_1", "hybrid_500_0", "hybrid_500_9", "hybrid_500", "store_1_1"):
        with pytest.raises(ValueError):
            multi_gpu.parse_hybrid(bad)
